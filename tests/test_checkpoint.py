"""CPU tests of the on-disk checkpoint path (app/weights.js:29-146, lora.js:103-134): the
safetensors reader and writer, comfy_quant layouts read back bit for bit, files of the
safetensors package read by ours and ours by it, malformed files rejected, and a LoRA file
matched to the model's linears."""

import json
import os
import struct

import numpy as np
import pytest
import torch

from tests.conftest import pkg


def _synthetic(n_blocks=3):
    syn = pkg("synthetic")
    t = syn.global_tensors(7)
    for i in range(n_blocks):
        t.update(syn.block_tensors(7, i, "mixed", n_blocks, direct=True))
    return t


def test_round_trip_keeps_every_tensor_bit_for_bit(tmp_path):
    ck = pkg("checkpoint")
    t = _synthetic()
    t["scalar_alpha"] = torch.tensor(16.0)
    t["empty"] = torch.empty(0, 4)
    path = str(tmp_path / "m.safetensors")
    ck.save_file(path, {"model.diffusion_model." + k: v for k, v in t.items()}, {"format": "pt"})
    with ck.SafeTensors(path, "model.diffusion_model.") as st:
        assert sorted(st.keys()) == sorted(t)
        assert st.metadata == {"format": "pt"}
        for k, v in t.items():
            got = st.tensor(k)
            assert got.dtype == v.dtype and got.shape == v.shape, k
            assert torch.equal(got.view(torch.uint8) if got.dtype == torch.float8_e4m3fn else got,
                               v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v), k
        assert st.f32("scalar_alpha").item() == 16.0
        # comfy_quant metadata survives as the JSON bytes the quantizers write
        meta = pkg("quant").meta_of(st.mapping(), "blocks.1.mlp.layer1.")
        assert meta["format"] == "asym_w4a8_int8" and meta["convrot"]


def test_interoperates_with_the_safetensors_package(tmp_path):
    safetensors_torch = pytest.importorskip("safetensors.torch")
    from safetensors import safe_open

    ck = pkg("checkpoint")
    t = {k: v for k, v in _synthetic(2).items()}
    theirs, ours = str(tmp_path / "theirs.safetensors"), str(tmp_path / "ours.safetensors")
    safetensors_torch.save_file({k: v.contiguous() for k, v in t.items()}, theirs)
    ck.save_file(ours, t)
    with ck.SafeTensors(theirs) as st:
        for k, v in t.items():
            assert torch.equal(st.tensor(k).view(torch.uint8), v.contiguous().view(torch.uint8)), k
    with safe_open(ours, "pt") as f:
        assert sorted(f.keys()) == sorted(t)
        for k, v in t.items():
            assert torch.equal(f.get_tensor(k).view(torch.uint8), v.contiguous().view(torch.uint8)), k


def test_malformed_files_are_rejected(tmp_path):
    ck = pkg("checkpoint")
    good = str(tmp_path / "g.safetensors")
    ck.save_file(good, {"a": torch.arange(10, dtype=torch.float32)})
    raw = open(good, "rb").read()
    cases = {
        "short": raw[:5],
        "header_overruns": struct.pack("<Q", len(raw)) + raw[8:],
        "not_json": struct.pack("<Q", 4) + b"{{{{" + raw[8:],
        "truncated_data": raw[:-8],
    }
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    hdr["a"]["dtype"] = "Q7"
    h = json.dumps(hdr).encode()
    cases["bad_dtype"] = struct.pack("<Q", len(h)) + h + raw[8 + n:]
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.safetensors")
        open(p, "wb").write(data)
        with pytest.raises(ValueError):
            ck.SafeTensors(p)
    with ck.SafeTensors(good) as st, pytest.raises(KeyError):
        st.tensor("b")


def test_dit_and_lora_load_from_files(tmp_path):
    """AnimaDiT's weight objects from a file equal those from the in-memory dict (CPU tensors),
    and a PEFT LoRA file matches every targeted linear."""
    ck, ditm, lora, syn = pkg("checkpoint"), pkg("dit"), pkg("lora"), pkg("synthetic")
    t = _synthetic(2)
    path = str(tmp_path / "dit.safetensors")
    ck.save_file(path, {"model.diffusion_model." + k: v for k, v in t.items()})
    lazy = ck.open_dit(path)
    a = ditm.AnimaDiT(lazy, "cpu", n_blocks=2)
    b = ditm.AnimaDiT(t, "cpu", n_blocks=2)
    for ba, bb in zip(a.blocks, b.blocks):
        for k in ("qkv", "self_o", "l1", "l2"):
            assert ba[k].kind == bb[k].kind and torch.equal(ba[k].data, bb[k].data) and torch.equal(ba[k].scale, bb[k].scale)
    targets = ("self_attn.q_proj", "mlp.layer1")
    lt = syn.lora_tensors(3, targets, rank=8, n_blocks=2, alpha=4.0)
    lpath = str(tmp_path / "lora.safetensors")
    ck.save_file(lpath, lt)
    with ck.SafeTensors(lpath) as st:
        L = lora.load_lora(st.mapping(), lora.linear_registry(a.blocks), device="cpu")
    assert L.matched == 4 and L.skipped == 0
    assert all(abs(m.alpha_scale - 0.5) < 1e-7 for m in L.modules)


@pytest.mark.gpu
def test_dit_from_file_runs_like_the_in_memory_model(tmp_path):
    ck, ditm, syn = pkg("checkpoint"), pkg("dit"), pkg("synthetic")
    t = _synthetic(3)
    path = str(tmp_path / "dit.safetensors")
    ck.save_file(path, {"model.diffusion_model." + k: v for k, v in t.items()})
    a = ditm.AnimaDiT.from_file(path, "cuda")
    b = ditm.AnimaDiT(t, "cuda")
    ctx = syn.randn(7, "ctx", (256, 1024)).cuda()
    x = syn.randn(7, "x", (1, 16, 32, 32)).cuda()
    va = a.forward(x, a.prepare_context(ctx), a.time_cond(0.7))
    vb = b.forward(x, b.prepare_context(ctx), b.time_cond(0.7))
    assert torch.equal(va, vb)
