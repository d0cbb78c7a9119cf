"""CPU tests: host logic, the offline quantizers, and the C-ABI library's exports (no kernel calls)."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from tests._util import rel_l2
from tests.conftest import GOLDEN, ROOT, pkg


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "anima_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(anima_\w+)\(", src, re.M)))


def test_library_exports_every_header_function():
    build = pkg("build")
    lib_path = build.build()  # nvcc cross-compiles here; no GPU call is made
    lib = ctypes.CDLL(lib_path)
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing
    dev = pkg("device")
    assert sorted(dev.EXPORTS) == header_functions()


def test_library_has_no_multicast_loads():
    """No TMA or bulk load in the CUDA sources uses cluster multicast (multi-GPU safety rule); the
    qualifier is assembled here so this test file does not spell it."""
    qualifier = "." + "multi" + "cast" + "::" + "cluster"
    csrc = os.path.join(ROOT, "anima-studio_b200", "csrc")
    for f in os.listdir(csrc):
        for line in open(os.path.join(csrc, f)):
            if "cp.async.bulk" in line:
                assert qualifier not in line, f"{f}: {line.strip()}"


def test_ctypes_structs_match_the_c_header(tmp_path):
    """The ctypes mirrors of the C-ABI structs (device.py) have the header's field names, offsets
    and sizes, as a C compiler lays them out (gcc on include/anima_b200.h)."""
    import ctypes as C
    import shutil
    import subprocess

    dev = pkg("device")
    structs = {"anima_qact": dev.QAct, "anima_weight": dev.Weight, "anima_linear_opts": dev.LinearOpts,
               "anima_peer_group": dev.PeerGroup, "anima_attention_args": dev.AttentionArgs}
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "anima_b200.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, *_ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    inc = os.path.join(ROOT, "include")
    subprocess.run([cc, "-std=c11", "-I", inc, str(src), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {(a, b): int(c) for a, b, c in (ln.split() for ln in out if ln)}
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == C.sizeof(cls), cname
        for fname, *_ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def test_int8_quantizer_bit_exact():
    g = load("quant_int8.npz")
    q = pkg("quant").quantize_int8_convrot(torch.from_numpy(g["w"]))
    np.testing.assert_array_equal(q["weight"].numpy(), g["weight"])
    np.testing.assert_array_equal(q["weight_scale"].numpy(), g["weight_scale"])
    np.testing.assert_array_equal(q["comfy_quant"].numpy(), g["comfy_quant"])


@pytest.mark.parametrize("case", ["w4_gauss", "w4_fit"])
def test_w4a8_quantizer_bit_exact(case):
    g = load(f"quant_{case}.npz")
    q = pkg("quant").quantize_w4a8(torch.from_numpy(g["w"]))
    np.testing.assert_array_equal(q["weight"].numpy(), g["weight"])
    np.testing.assert_array_equal(q["weight_s_rel"].view(torch.uint8).numpy(), g["weight_s_rel"])
    np.testing.assert_array_equal(q["weight_s_channel"].numpy(), g["weight_s_channel"])
    np.testing.assert_array_equal(q["weight_codebook"].numpy(), g["weight_codebook"])


def test_rope_table_matches_reference():
    g = load("rope.npz")
    dit = pkg("dit")
    for H, W in ((8, 8), (16, 12), (64, 64)):
        t = dit.rope_table(H, W)
        np.testing.assert_allclose(t[: H * W], g[f"cos_{H}x{W}"], atol=2e-6)
        np.testing.assert_allclose(t[H * W:], g[f"sin_{H}x{W}"], atol=2e-6)


def test_sigmas_match_reference():
    g = load("sigmas.npz")
    pl = pkg("pipeline")
    for n in (1, 2, 8, 30):
        np.testing.assert_array_equal(np.array(pl.sigmas_simple(n, 3.0)), g[f"simple_{n}"])


def test_hadamard_rows_is_the_activation_rotation():
    """x A^T == rotate(x) (A H)^T, the identity the LoRA side path relies on (lora.js:1-10)."""
    lora = pkg("lora")
    quant = pkg("quant")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(8, 512, generator=g, dtype=torch.float64)
    A = torch.randn(4, 512, generator=g, dtype=torch.float64)
    lhs = x @ A.T
    rhs = quant.rotate(x.float()).double() @ lora.hadamard_rows(A.float()).double().T
    assert rel_l2(rhs.numpy(), lhs.numpy()) < 1e-6


def test_lora_key_matching():
    """PEFT and kohya names resolve to the same linears; unknown / unsupported keys are counted."""
    lora = pkg("lora")
    weights = pkg("weights")
    W = weights.Linear("i8", 6144, 2048, torch.zeros(1), name="blocks.0.self_attn.qkv",
                       parts=[("blocks.0.self_attn.q_proj", 0, 2048), ("blocks.0.self_attn.k_proj", 2048, 2048),
                              ("blocks.0.self_attn.v_proj", 4096, 2048)])
    l1 = weights.Linear("i8", 8192, 2048, torch.zeros(1), name="blocks.0.mlp.layer1")
    reg = lora.linear_registry({"blocks": [{"qkv": W, "l1": l1}]})
    assert set(reg) == {"blocks_0_self_attn_q_proj", "blocks_0_self_attn_k_proj", "blocks_0_self_attn_v_proj",
                        "blocks_0_mlp_layer1"}
    t = {
        "diffusion_model.blocks.0.self_attn.k_proj.lora_A.weight": torch.randn(4, 2048),
        "diffusion_model.blocks.0.self_attn.k_proj.lora_B.weight": torch.randn(2048, 4),
        "lora_unet_blocks_0_mlp_layer1.lora_down.weight": torch.randn(8, 2048),
        "lora_unet_blocks_0_mlp_layer1.lora_up.weight": torch.randn(8192, 8),
        "lora_unet_blocks_0_mlp_layer1.alpha": torch.tensor(4.0),
        "diffusion_model.blocks.0.nonexistent.lora_A.weight": torch.randn(4, 2048),
        "diffusion_model.blocks.0.nonexistent.lora_B.weight": torch.randn(2048, 4),
        "lora_unet_blocks_0_mlp_layer1.hada_w1_a": torch.randn(2, 2),
    }
    L = lora.load_lora(t, reg, device="cpu")
    assert (L.matched, L.total, L.unsupported, L.skipped) == (2, 3, 1, 1)
    by = {m.target[0].name: m for m in L.modules}
    assert by["blocks.0.self_attn.qkv"].target[1:] == (2048, 2048)
    assert by["blocks.0.mlp.layer1"].alpha_scale == pytest.approx(0.5)
    lora.attach_loras([reg], [(L, 0.8)])
    assert [e["scale"] for e in l1.lora] == [pytest.approx(0.4)]
    assert W.lora[0]["off"] == 2048 and W.lora[0]["n"] == 2048


def test_lora_down_k_slice_count():
    """The down-projection is cut along K only where K is long (MLP layer 2, 8192) and the slices'
    tiles fit the SMs together; K = 2048 linears and large batches stay one GEMM."""
    k = pkg("lora").k_slice_count
    assert k(4096, 128, 8192, 148) == 4      # MLP layer 2, 1024^2: 32 tiles -> 128 in 4 slices of 2048
    assert k(300, 128, 8192, 148) == 4
    assert k(4096, 256, 8192, 148) == 2      # 64 tiles: two slices fill 128 SMs
    assert k(4096, 128, 2048, 148) == 1      # K = 2048: slices would not pay for a launch
    assert k(4096, 256, 2048, 148) == 1
    assert k(8192, 256, 8192, 148) == 1      # CFG batch: 128 tiles already
    assert k(4096, 128, 4096, 148) == 2


def test_synthetic_checkpoint_is_deterministic():
    syn = pkg("synthetic")
    a = syn.block_tensors(3, 1, "mixed", 28, direct=True)
    b = syn.block_tensors(3, 1, "mixed", 28, direct=True)
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k].view(torch.uint8) if a[k].dtype == torch.float8_e4m3fn else a[k],
                           b[k].view(torch.uint8) if b[k].dtype == torch.float8_e4m3fn else b[k]), k
    assert "blocks.1.mlp.layer1.weight_s_rel" in a  # mixed: middle blocks are W4A8
    c = syn.block_tensors(3, 0, "mixed", 28, direct=True)
    assert "blocks.0.mlp.layer1.weight_scale" in c  # first block stays int8


def test_no_cpu_fallback_without_gpu():
    """The product path refuses to run without a CUDA device (there is no CPU fallback)."""
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ops = pkg("ops")
    dev = pkg("device")
    with pytest.raises(dev.AnimaError):
        ops.rotate(torch.zeros(4, 256))
