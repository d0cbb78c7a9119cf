"""The numpy oracle against the golden fixtures made by the reference's own code."""

import os
import time

import numpy as np
import pytest
import torch

import oracle
from tests._util import rel_l2, to_np
from tests.conftest import GOLDEN, pkg


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def test_int8_dequant_matches_reference():
    g = load("quant_int8.npz")
    t = {k: g[k] for k in ("weight", "weight_scale", "comfy_quant")}
    assert rel_l2(oracle.dequantize(t), g["deq"]) < 1e-6


@pytest.mark.parametrize("case", ["w4_gauss", "w4_fit"])
def test_w4_grid_bit_exact(case):
    g = load(f"quant_{case}.npz")
    grid = oracle.decode_w4_grid(g["weight"], g["weight_s_rel"], g["weight_codebook"])
    np.testing.assert_array_equal(grid, g["grid"])
    assert np.abs(grid).max() <= 127
    t = {k: g[k] for k in ("weight", "weight_s_rel", "weight_s_channel", "weight_codebook", "comfy_quant")}
    assert rel_l2(oracle.dequantize(t), g["deq"]) < 1e-6


def test_w4_fit_case_uses_fitted_codebook():
    g = load("quant_w4_fit.npz")
    assert not np.allclose(g["weight_codebook"], oracle.FIXED_LUT)
    g2 = load("quant_w4_gauss.npz")
    np.testing.assert_array_equal(g2["weight_codebook"], oracle.FIXED_LUT)


def test_fp8_table_matches_torch():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(oracle.fp8_e4m3fn_table(), ref)


def test_rope_tables():
    g = load("rope.npz")
    for H, W in ((8, 8), (16, 12), (64, 64)):
        c, s = oracle.dit_rope(H, W)
        np.testing.assert_allclose(c, g[f"cos_{H}x{W}"], atol=2e-6)
        np.testing.assert_allclose(s, g[f"sin_{H}x{W}"], atol=2e-6)


def test_sigma_schedules():
    g = load("sigmas.npz")
    for n in (1, 2, 8, 30):
        np.testing.assert_array_equal(np.array(oracle.sigmas_simple(n, 3.0)), g[f"simple_{n}"])


def test_block0_matches_reference():
    g = load("block0_L64.npz")
    seed = int(g["seed"])
    syn = pkg("synthetic")
    t = to_np(syn.global_tensors(seed))
    t.update(to_np(syn.block_tensors(seed, 0, "int8", 28)))
    W = oracle.DequantWeights(t)
    temb, adaln_lora, emb = oracle.time_cond(W, float(g["sigma"]))
    assert rel_l2(temb, g["temb"]) < 1e-6
    assert rel_l2(adaln_lora, g["adaln_lora"]) < 1e-5
    assert rel_l2(emb, g["emb"]) < 1e-6
    cos, sin = oracle.dit_rope(8, 8)
    cos, sin = np.concatenate([cos, cos], -1), np.concatenate([sin, sin], -1)
    ctx = np.concatenate([g["ctx256"], np.zeros_like(g["ctx256"])], 0)
    out = oracle.dit_block(W, 0, g["x"], ctx, emb, adaln_lora, cos, sin)
    assert rel_l2(out, g["out"]) < 1e-5


@pytest.mark.parametrize("fmt", ["int8", "mixed"])
def test_full_forward_and_euler_match_reference(fmt):
    """28 blocks + 2 Euler steps at a 16x16 latent against tools/reference.py's own dit_forward."""
    g = load(f"forward_{fmt}_16x16.npz")
    seed = int(g["seed"])
    syn = pkg("synthetic")
    t0 = time.time()

    class LazyBlocks:
        """Builds one block's tensors at a time, like the reference reading its checkpoint."""

        def __init__(self):
            self.glob = to_np(syn.global_tensors(seed))
            self.i = None
            self.W = None

        def __call__(self, name):
            if name.startswith("blocks."):
                i = int(name.split(".")[1])
                if i != self.i:
                    self.i = i
                    self.W = oracle.DequantWeights(to_np(syn.block_tensors(seed, i, fmt, 28, direct=True)))
                return self.W(name)
            return oracle.DequantWeights(self.glob)(name)

    W = LazyBlocks()
    ctx = np.concatenate([to_np({"c": syn.randn(seed, "golden.ctx", (256, 1024))})["c"], np.zeros((256, 1024), np.float32)])
    dump = {}
    steps = 2 if fmt == "int8" else 1
    lat = oracle.euler_sample(W, g["noise"], ctx, steps, dump=dump)
    for k in ("dit_x_embed", "dit_emb", "dit_adaln_lora", "dit_block0"):
        assert rel_l2(dump[k], g[k]) < 1e-5, k
    assert rel_l2(dump["velocity0"], g["velocity0"]) < 1e-4
    assert rel_l2(dump["denoised0"], g["denoised0"]) < 1e-4
    if steps == 2:
        assert rel_l2(lat, g["latent_final"]) < 1e-4
    print(f"oracle forward {fmt}: {time.time() - t0:.1f}s")


def test_beta_scheduler_matches_reference_algorithm():
    """pipeline.sigmas_beta (scipy's Beta quantile) against the reference's own bisection of its
    continued-fraction Beta CDF (app/samplers.js:24-93, restated in oracle/samplers_np.py)."""
    from oracle import samplers_np
    from tests.conftest import pkg
    pl = pkg("pipeline")
    for steps in (1, 3, 4, 8, 12, 20, 30, 50):
        for shift in (1.0, 3.0, 6.0):
            assert pl.sigmas_beta(steps, shift) == samplers_np.sigmas_beta(steps, shift)


def test_text_oracle_matches_reference_fixture():
    """The numpy Qwen3 + LLM adapter (oracle/text_np.py) against tools/reference.py's qwen3 and
    llm_adapter on the same synthetic weights (tests/golden/text_1024.npz)."""
    from oracle import text_np

    g = load("text_1024.npz")
    seed, vocab = int(g["seed"]), int(g["vocab"])
    syn = pkg("synthetic")
    W = oracle.DequantWeights(oracle.to_numpy(syn.te_tensors(seed, 28, vocab, direct=True)))
    hs = text_np.qwen3(W, g["qwen_ids"])
    assert rel_l2(hs, g["hidden"]) < 1e-5
    Wa = oracle.DequantWeights(oracle.to_numpy(syn.adapter_tensors(seed, 6, vocab)))
    ctx = text_np.llm_adapter(Wa, g["hidden"], g["t5_ids"])
    assert rel_l2(ctx[:60], g["ctx60"]) < 1e-5 and not ctx[60:].any()


def test_vae_oracle_matches_reference_fixture():
    """The numpy Wan-2.1 decoder (oracle/vae_np.py) against tools/reference.py's vae_decode on the
    same synthetic decoder and latent (tests/golden/vae_64.npz)."""
    from oracle import vae_np

    g = load("vae_64.npz")
    syn = pkg("synthetic")
    W = oracle.DequantWeights(oracle.to_numpy(syn.vae_tensors(int(g["seed"]))))
    z = g["latent"] * np.array(syn.LATENT_STD, np.float32)[:, None, None] + \
        np.array(syn.LATENT_MEAN, np.float32)[:, None, None]
    assert rel_l2(vae_np.vae_decode(W, z), g["image"]) < 1e-5
