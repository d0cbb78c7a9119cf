"""The text conditioning on a B200: the Qwen3 text encoder and the LLM adapter against the
reference's own qwen3 / llm_adapter (tests/golden/text_1024.npz: 28-layer INT8 ConvRot Qwen3, the
6-block bf16 adapter, 77 Qwen3 and 60 T5 tokens), and the attention kernel of the text path
(causal, grouped k/v heads, head_dim 64) against the numpy oracle.

Tolerances (relative L2): the text-path attention on fp32 inputs 1e-5 (fp32 math, exp2 with the
hardware's approximation), on 16-bit inputs at head_dim 128 (the tcgen05 kernel, probabilities in
the same 16-bit type) 1e-3 (fp16) / 8e-3 (bf16); the adapter alone (bf16 weights, fp32 math) 1e-4;
Qwen3, whose linears take two-plane int8 activations as the DiT's do and whose attention runs on
fp16 q/k/v, and the full chain 3e-3, the north star's end-to-end bar."""

import os

import numpy as np
import pytest
import torch

from oracle import text_np
from tests._util import rel_l2
from tests.conftest import GOLDEN, pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


# head_dim 128 with 16-bit q/k/v runs on the tcgen05 flash kernel (P in the inputs' 16-bit type:
# rel. L2 ~5e-4 fp16, ~4e-3 bf16); fp32 inputs and head_dim 64 on the CUDA-core kernel (fp32, 1e-5)
TOL = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}


@pytest.mark.parametrize("Lq,Lk,H,group,D,causal,dtype", [
    (77, 77, 16, 2, 128, True, torch.float32),     # Qwen3 self-attention, fp32
    (77, 77, 16, 2, 128, True, torch.float16),     # Qwen3 self-attention as the encoder runs it
    (512, 512, 16, 2, 128, True, torch.float16),   # a 512-token prompt: two query-tile pairs
    (300, 300, 16, 2, 128, True, torch.bfloat16),  # longer prompt, bf16 inputs
    (300, 300, 8, 1, 128, False, torch.float16),   # non-causal, one k/v head per q head
    (60, 77, 16, 1, 64, False, torch.float32),     # adapter cross-attention
    (33, 33, 4, 4, 64, True, torch.float16),       # odd sizes, one k/v head per four q heads
])
def test_text_attention_matches_oracle(Lq, Lk, H, group, D, causal, dtype):
    ops = pkg("ops")
    KH = H // group
    q, k, v = _rand((Lq, H * D), 1, dtype), _rand((Lk, KH * D), 2, dtype), _rand((Lk, KH * D), 3, dtype)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=Lq, Lk=Lk, H=H, D=D, group=group, causal=causal,
                        out_dtype=torch.float32).cpu().numpy()
    qh = q.float().numpy().reshape(Lq, H, D).transpose(1, 0, 2)
    kh = np.repeat(k.float().numpy().reshape(Lk, KH, D).transpose(1, 0, 2), group, 0)
    vh = np.repeat(v.float().numpy().reshape(Lk, KH, D).transpose(1, 0, 2), group, 0)
    ref = text_np.attention(qh, kh, vh, causal=causal).transpose(1, 0, 2).reshape(Lq, H * D)
    assert rel_l2(out, ref) < (TOL[dtype] if D == 128 else 1e-5)


def test_text_attention_key_len_and_batch():
    """Batch of 2 with per-item key lengths (one item fully masked gives zeros)."""
    ops = pkg("ops")
    L, H, D = 50, 16, 64
    q, k, v = _rand((2 * L, H * D), 4), _rand((2 * L, H * D), 5), _rand((2 * L, H * D), 6)
    kl = torch.tensor([31, 0], dtype=torch.int32, device=DEV)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=L, Lk=L, H=H, D=D, batch=2, q_bstride=L * H * D,
                        k_bstride=L * H * D, v_bstride=L * H * D, key_len=kl, out_dtype=torch.float32).cpu().numpy()
    qh = q[:L].numpy().reshape(L, H, D).transpose(1, 0, 2)
    kh = k[:31].numpy().reshape(31, H, D).transpose(1, 0, 2)
    vh = v[:31].numpy().reshape(31, H, D).transpose(1, 0, 2)
    ref = text_np.attention(qh, kh, vh).transpose(1, 0, 2).reshape(L, H * D)
    assert rel_l2(out[:L], ref) < 1e-5
    assert not out[L:].any()


@pytest.fixture(scope="module")
def fixture():
    g = dict(np.load(os.path.join(GOLDEN, "text_1024.npz")))
    syn = pkg("synthetic")
    seed, vocab = int(g["seed"]), int(g["vocab"])
    return g, syn.te_tensors(seed, 28, vocab, direct=True), syn.adapter_tensors(seed, 6, vocab)


def test_qwen3_matches_reference(fixture):
    g, te, _ = fixture
    model = pkg("text").Qwen3(te, DEV)
    hs = model.encode(g["qwen_ids"]).cpu().numpy()
    err = rel_l2(hs, g["hidden"])
    print(f"qwen3 (28 layers, int8): rel L2 {err:.2e}")
    assert err < 3e-3


def test_llm_adapter_matches_reference(fixture):
    g, te, ad = fixture
    text = pkg("text")
    adapter = text.LLMAdapter(ad, DEV)
    ctx = adapter(torch.from_numpy(g["hidden"]).to(DEV), g["t5_ids"]).cpu().numpy()
    assert ctx.shape == (512, 1024) and not ctx[60:].any()
    err = rel_l2(ctx[:60], g["ctx60"])
    # and the whole chain: token ids -> DiT context
    ctx2 = adapter(text.Qwen3(te, DEV).encode(g["qwen_ids"]), g["t5_ids"]).cpu().numpy()
    err2 = rel_l2(ctx2[:60], g["ctx60"])
    print(f"adapter alone: rel L2 {err:.2e}; qwen3 + adapter: {err2:.2e}")
    assert err < 1e-4 and err2 < 3e-3
    # per-token T5 weights scale the rows (tools/reference.py:165-166)
    w = np.linspace(0.5, 1.5, 60).astype(np.float32)
    ctx3 = adapter(torch.from_numpy(g["hidden"]).to(DEV), g["t5_ids"], t5_weights=w).cpu().numpy()
    np.testing.assert_allclose(ctx3[:60], ctx[:60] * w[:, None], rtol=1e-6, atol=1e-7)
