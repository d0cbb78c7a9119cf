"""anima_attention_noalloc, the attention entry point for hosts that cannot call cudaMalloc (their
device memory belongs to another allocator, or they must not allocate once running): its stream-K
workspace is a static device array in the library instead of an allocation. On two calls in a row
with different inputs it must give exactly what anima_attention (context-owned workspace) gives.
Collected last, so it also runs after every other GPU test has used the library; it passes alone
as well."""

import numpy as np
import pytest
import torch

from tests.conftest import pkg

pytestmark = pytest.mark.gpu


def _qkv(seed, L):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(L, 6144, generator=g).to(torch.bfloat16).cuda()


def _attn(ops, qkv, L, noalloc, key_len=None):
    return ops.attention(qkv, qkv, qkv, Lq=L, Lk=L, H=16, ldq=6144, ldk=6144, ldv=6144, q_off=0, k_off=2048,
                         v_off=4096, key_len=key_len, out_dtype=torch.float32, noalloc=noalloc)


def test_noalloc_attention_matches_allocating_entry_point():
    ops, dev = pkg("ops"), pkg("device")
    ctx = dev.Context.get(0)
    ctx.set_attention_split(-1)  # 4096 tokens x 16 heads: stream-K, so the static workspace is used
    L = 4096
    for seed in (101, 102):  # two consecutive calls: flags left by the first must not leak
        qkv = _qkv(seed, L)
        ref = _attn(ops, qkv, L, False).cpu().numpy()
        got = _attn(ops, qkv, L, True).cpu().numpy()
        assert np.array_equal(got, ref), seed
    ctx.sync()


def test_noalloc_attention_whole_unit_schedule():
    """With a key mask no workspace is needed; the entry point still matches."""
    ops = pkg("ops")
    L = 1024
    kl = torch.tensor([700], dtype=torch.int32).cuda()
    for seed in (103, 104):
        qkv = _qkv(seed, L)
        ref = _attn(ops, qkv, L, False, kl).cpu().numpy()
        got = _attn(ops, qkv, L, True, kl).cpu().numpy()
        assert np.array_equal(got, ref), seed
