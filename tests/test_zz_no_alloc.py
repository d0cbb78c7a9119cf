"""anima_attention_noalloc, the attention entry point for hosts that cannot call cudaMalloc (their
device memory belongs to another allocator, or they must not allocate once running): its stream-K
workspace is a static device array in the library instead of an allocation. On two calls in a row
with different inputs it must give exactly what anima_attention (context-owned workspace) gives.

The first test runs in a fresh child process, so the no-alloc call is the first stream-K call of
its context (the context's workspace does not exist yet) and the device's free memory can be read
around it: the call must leave it unchanged, while the allocating entry point called afterwards
takes its workspace (the check can see an allocation). Collected last, so the in-process tests
also run after every other GPU test has used the library; they pass alone as well."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from tests.conftest import ROOT, pkg

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys
import torch
sys.path.insert(0, ROOT)
import importlib
ops = importlib.import_module("anima-studio_b200.ops")
dev = importlib.import_module("anima-studio_b200.device")

L = 4096
def qkv(seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(L, 6144, generator=g).to(torch.bfloat16).cuda()
def attn(x, out, noalloc, key_len=None):
    return ops.attention(x, x, x, Lq=L, Lk=L, H=16, ldq=6144, ldk=6144, ldv=6144, q_off=0, k_off=2048,
                         v_off=4096, key_len=key_len, out=out, noalloc=noalloc)

ctx = dev.Context.get(0)
ctx.set_attention_split(-1)          # 16 heads x 4096 tokens: the stream-K schedule
inputs = [qkv(201), qkv(202)]
outs = [torch.empty(L, 2048, dtype=torch.float32, device="cuda") for _ in range(4)]
kl = torch.tensor([3000], dtype=torch.int32, device="cuda")
# load the library's module (and with it the static array) and the attention kernel's code: a
# masked call takes the whole-unit schedule, which needs no workspace
attn(inputs[0], outs[0], True, kl)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for i in range(2):                  # two stream-K calls in a row through the static array
    attn(inputs[i], outs[i], True)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
ctx.sync()
for i in range(2):                  # the allocating entry point: allocates its workspace now
    attn(inputs[i], outs[2 + i], False)
torch.cuda.synchronize()
free2 = torch.cuda.mem_get_info()[0]
ctx.sync()
same = [bool(torch.equal(outs[i], outs[2 + i])) for i in range(2)]
finite = bool(torch.isfinite(outs[0]).all() and torch.isfinite(outs[1]).all())
print("RESULT " + json.dumps({"free0": free0, "free1": free1, "free2": free2, "same": same, "finite": finite}))
"""


def test_noalloc_first_call_allocates_nothing_fresh_process():
    code = "ROOT = " + repr(ROOT) + "\n" + CHILD
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=dict(os.environ))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    # the no-alloc calls took no device memory ...
    assert res["free1"] == res["free0"], res
    # ... while the allocating entry point's first stream-K call did (its ~20 MB workspace), so the
    # comparison above would have seen an allocation
    assert res["free0"] - res["free2"] >= 16 << 20, res
    assert res["finite"] and all(res["same"]), res


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
        got = _attn(ops, qkv, L, True).cpu().numpy()
        ref = _attn(ops, qkv, L, False).cpu().numpy()
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
