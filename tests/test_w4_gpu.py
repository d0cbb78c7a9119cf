"""W4A8 linears through anima_linear (kind W4): the packed nibbles stay resident and each call
decodes them to the int8 grid right before the GEMM. The outputs must be bit-identical to
decoding once with anima_unpack_w4 and running the same GEMM as kind I8 (the decode itself is
pinned bit-exact to the reference's quantizer output in test_kernels_gpu.py), for both codebook
kinds of tools/quant.py:116-124 (FIXED_LUT and a Lloyd fit) and every epilogue the DiT uses."""

import numpy as np
import pytest
import torch

from tests.conftest import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _w4_weight(kind, N, K, seed):
    quant, W = pkg("quant"), pkg("weights")
    g = torch.Generator().manual_seed(seed)
    if kind == "gauss":
        w = torch.randn(N, K, generator=g) * 0.02
    else:  # sparse rotated weight: heavy tails, so the quantizer fits its own codebook
        sp = torch.zeros(N, K)
        idx = torch.randint(0, K, (N, K // 20), generator=g)
        sp.scatter_(1, idx, torch.randn(N, K // 20, generator=g))
        w = quant.rotate(sp + 0.01 * torch.randn(N, K, generator=g)) * 0.02
    q = quant.quantize_w4a8(w)
    t = {"l." + k: v for k, v in q.items()}
    lin = W.linear_weights(t, "l.", DEV)
    assert lin.kind == "w4" and lin.data.dtype == torch.uint8 and lin.data.shape == (N, K // 2)
    fitted = not torch.equal(q["weight_codebook"], torch.tensor(quant.FIXED_LUT, dtype=torch.float32))
    return lin, fitted


def _as_i8(lin):
    W = pkg("weights")
    return W.Linear("i8", lin.N, lin.K, lin.grid().contiguous(), lin.scale, lin.bias, name=lin.name + ".grid")


@pytest.mark.parametrize("kind", ["gauss", "fit"])
@pytest.mark.parametrize("planes", [2, 1])
def test_w4_linear_bit_identical_to_unpacked_int8(kind, planes):
    ops = pkg("ops")
    N, K, M = 1024, 2048, 700
    lin, fitted = _w4_weight(kind, N, K, 5 + planes)
    assert fitted == (kind == "fit")
    ref_w = _as_i8(lin)
    g = torch.Generator().manual_seed(9)
    qa = ops.rotate_quant(torch.randn(M, K, generator=g).to(DEV), planes)
    # plain store, fp32
    a = ops.linear(qa, lin, out=torch.empty(M, N, device=DEV))
    b = ops.linear(qa, ref_w, out=torch.empty(M, N, device=DEV))
    assert torch.equal(a, b)
    # GELU, fp16 out (the MLP layer-1 form)
    a = ops.linear(qa, lin, out=torch.empty(M, N, dtype=torch.float16, device=DEV), act="gelu")
    b = ops.linear(qa, ref_w, out=torch.empty(M, N, dtype=torch.float16, device=DEV), act="gelu")
    assert torch.equal(a, b)
    # gated residual into fp32 x (the out-projection / layer-2 form)
    x0 = torch.randn(M, N, generator=g).to(DEV)
    gate = torch.randn(3 * N, generator=g).to(DEV)
    xa, xb = x0.clone(), x0.clone()
    ops.linear(qa, lin, out=xa, resid=True, gate=gate, g_off=2 * N)
    ops.linear(qa, ref_w, out=xb, resid=True, gate=gate, g_off=2 * N)
    assert torch.equal(xa, xb)
    pkg("device").Context.get(0).sync()


def test_w4_stacked_qkv_and_larger_layer_after_smaller():
    """q|k|v stacked from W4 parts (one codebook) with the qkv epilogue, then a larger W4 layer:
    the decode buffer is reused and grown, and each call still sees its own weight."""
    ops, W, dit = pkg("ops"), pkg("weights"), pkg("dit")
    parts = [_w4_weight("gauss", 512, 1024, 20 + i)[0] for i in range(3)]
    qkv = W.concat_linears(parts)
    assert qkv is not None and qkv.kind == "w4" and qkv.N == 1536
    ref = _as_i8(qkv)
    M = 256
    g = torch.Generator().manual_seed(3)
    qa = ops.rotate_quant(torch.randn(M, 1024, generator=g).to(DEV), 2)
    nq, nk = (1 + 0.1 * torch.randn(128, generator=g)).to(DEV), (1 + 0.1 * torch.randn(128, generator=g)).to(DEV)
    cs = torch.from_numpy(dit.rope_table(16, 16)).to(DEV)
    outs = []
    for w in (qkv, ref):
        outs.append(ops.linear(qa, w, out=torch.empty(M, 1536, dtype=torch.float16, device=DEV), mode="qkv",
                               qk=(nq, nk), rope_cs=cs, n_q=512))
    assert torch.equal(outs[0], outs[1])
    big, _ = _w4_weight("gauss", 8192, 4096, 31)  # 32 MiB grid: larger than the first buffer
    ref_big = _as_i8(big)
    qb = ops.rotate_quant(torch.randn(M, 4096, generator=g).to(DEV), 2)
    a = ops.linear(qb, big, out=torch.empty(M, 8192, device=DEV))
    b = ops.linear(qb, ref_big, out=torch.empty(M, 8192, device=DEV))
    assert torch.equal(a, b)
    a2 = ops.linear(qa, qkv, out=torch.empty(M, 1536, dtype=torch.float16, device=DEV), mode="qkv", qk=(nq, nk),
                    rope_cs=cs, n_q=512)
    assert torch.equal(a2, outs[1])
    pkg("device").Context.get(0).sync()


def test_mixed_model_keeps_w4_blocks_packed():
    """A W4A8 "mixed" DiT holds its middle blocks at half a byte per weight (plus 1/16 byte of
    fp8 group scales), the first and last block at one byte."""
    syn, ditm = pkg("synthetic"), pkg("dit")
    t = syn.dit_tensors(3, "mixed", 3, direct=True)
    model = ditm.AnimaDiT(t, DEV, n_blocks=3)
    per_block = []
    for blk in model.blocks:
        lins = [blk[k] for k in ("qkv", "self_o", "cross_q", "cross_k", "cross_v", "cross_o", "l1", "l2")]
        n_w = sum(w.N * w.K for w in lins)
        per_block.append(sum(w.nbytes() for w in lins) / n_w)
        assert {w.kind for w in lins} == ({"w4"} if len(per_block) == 2 else {"i8"})
    assert per_block[1] < 0.57 and per_block[0] > 1.0 and per_block[2] > 1.0, per_block
