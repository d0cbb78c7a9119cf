"""Kernel parity on a B200: every operator of libanima_b200 against the numpy oracle.

Integer work (W4 decode, the int8 GEMM accumulation) is checked bit-exact / to fp32 rounding;
floating-point ops against the oracle's fp32 math with the tolerance stated in each test.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from tests._util import rel_l2, to_np
from tests.conftest import GOLDEN, pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    return pkg("ops")


def gen(seed):
    return torch.Generator(device="cpu").manual_seed(seed)


def randn(shape, seed, scale=1.0):
    return torch.randn(shape, generator=gen(seed)) * scale


# ----------------------------------------------------------------------------- weights

@pytest.mark.parametrize("case", ["w4_gauss", "w4_fit"])
def test_unpack_w4_bit_exact(ops, case):
    g = dict(np.load(os.path.join(GOLDEN, f"quant_{case}.npz")))
    N, half = g["weight"].shape
    out = ops.unpack_w4(torch.from_numpy(g["weight"].view(np.uint8)).to(DEV),
                        torch.from_numpy(g["weight_s_rel"]).to(DEV),
                        torch.from_numpy(g["weight_codebook"]).to(DEV), N, 2 * half)
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.float32), g["grid"])


def test_unpack_w4_all_codes_and_scales(ops):
    """Every (code, fp8 scale byte) pair except NaN bytes, against the oracle's decode."""
    s_bytes = np.array([b for b in range(256) if (b & 0x7F) != 0x7F], dtype=np.uint8)
    N = len(s_bytes)
    K = 16 * 16
    codes = np.tile(np.arange(16, dtype=np.uint8), (N, K // 16))
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    s_rel = np.repeat(s_bytes[:, None], K // 16, 1)
    cb = (oracle.FIXED_LUT * 3.7).astype(np.float32)
    out = ops.unpack_w4(torch.from_numpy(packed).to(DEV), torch.from_numpy(s_rel).to(DEV),
                        torch.from_numpy(cb).to(DEV), N, K)
    ref = oracle.decode_w4_grid(packed, s_rel, cb)
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.float32), ref)


# ----------------------------------------------------------------------------- row ops

@pytest.mark.parametrize("rotate", [False, True])
def test_layernorm_mod(ops, rotate):
    x = randn((300, 2048), 1) * 3 + 0.5
    mod = randn((6144,), 2, 0.5)
    y = ops.layernorm_mod(x.to(DEV), mod.to(DEV), 0, 2048, 2048, rotate=rotate).cpu().numpy()
    ref = oracle.layer_norm(x.numpy()) * (1 + mod[2048:4096].numpy()) + mod[:2048].numpy()
    if rotate:
        ref = oracle.rotate(ref)
    assert rel_l2(y, ref) < 2e-6


# two planes: |error| <= s / 508 per element, ~3.6e-5 relative for Gaussian rows
@pytest.mark.parametrize("planes,tol", [(2, 6e-5), (1, 1e-2)])
def test_layernorm_mod_quant(ops, planes, tol):
    x = randn((257, 2048), 3) * 2
    mod = randn((6144,), 4, 0.5)
    q = ops.layernorm_mod_quant(x.to(DEV), mod.to(DEV), 0, 2048, 2048, planes=planes)
    ref = oracle.rotate(oracle.layer_norm(x.numpy()) * (1 + mod[2048:4096].numpy()) + mod[:2048].numpy())
    assert rel_l2(q.dequant().cpu().numpy(), ref) < tol
    assert q.hi.abs().max().item() <= 127
    s = q.scale.cpu().numpy()
    np.testing.assert_allclose(s, np.abs(ref).max(1) / 127, rtol=1e-5)


@pytest.mark.parametrize("cols", [256, 512, 1024, 2048, 4096, 8192])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_rotate_quant(ops, cols, dtype):
    x = (randn((130, cols), 5) * 1.5).to(dtype)
    q = ops.rotate_quant(x.to(DEV))
    ref = oracle.rotate(x.float().numpy())
    assert rel_l2(q.dequant().cpu().numpy(), ref) < 6e-5


def test_gelu_rotate_quant(ops):
    """GELU -> ConvRot -> per-token quant of an fp16 MLP pre-activation [rows, 8192]."""
    x = (randn((77, 8192), 47) * 3).to(torch.float16)
    q = ops.rotate_quant(x.to(DEV), act="gelu")
    ref = oracle.rotate(oracle.gelu(x.float().numpy()))
    assert rel_l2(q.dequant().cpu().numpy(), ref) < 6e-5


# The int8 outputs of 2048- and 8192-column rows run on the persistent ring kernel (rows streamed
# into shared-memory stages by bulk copies). Row counts: fewer than one CTA's teams, not a multiple
# of the grid, and more rows per CTA than the ring has stages (stages refilled); rows read at a
# stride wider than the row. Every row is checked, not only the whole-matrix error.
@pytest.mark.parametrize("kind,rows,pad", [
    ("ln", 1, 0), ("ln", 1633, 0), ("ln", 4096, 0),
    ("rot16", 5, 64), ("rot16", 6000, 0), ("rotbf16", 300, 0), ("rot32", 4000, 0),
    ("gelu", 3, 0), ("gelu", 4096, 0), ("rot32_8192", 1000, 256)])
def test_ring_rows(ops, kind, rows, pad):
    cols = 8192 if kind in ("gelu", "rot32_8192") else 2048
    dtype = {"rot16": torch.float16, "gelu": torch.float16, "rotbf16": torch.bfloat16}.get(kind, torch.float32)
    wide = (randn((rows, cols + pad), 61 + rows) * 2 + 0.25).to(dtype)
    x = wide[:, :cols]
    xf = x.float().numpy()
    if kind == "ln":
        mod = randn((6144,), 62, 0.5)
        q = ops.layernorm_mod_quant(x.contiguous().to(DEV), mod.to(DEV), 0, 2048, 2048)
        ref = oracle.rotate(oracle.layer_norm(xf) * (1 + mod[2048:4096].numpy()) + mod[:2048].numpy())
    else:
        q = ops.rotate_quant(wide.to(DEV)[:, :cols], act="gelu" if kind == "gelu" else None)
        ref = oracle.rotate(oracle.gelu(xf) if kind == "gelu" else xf)
    got = q.dequant().cpu().numpy()
    row_err = np.sqrt(((got - ref) ** 2).sum(1) / (ref ** 2).sum(1))
    assert row_err.max() < 1.5e-4, (row_err.argmax(), row_err.max())
    assert rel_l2(got, ref) < 6e-5
    np.testing.assert_allclose(q.scale.cpu().numpy(), np.abs(ref).max(1) / 127, rtol=1e-5)
    assert q.hi.abs().max().item() <= 127 and q.lo.abs().max().item() <= 127


@pytest.mark.parametrize("cols", [256, 2048])
def test_rotate_plain(ops, cols):
    x = randn((67, cols), 6)
    y = ops.rotate(x.to(DEV)).cpu().numpy()
    assert rel_l2(y, oracle.rotate(x.numpy())) < 1e-6


def test_rmsnorm_and_qk_norm_rope(ops):
    L, H = 96, 16
    x = randn((L * H, 128), 7) * 2
    w = 1 + randn((128,), 8, 0.1)
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 128).cpu().numpy()
    assert rel_l2(y, oracle.rms_norm(x.numpy(), w.numpy())) < 2e-6
    qkv = randn((L, 3 * 2048), 9)
    qn, kn = 1 + randn((128,), 10, 0.1), 1 + randn((128,), 11, 0.1)
    cs = torch.from_numpy(pkg("dit").rope_table(8, 12))
    t = qkv.clone().to(DEV)
    ops.qk_norm_rope(t, qn.to(DEV), kn.to(DEV), cs.to(DEV), L, H, 128)
    cos, sin = oracle.dit_rope(8, 12)
    cos, sin = np.concatenate([cos, cos], -1)[:, None], np.concatenate([sin, sin], -1)[:, None]
    q = oracle.rms_norm(qkv[:, :2048].numpy().reshape(L, H, 128), qn.numpy())
    k = oracle.rms_norm(qkv[:, 2048:4096].numpy().reshape(L, H, 128), kn.numpy())
    q = q * cos + oracle.rotate_half(q) * sin
    k = k * cos + oracle.rotate_half(k) * sin
    got = t.cpu().numpy()
    assert rel_l2(got[:, :2048], q.reshape(L, -1)) < 2e-6
    assert rel_l2(got[:, 2048:4096], k.reshape(L, -1)) < 2e-6
    np.testing.assert_array_equal(got[:, 4096:], qkv[:, 4096:].numpy())


def test_elementwise_patchify_timestep_euler(ops):
    a, b = randn((1000,), 12), randn((1000,), 13)
    for op, ref in (("copy", a), ("add", a + b), ("silu", oracle.silu(a.numpy())),
                    ("silu_mul", oracle.silu(a.numpy()) * b.numpy())):
        y = ops.elementwise(op, a.to(DEV), b.to(DEV)).cpu().numpy()
        assert rel_l2(y, np.asarray(ref)) < 1e-6, op
    lat = randn((2, 16, 12, 20), 14)
    p = ops.patchify(lat.to(DEV)).cpu().numpy()
    ref = np.concatenate([oracle.patchify(lat[i].numpy()) for i in range(2)])
    np.testing.assert_array_equal(p, ref)
    o = randn((2 * 6 * 10, 64), 15)
    u = ops.unpatchify(o.to(DEV), 2, 12, 20).cpu().numpy()
    ref = np.stack([oracle.unpatchify(o[i * 60:(i + 1) * 60].numpy(), 12, 20) for i in range(2)])
    np.testing.assert_array_equal(u, ref)
    sig = torch.tensor([0.9, 0.25, 1.0])
    t = ops.timestep_embedding(sig.to(DEV)).cpu().numpy()
    for i, s in enumerate(sig.tolist()):
        assert np.abs(t[i] - oracle.timestep_embedding(s)[0]).max() < 2e-6
    x, v, vn = randn((500,), 16), randn((500,), 17), randn((500,), 18)
    xd = x.clone().to(DEV)
    ops.euler_step(xd, v.to(DEV), 0.8, 0.5, v_uncond=vn.to(DEV), cfg=4.5)
    vel = vn + (v - vn) * 4.5
    den = x - vel * 0.8
    assert rel_l2(xd.cpu().numpy(), (x + (x - den) / 0.8 * (0.5 - 0.8)).numpy()) < 1e-6
    xd = x.clone().to(DEV)
    ops.euler_step(xd, v.to(DEV), 0.3, 0.0)
    assert rel_l2(xd.cpu().numpy(), (x - v * 0.3).numpy()) < 1e-6


@pytest.mark.parametrize("M,N,K", [(1, 6144, 2048), (64, 2048, 68), (130, 64, 2048), (2000, 1000, 100),
                                   (1000, 1000, 300), (4096, 64, 2048)])
@pytest.mark.parametrize("kind", ["bf16", "f32"])
def test_matmul_simt(ops, M, N, K, kind):
    W = pkg("weights")
    x = randn((M, K), 19)
    w = randn((N, K), 20, 0.02)
    wt = w.to(torch.bfloat16) if kind == "bf16" else w
    lin = W.Linear(kind, N, K, wt.to(DEV).contiguous())
    y = ops.matmul(x.to(DEV), lin, act="silu").cpu().numpy()
    ref = oracle.silu(x.numpy() @ wt.float().numpy().T)
    assert rel_l2(y, ref) < 2e-6


# bf16 weights without scale, activation or gate run on the tensor cores (A split into two bf16
# planes: ~2^-17 relative per element, fp32 sums); the rest stays on the CUDA-core kernel above
@pytest.mark.parametrize("M,N,K,resid", [(4096, 64, 2048, False), (512, 1024, 1024, True), (300, 3, 16, False),
                                         (1000, 384, 96, True)])
def test_matmul_bf16_tensor_cores(ops, M, N, K, resid):
    W = pkg("weights")
    x = randn((M, K), 23)
    w = (randn((N, K), 24, 0.05)).to(torch.bfloat16)
    b = randn((N,), 25, 0.1)
    lin = W.Linear("bf16", N, K, w.to(DEV).contiguous(), None, bias=b.to(DEV))
    base = randn((M, N), 26)
    out = base.clone().to(DEV) if resid else None
    y = ops.matmul(x.to(DEV), lin, out=out, resid=resid).cpu().numpy()
    ref = x.double().numpy() @ w.double().numpy().T + b.double().numpy()
    if resid:
        ref = ref + base.double().numpy()
    assert rel_l2(y, ref) < 2e-5


# ----------------------------------------------------------------------------- tcgen05 int8 GEMM

def make_linear(N, K, seed):
    W = pkg("weights")
    g = gen(seed)
    q = (torch.randn(N, K, generator=g) * 40).round().clamp(-127, 127).to(torch.int8)
    s = 0.0005 * (1 + torch.rand(N, generator=g))
    return W.Linear("i8", N, K, q.to(DEV), s.to(DEV)), q.float().numpy(), s.numpy()


def gemm_ref(qa, wq, ws):
    return qa.dequant().cpu().double().numpy() @ wq.astype(np.float64).T * ws.astype(np.float64)


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (200, 2048, 2048), (4096, 6144, 2048), (333, 2048, 8192),
                                   (512, 8192, 2048), (77, 2048, 1024), (256, 384, 256)])
@pytest.mark.parametrize("planes", [2, 1])
def test_linear_store_f32(ops, M, N, K, planes):
    lin, wq, ws = make_linear(N, K, M + N + K)
    x = randn((M, K), 21) * 2
    qa = ops.rotate_quant(x.to(DEV), planes=planes)
    y = ops.linear(qa, lin).cpu().numpy()
    ref = gemm_ref(qa, wq, ws)
    # integer accumulation is exact; the epilogue's fp32 scaling rounds at ~1e-7
    assert rel_l2(y, ref) < 1e-6


@pytest.mark.parametrize("out_dtype,tol", [(torch.bfloat16, 5e-3), (torch.float16, 6e-4)])
def test_linear_store_16bit_gelu(ops, out_dtype, tol):
    M, N, K = 300, 8192, 2048
    lin, wq, ws = make_linear(N, K, 3)
    qa = ops.rotate_quant((randn((M, K), 22) * 2).to(DEV))
    y = ops.linear(qa, lin, act="gelu", out_dtype=out_dtype).float().cpu().numpy()
    ref = oracle.gelu(gemm_ref(qa, wq, ws).astype(np.float32))
    assert rel_l2(y, ref) < tol


def test_linear_gated_residual_bias_add(ops):
    M, N, K = 260, 2048, 2048
    lin, wq, ws = make_linear(N, K, 4)
    lin.bias = (randn((N,), 23, 0.1)).to(DEV)
    qa = ops.rotate_quant((randn((M, K), 24)).to(DEV))
    x0 = randn((M, N), 25)
    add = randn((M, N), 26, 0.05)
    mod = randn((6144,), 27, 0.5)
    out = x0.clone().to(DEV)
    ops.linear(qa, lin, out=out, resid=True, gate=mod.to(DEV), g_off=4096, add=add.to(DEV))
    y = gemm_ref(qa, wq, ws) + lin.bias.cpu().numpy() + add.numpy()
    ref = x0.numpy() + mod[4096:].numpy() * y
    assert rel_l2(out.cpu().numpy(), ref) < 1e-6


def test_linear_qkv_norm_rope_epilogue(ops):
    Hp, Wp = 8, 12
    L = Hp * Wp
    B = 2
    M, N, K = B * L, 6144, 2048
    lin, wq, ws = make_linear(N, K, 5)
    qa = ops.rotate_quant((randn((M, K), 28)).to(DEV))
    qn, kn = 1 + randn((128,), 29, 0.1), 1 + randn((128,), 30, 0.1)
    cs = torch.from_numpy(pkg("dit").rope_table(Hp, Wp)).to(DEV)
    out = ops.linear(qa, lin, mode="qkv", qk=(qn.to(DEV), kn.to(DEV)), rope_cs=cs, n_q=2048,
                     out_dtype=torch.float32).cpu().numpy()
    y = gemm_ref(qa, wq, ws).astype(np.float32)
    cos, sin = oracle.dit_rope(Hp, Wp)
    cos = np.tile(np.concatenate([cos, cos], -1), (B, 1))[:, None]
    sin = np.tile(np.concatenate([sin, sin], -1), (B, 1))[:, None]
    q = oracle.rms_norm(y[:, :2048].reshape(M, 16, 128), qn.numpy())
    k = oracle.rms_norm(y[:, 2048:4096].reshape(M, 16, 128), kn.numpy())
    q = q * cos + oracle.rotate_half(q) * sin
    k = k * cos + oracle.rotate_half(k) * sin
    assert rel_l2(out[:, :2048], q.reshape(M, -1)) < 2e-6
    assert rel_l2(out[:, 2048:4096], k.reshape(M, -1)) < 2e-6
    assert rel_l2(out[:, 4096:], y[:, 4096:]) < 1e-6
    # head-norm mode (cross q) on the first 2048 columns
    lin2, wq2, ws2 = make_linear(2048, K, 6)
    h = ops.linear(qa, lin2, mode="head_norm", qk=(qn.to(DEV),), out_dtype=torch.float32).cpu().numpy()
    ref = oracle.rms_norm(gemm_ref(qa, wq2, ws2).astype(np.float32).reshape(M, 16, 128), qn.numpy())
    assert rel_l2(h, ref.reshape(M, -1)) < 2e-6


def _lora_entries(K, spec, seed):
    """LoRA entries [(off, n, r, scale)] with A [r, K], B [n, r] on the device + numpy copies."""
    out = []
    for i, (off, n, r, scale) in enumerate(spec):
        A = randn((r, K), seed + 2 * i, 0.01)
        B = randn((n, r), seed + 2 * i + 1, 0.01)
        out.append({"A": A.to(DEV), "B": B.to(DEV), "r": r, "scale": scale, "off": off, "n": n,
                    "A_np": A.numpy(), "B_np": B.numpy()})
    return out


def _lora_ref(qa, entries, N):
    x = qa.dequant().cpu().double().numpy()
    d = np.zeros((x.shape[0], N))
    for e in entries:
        d[:, e["off"]:e["off"] + e["n"]] += e["scale"] * (x @ e["A_np"].T.astype(np.float64)) @ e["B_np"].T
    return d


def test_lora_down_product_k_slices(ops):
    """A long-K down-projection (MLP layer 2, K = 8192) runs as K slices on side streams whose fp32
    partials are summed in a fixed order: the same T as one GEMM, to fp32 rounding."""
    lora = pkg("lora")
    M, N, K = 300, 2048, 8192
    lin, _, _ = make_linear(N, K, 8)
    lin.lora = [{k: v for k, v in e.items() if not k.endswith("_np")}
                for e in _lora_entries(K, [(0, 2048, 32, 1.0)], 51)]
    qa = ops.rotate_quant(randn((M, K), 52).to(DEV))
    assert lora._k_slices(M, lora._down_linear(lin), qa.hi.device) == 4
    T = lora.down_product(qa, lin).cpu().numpy()
    T1 = ops.linear(qa, lora._down_linear(lin)).cpu().numpy()
    assert rel_l2(T, T1) < 1e-6


# fused (ranks multiple of 4, 16-aligned ranges) and the [M, N] delta fallback (rank 6)
@pytest.mark.parametrize("spec,mode", [([(0, 2048, 32, 1.0), (2048, 2048, 32, 0.5), (4096, 2048, 16, 2.0)], "store"),
                                       ([(128, 1024, 8, 1.5)], "resid"),
                                       ([(0, 2048, 32, 1.0), (2048, 2048, 32, 1.0)], "qkv"),
                                       ([(0, 6144, 6, 1.0)], "store")])
@pytest.mark.parametrize("path", ["delta", "fused"])
def test_linear_lora_epilogue(ops, spec, mode, path, monkeypatch):
    """Both side-path forms carry fp16 copies of scale * B^T and fp32 sums (the fused epilogue also
    an fp16 copy of x_r A^T; the tensor-core delta two fp16 planes of it), so the output carries
    ~2^-11 of the LoRA delta (a few % of y here) on top of the base GEMM's fp32 rounding: 3e-5 of
    the output where the base path alone is held to 2e-6. With the fused form, entries it cannot
    take (rank 6) go through the fp32 CUDA-core delta."""
    monkeypatch.setattr(pkg("lora"), "PATH", path)
    M, K = 260, 2048
    fused = all(r % 4 == 0 for (_, _, r, _) in spec)
    tol = 3e-5 if (fused or path == "delta") else 2e-6
    N = 6144 if mode in ("store", "qkv") else 2048
    lin, wq, ws = make_linear(N, K, 8)
    lin.lora = [{k: v for k, v in e.items() if not k.endswith("_np")} for e in _lora_entries(K, spec, 50)]
    ents = _lora_entries(K, spec, 50)
    qa = ops.rotate_quant((randn((M, K), 33)).to(DEV))
    y = gemm_ref(qa, wq, ws) + _lora_ref(qa, ents, N)
    if mode == "store":
        out = ops.linear(qa, lin, act="gelu").cpu().numpy()
        assert rel_l2(out, oracle.gelu(y.astype(np.float32))) < tol
    elif mode == "resid":
        x0 = randn((M, N), 34)
        mod = randn((6144,), 35, 0.5)
        out = x0.clone().to(DEV)
        ops.linear(qa, lin, out=out, resid=True, gate=mod.to(DEV), g_off=4096)
        ref = x0.numpy() + mod[4096:].numpy() * y
        assert rel_l2(out.cpu().numpy() - x0.numpy(), ref - x0.numpy()) < tol
    else:
        Hp, Wp = 10, 26
        qn, kn = 1 + randn((128,), 36, 0.1), 1 + randn((128,), 37, 0.1)
        cs = torch.from_numpy(pkg("dit").rope_table(Hp, Wp)).to(DEV)
        out = ops.linear(qa, lin, mode="qkv", qk=(qn.to(DEV), kn.to(DEV)), rope_cs=cs, n_q=2048,
                         out_dtype=torch.float32).cpu().numpy()
        yf = y.astype(np.float32)
        cos, sin = oracle.dit_rope(Hp, Wp)
        cos = np.concatenate([cos, cos], -1)[:, None]
        sin = np.concatenate([sin, sin], -1)[:, None]
        q = oracle.rms_norm(yf[:, :2048].reshape(M, 16, 128), qn.numpy())
        q = q * cos + oracle.rotate_half(q) * sin
        assert rel_l2(out[:, :2048], q.reshape(M, -1)) < tol
        assert rel_l2(out[:, 4096:], yf[:, 4096:]) < 1e-6


# block-sized shapes whose tile counts leave a partial last wave on 148 SMs
@pytest.mark.parametrize("M,N,mode", [(4096, 2048, "resid"), (2560, 2048, "store"), (2560, 6144, "qkv")])
def test_linear_partial_last_wave(ops, M, N, mode):
    K = 2048
    lin, wq, ws = make_linear(N, K, 9)
    qa = ops.rotate_quant((randn((M, K), 38)).to(DEV))
    y = gemm_ref(qa, wq, ws)
    if mode == "resid":
        x0 = randn((M, N), 39)
        mod = randn((6144,), 40, 0.5)
        out = x0.clone().to(DEV)
        ops.linear(qa, lin, out=out, resid=True, gate=mod.to(DEV), g_off=4096)
        assert rel_l2(out.cpu().numpy(), x0.numpy() + mod[4096:].numpy() * y) < 1e-6
    elif mode == "store":
        assert rel_l2(ops.linear(qa, lin).cpu().numpy(), y) < 1e-6
    else:
        Hp, Wp = 40, 64
        qn, kn = 1 + randn((128,), 41, 0.1), 1 + randn((128,), 42, 0.1)
        cs = torch.from_numpy(pkg("dit").rope_table(Hp, Wp)).to(DEV)
        out = ops.linear(qa, lin, mode="qkv", qk=(qn.to(DEV), kn.to(DEV)), rope_cs=cs, n_q=2048,
                         out_dtype=torch.float32).cpu().numpy()
        yf = y.astype(np.float32)
        cos, sin = oracle.dit_rope(Hp, Wp)
        cos = np.concatenate([cos, cos], -1)[:, None]
        sin = np.concatenate([sin, sin], -1)[:, None]
        k = oracle.rms_norm(yf[:, 2048:4096].reshape(M, 16, 128), kn.numpy())
        k = k * cos + oracle.rotate_half(k) * sin
        assert rel_l2(out[:, 2048:4096], k.reshape(M, -1)) < 2e-6
        assert rel_l2(out[:, 4096:], yf[:, 4096:]) < 1e-6
    # the same call twice gives the same bits
    if mode == "store":
        a = ops.linear(qa, lin).cpu()
        b = ops.linear(qa, lin).cpu()
        assert torch.equal(a, b)


def test_linear_rejects_bad_shapes(ops):
    dev = pkg("device")
    lin, _, _ = make_linear(2048, 2048, 7)
    qa = ops.rotate_quant(randn((16, 1024), 31).to(DEV))
    with pytest.raises(dev.AnimaError, match="columns"):
        ops.linear(qa, lin)


# ----------------------------------------------------------------------------- attention

def attn_ref(q, k, v, key_len=None):
    """fp32 oracle attention on the same 16-bit inputs; q [H, Lq, D]."""
    return oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), key_len)


@pytest.mark.parametrize("L", [128, 200, 1024])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_self_attention_qkv_layout(ops, L, dtype):
    H = 16
    qkv = (randn((L, 3 * 2048), 32 + L)).to(dtype)
    out = ops.attention(qkv.to(DEV), qkv.to(DEV), qkv.to(DEV), Lq=L, Lk=L, H=H, ldq=6144, ldk=6144, ldv=6144,
                        q_off=0, k_off=2048, v_off=4096, out_dtype=torch.float32).cpu().numpy()
    q = qkv[:, :2048].reshape(L, H, 128).transpose(0, 1)
    k = qkv[:, 2048:4096].reshape(L, H, 128).transpose(0, 1)
    v = qkv[:, 4096:].reshape(L, H, 128).transpose(0, 1)
    ref = attn_ref(q, k, v).transpose(1, 0, 2).reshape(L, 2048)
    # P is rounded to the 16-bit input type before P V (bf16: ~2^-9 relative per probability)
    tol = 6e-3 if dtype == torch.bfloat16 else 1e-3
    assert rel_l2(out, ref) < tol


def test_cross_attention_batched_masked(ops):
    B, H, Lq, Lk = 2, 16, 300, 256
    q = randn((B * Lq, 2048), 40).to(torch.bfloat16)
    k = randn((B * Lk, 2048), 41).to(torch.bfloat16)
    v = randn((B * Lk, 2048), 42).to(torch.bfloat16)
    kl = torch.tensor([37, 256], dtype=torch.int32)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=Lq, Lk=Lk, H=H, batch=B, q_bstride=Lq * 2048,
                        k_bstride=Lk * 2048, v_bstride=Lk * 2048, key_len=kl.to(DEV),
                        out_dtype=torch.float32).cpu().numpy()
    for b in range(B):
        qb = q[b * Lq:(b + 1) * Lq].reshape(Lq, H, 128).transpose(0, 1)
        kb = k[b * Lk:(b + 1) * Lk].reshape(Lk, H, 128).transpose(0, 1)
        vb = v[b * Lk:(b + 1) * Lk].reshape(Lk, H, 128).transpose(0, 1)
        ref = attn_ref(qb, kb, vb, int(kl[b])).transpose(1, 0, 2).reshape(Lq, 2048)
        assert rel_l2(out[b * Lq:(b + 1) * Lq], ref) < 6e-3, b


def test_cross_attention_shared_kv_zero_padded(ops):
    """The reference's semantics: context zero-padded to 512 rows, no mask (dit.js:185-190)."""
    B, H, Lq, Lk = 2, 16, 256, 512
    q = randn((B * Lq, 2048), 43).to(torch.bfloat16)
    k = torch.cat([randn((200, 2048), 44), torch.zeros(312, 2048)]).to(torch.bfloat16)
    v = torch.cat([randn((200, 2048), 45), torch.zeros(312, 2048)]).to(torch.bfloat16)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=Lq, Lk=Lk, H=H, batch=B, q_bstride=Lq * 2048,
                        k_bstride=0, v_bstride=0, out_dtype=torch.float32).cpu().numpy()
    kb = k.reshape(Lk, H, 128).transpose(0, 1)
    vb = v.reshape(Lk, H, 128).transpose(0, 1)
    for b in range(B):
        qb = q[b * Lq:(b + 1) * Lq].reshape(Lq, H, 128).transpose(0, 1)
        ref = attn_ref(qb, kb, vb).transpose(1, 0, 2).reshape(Lq, 2048)
        assert rel_l2(out[b * Lq:(b + 1) * Lq], ref) < 6e-3


def test_device_errors_surface_at_sync(ops):
    """Synchronising reports success when nothing faulted (the error word starts clear)."""
    ctx = pkg("device").Context.get(0)
    x = randn((4, 2048), 46).to(DEV)
    ops.rotate(x)
    ctx.sync()


# ----------------------------------------------------------------------------- stream-K attention

def _self_attn(ops, qkv, L, H, batch=1, bstride=None):
    return ops.attention(qkv, qkv, qkv, Lq=L, Lk=L, H=H, ldq=3 * H * 128, ldk=3 * H * 128, ldv=3 * H * 128,
                         q_off=0, k_off=H * 128, v_off=2 * H * 128, batch=batch, q_bstride=bstride or 0,
                         k_bstride=bstride or 0, v_bstride=bstride or 0, out_dtype=torch.float32)


def _split(mode):
    pkg("device").Context.get(0).set_attention_split(mode)


@pytest.fixture
def split_mode():
    yield _split
    _split(-1)


@pytest.mark.parametrize("L,H,batch", [(4096, 16, 1), (4000, 16, 1), (2048, 24, 2), (1536, 64, 1)])
def test_stream_k_attention_matches_whole_units(ops, split_mode, L, H, batch):
    """The key blocks of all units split evenly over the SMs (a unit cut into a head part and a tail
    part, merged through the workspace) give the whole-unit result up to rounding: each part keeps
    its own running max, so its 16-bit probabilities round differently. Checked against the oracle
    on two heads."""
    D = 3 * H * 128
    qkv = randn((batch * L, D), 60 + L + H).to(torch.bfloat16).to(DEV)
    split_mode(0)
    whole = _self_attn(ops, qkv, L, H, batch, L * D if batch > 1 else None).cpu().numpy()
    split_mode(1)
    sk = _self_attn(ops, qkv, L, H, batch, L * D if batch > 1 else None).cpu().numpy()
    assert rel_l2(sk, whole) < 2e-3
    c = qkv[:L].cpu()
    for h in (0, H - 1):
        q = c[:, h * 128:(h + 1) * 128][None]
        k = c[:, H * 128 + h * 128:H * 128 + (h + 1) * 128][None]
        v = c[:, 2 * H * 128 + h * 128:2 * H * 128 + (h + 1) * 128][None]
        ref = attn_ref(q, k, v)[0]
        assert rel_l2(sk[:L, h * 128:(h + 1) * 128], ref) < 6e-3, h


def test_stream_k_attention_consecutive_calls(ops, split_mode):
    """Two stream-K calls on different inputs: the second must not merge partials or flags left by the
    first (every flag is cleared by the CTA that consumes it), and repeating a call is bit-exact."""
    L, H = 4096, 16
    a = randn((L, 6144), 70).to(torch.bfloat16).to(DEV)
    b = randn((L, 6144), 71).to(torch.bfloat16).to(DEV)
    split_mode(0)
    ref_b = _self_attn(ops, b, L, H).cpu().numpy()
    split_mode(1)
    _self_attn(ops, a, L, H)
    out_b1 = _self_attn(ops, b, L, H).cpu().numpy()
    out_b2 = _self_attn(ops, b, L, H).cpu().numpy()
    assert np.array_equal(out_b1, out_b2)
    assert rel_l2(out_b1, ref_b) < 2e-3  # a merge with the first call's partials would be O(1) off


def test_stream_k_not_used_with_key_mask(ops, split_mode):
    """With key_len the units differ in length: the whole-unit schedule runs even when forced."""
    B, H, Lq, Lk = 1, 16, 4096, 512
    q = randn((Lq, 2048), 72).to(torch.bfloat16)
    k = randn((Lk, 2048), 73).to(torch.bfloat16)
    v = randn((Lk, 2048), 74).to(torch.bfloat16)
    kl = torch.tensor([300], dtype=torch.int32)
    split_mode(1)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=Lq, Lk=Lk, H=H, key_len=kl.to(DEV),
                        out_dtype=torch.float32).cpu().numpy()
    qb = q.reshape(Lq, H, 128).transpose(0, 1)[:2]
    kb = k.reshape(Lk, H, 128).transpose(0, 1)[:2]
    vb = v.reshape(Lk, H, 128).transpose(0, 1)[:2]
    ref = attn_ref(qb, kb, vb, 300).transpose(1, 0, 2).reshape(Lq, 256)
    assert rel_l2(out[:, :256], ref) < 6e-3


def test_cross_attention_persistent_grid(ops):
    """4096 queries x 512 keys x 16 heads: 256 whole units on a persistent grid (one CTA per SM, each
    taking every grid-th unit); checked against the oracle on two heads."""
    Lq, Lk, H = 4096, 512, 16
    q = randn((Lq, 2048), 80).to(torch.bfloat16)
    kv = randn((Lk, 4096), 81).to(torch.bfloat16)
    out = ops.attention(q.to(DEV), kv.to(DEV), kv.to(DEV), Lq=Lq, Lk=Lk, H=H, ldk=4096, ldv=4096, k_off=0,
                        v_off=2048, out_dtype=torch.float32).cpu().numpy()
    for h in (0, H - 1):
        qh = q[:, h * 128:(h + 1) * 128][None]
        kh = kv[:, h * 128:(h + 1) * 128][None]
        vh = kv[:, 2048 + h * 128:2048 + (h + 1) * 128][None]
        ref = attn_ref(qh, kh, vh)[0]
        assert rel_l2(out[:, h * 128:(h + 1) * 128], ref) < 6e-3, h


def test_stream_k_shared_kv_batch(ops, split_mode):
    """Stream-K forced on a batch of 2 sharing one K/V (the CFG cross-attention layout): matches the
    whole-unit schedule and the oracle."""
    B, H, Lq, Lk = 2, 16, 2048, 1024
    q = randn((B * Lq, 2048), 82).to(torch.bfloat16).to(DEV)
    kv = randn((Lk, 4096), 83).to(torch.bfloat16).to(DEV)
    args = dict(Lq=Lq, Lk=Lk, H=H, ldk=4096, ldv=4096, k_off=0, v_off=2048, batch=B, q_bstride=Lq * 2048,
                k_bstride=0, v_bstride=0, out_dtype=torch.float32)
    split_mode(0)
    whole = ops.attention(q, kv, kv, **args).cpu().numpy()
    split_mode(1)
    sk = ops.attention(q, kv, kv, **args).cpu().numpy()
    assert rel_l2(sk, whole) < 2e-3
    kh = kv[:, :128].cpu()[None]
    vh = kv[:, 2048:2048 + 128].cpu()[None]
    for b in range(B):
        qh = q[b * Lq:(b + 1) * Lq, :128].cpu()[None]
        assert rel_l2(sk[b * Lq:(b + 1) * Lq, :128], attn_ref(qh, kh, vh)[0]) < 6e-3, b


def test_persistent_grid_batched_key_len(ops):
    """More than one wave of whole units with a different key_len per batch item (each unit looks up
    its own item's length on the persistent grid)."""
    B, H, Lq, Lk = 2, 16, 2048, 384
    q = randn((B * Lq, 2048), 84).to(torch.bfloat16)
    k = randn((B * Lk, 2048), 85).to(torch.bfloat16)
    v = randn((B * Lk, 2048), 86).to(torch.bfloat16)
    kl = torch.tensor([130, 384], dtype=torch.int32)
    out = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), Lq=Lq, Lk=Lk, H=H, batch=B, q_bstride=Lq * 2048,
                        k_bstride=Lk * 2048, v_bstride=Lk * 2048, key_len=kl.to(DEV),
                        out_dtype=torch.float32).cpu().numpy()
    for b in range(B):
        qb = q[b * Lq:(b + 1) * Lq].reshape(Lq, H, 128).transpose(0, 1)[[0, H - 1]]
        kb = k[b * Lk:(b + 1) * Lk].reshape(Lk, H, 128).transpose(0, 1)[[0, H - 1]]
        vb = v[b * Lk:(b + 1) * Lk].reshape(Lk, H, 128).transpose(0, 1)[[0, H - 1]]
        ref = attn_ref(qb, kb, vb, int(kl[b]))
        got = out[b * Lq:(b + 1) * Lq].reshape(Lq, H, 128)[:, [0, H - 1]].transpose(1, 0, 2)
        assert rel_l2(got, ref) < 6e-3, b
