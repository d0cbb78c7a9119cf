"""numpy restatement of the reference's DiT denoising path (TEST ORACLE, never the product).

Every function cites the reference line it restates. The reference computes in fp32 with weights
dequantized on access (tools/reference.py:38-45); this module does the same.

Parity status: pinned. tests/golden/*.npz were produced by the reference's own tools/quant.py and
tools/reference.py (tests/golden/make_golden.py); tests/test_oracle.py checks every function here
against them.
"""

from __future__ import annotations

import json
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

try:  # exact erf for GELU (reference: F.gelu, tools/reference.py:242)
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover - scipy ships in the image
    _erf = np.vectorize(math.erf, otypes=[np.float64])

D_MODEL = 2048
HEADS = 16
HEAD_DIM = 128
MLP = 8192
N_BLOCKS = 28
CONVROT_GROUP = 256  # tools/quant.py:18
W4_GROUP = 16  # tools/quant.py:19
# tools/quant.py:22-25: Lloyd-Max levels used by asym_w4a8_int8 when the kurtosis gate selects them
FIXED_LUT = np.array([
    -0.980602, -0.794529, -0.638165, -0.500986, -0.377321, -0.263187, -0.155210, -0.050720,
    0.052541, 0.156985, 0.265284, 0.379533, 0.502636, 0.638953, 0.794876, 0.980671,
], dtype=np.float32)

f32 = np.float32

# Row-wise elementwise work (the softmax of a score matrix, the GELU of the MLP hidden) runs over
# row chunks on a thread pool: numpy and scipy release the GIL inside these loops, and every row's
# result is computed by the same operations whatever the chunking, so the values do not depend on
# the thread count. Threads only: no process is forked.
_POOL = None


def _threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover - not Linux
        return max(1, os.cpu_count() or 1)


def _by_rows(fn, n_rows: int, min_rows: int = 64) -> None:
    """fn(r0, r1) for row chunks [r0, r1) covering [0, n_rows), on the pool when it pays."""
    global _POOL
    nt = _threads()
    if nt == 1 or n_rows < 2 * min_rows:
        fn(0, n_rows)
        return
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=nt)
    step = max(min_rows, -(-n_rows // nt))
    list(_POOL.map(lambda r0: fn(r0, min(n_rows, r0 + step)), range(0, n_rows, step)))


# ----------------------------------------------------------------------------- weight formats

def hadamard(size: int = CONVROT_GROUP) -> np.ndarray:
    """Normalized regular Hadamard matrix kron(H4, ..., H4)/sqrt(size) (tools/quant.py:30-38)."""
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=f32)
    h = h4
    while h.shape[0] < size:
        h = np.kron(h, h4)
    return (h / f32(math.sqrt(size))).astype(f32)


def rotate(w: np.ndarray, group: int = CONVROT_GROUP) -> np.ndarray:
    """ConvRot: w @ H^T per contiguous group of `group` columns (tools/quant.py:41-45)."""
    n, k = w.shape
    h = hadamard(group)
    return (w.astype(f32).reshape(n * (k // group), group) @ h.T).reshape(n, k)


def fp8_e4m3fn_table() -> np.ndarray:
    """fp8 e4m3fn byte -> fp32, as torch's float8_e4m3fn.float() (tools/quant.py:180).

    Same bit semantics as the WGSL decoder (app/gpu/gemm.js:144-151) except that 0x7f/0xff decode
    to NaN here, as in torch (the shader would give 480; quantize_w4a8 never emits them).
    """
    t = np.zeros(256, dtype=f32)
    for b in range(256):
        e, m = (b >> 3) & 15, b & 7
        v = m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7)
        if e == 15 and m == 7:
            v = float("nan")
        t[b] = -v if b & 128 else v
    return t


_FP8 = fp8_e4m3fn_table()


def unpack_w4_codes(packed: np.ndarray) -> np.ndarray:
    """uint8 [N, K/2] -> codes [N, K]; low nibble is the even k (tools/quant.py:162,173-178)."""
    p = packed.view(np.uint8).astype(np.int32)
    n, half = p.shape
    codes = np.empty((n, half * 2), dtype=np.int32)
    codes[:, 0::2] = p & 0xF
    codes[:, 1::2] = (p >> 4) & 0xF
    return codes


def decode_w4_grid(packed: np.ndarray, s_rel: np.ndarray, codebook: np.ndarray) -> np.ndarray:
    """int8-grid value of each 4-bit weight: clamp(rne(fp32(cb[code] * fp8(s_rel))), -127, 127).

    tools/quant.py:179-180 (also app/gpu/gemm.js:142 and app/webnn/dit.js:99-116). The product is
    one fp32 multiply and np.rint rounds half to even, as torch.round does.
    """
    codes = unpack_w4_codes(packed)
    n, k = codes.shape
    vals = codebook.astype(f32)[codes].reshape(n, k // W4_GROUP, W4_GROUP)
    s = _FP8[s_rel.view(np.uint8).astype(np.int64)].astype(f32)
    prod = (vals * s[..., None]).astype(f32)
    return np.clip(np.rint(prod), -127, 127).astype(f32).reshape(n, k)


def dequantize_int8_convrot(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """rotate(q * weight_scale) (tools/quant.py:81-83)."""
    return rotate(q.astype(f32) * scale.astype(f32).reshape(-1, 1))


def dequantize_w4a8(packed, s_rel, s_channel, codebook) -> np.ndarray:
    """rotate(grid * weight_s_channel) (tools/quant.py:172-182)."""
    grid = decode_w4_grid(packed, s_rel, codebook)
    return rotate(grid * s_channel.astype(f32).reshape(-1, 1))


def dequantize(t: dict) -> np.ndarray:
    """Dispatch on the comfy_quant metadata bytes (tools/quant.py:185-191)."""
    meta = json.loads(bytes(np.asarray(t["comfy_quant"], dtype=np.uint8).tolist()).decode())
    if meta["format"] == "int8_tensorwise":
        if not meta.get("convrot"):
            return t["weight"].astype(f32) * t["weight_scale"].astype(f32).reshape(-1, 1)
        return dequantize_int8_convrot(t["weight"], t["weight_scale"])
    if meta["format"] == "asym_w4a8_int8":
        return dequantize_w4a8(t["weight"], t["weight_s_rel"], t["weight_s_channel"], t["weight_codebook"])
    raise ValueError(f"unsupported quant format {meta['format']}")


# ----------------------------------------------------------------------------- math helpers

def rms_norm(x, w, eps=1e-6):
    """x * rsqrt(mean(x^2) + eps) * w (tools/reference.py:93-94)."""
    x = x.astype(f32)
    r = (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True, dtype=f32) + f32(eps))).astype(f32)
    return (x * r * w.astype(f32)).astype(f32)


def layer_norm(x, eps=1e-6):
    """LayerNorm without affine, biased variance (tools/reference.py:190-191)."""
    x = x.astype(f32)
    mu = np.mean(x, axis=-1, keepdims=True, dtype=f32)
    d = x - mu
    var = np.mean(d * d, axis=-1, keepdims=True, dtype=f32)
    return (d / np.sqrt(var + f32(eps))).astype(f32)


def rotate_half(x):
    """cat(-x[h:], x[:h]) on the last axis (tools/reference.py:97-99)."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def gelu(x):
    """Exact erf GELU, as F.gelu (tools/reference.py:242), evaluated in float64."""
    x = np.asarray(x)
    if x.ndim == 0:
        x64 = np.float64(x)
        return f32(0.5 * x64 * (1.0 + _erf(x64 / math.sqrt(2.0))))
    x2 = x.reshape(-1, x.shape[-1]) if x.ndim > 1 else x.reshape(1, -1)
    out = np.empty(x2.shape, dtype=f32)

    def rows(r0, r1):
        x64 = x2[r0:r1].astype(np.float64)
        out[r0:r1] = 0.5 * x64 * (1.0 + _erf(x64 / math.sqrt(2.0)))

    _by_rows(rows, x2.shape[0])
    return out.reshape(x.shape)


def silu(x):
    x64 = x.astype(np.float64)
    return (x64 / (1.0 + np.exp(-x64))).astype(f32)


def attention(q, k, v, key_len=None):
    """softmax(q k^T / sqrt(D)) v per head, non-causal (tools/reference.py:109-111).

    q [H, Lq, D], k/v [H, Lk, D]. key_len (optional) masks keys >= key_len: BASELINE's padded-text
    variant, which the reference itself never uses (it zero-pads the context to 512 rows instead,
    tools/reference.py:167-168).
    """
    H, Lq, D = q.shape
    out = np.empty((H, Lq, v.shape[-1]), dtype=f32)
    scale = f32(1.0 / math.sqrt(D))
    for h in range(H):  # fp32 with max subtraction, like the reference's fp32 SDPA on the CPU
        s = (q[h].astype(f32) @ k[h].astype(f32).T) * scale

        def softmax_rows(r0, r1, s=s):
            b = s[r0:r1]
            if key_len is not None:
                b[:, key_len:] = -np.inf
            b -= b.max(axis=-1, keepdims=True)
            np.exp(b, out=b)
            b /= b.sum(axis=-1, keepdims=True, dtype=f32)

        _by_rows(softmax_rows, Lq)
        out[h] = s @ v[h].astype(f32)
    return out


def dit_rope(H, W):
    """VideoRopePosition3DEmb angles for T=1 -> (cos, sin) [H*W, 64] (tools/reference.py:174-187).

    Slots 0..21 are temporal (angle 0), 22..42 height, 43..63 width; theta_h = 1e4 * 4^(42/40).
    Computed in fp32 like the reference's torch code.
    """
    head_dim = 128
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    sp = (np.arange(0, dim_h, 2, dtype=np.int64)[: dim_h // 2].astype(f32) / f32(dim_h)).astype(f32)
    h_theta = 10000.0 * 4.0 ** (dim_h / (dim_h - 2))
    hf = (f32(1.0) / np.power(f32(h_theta), sp, dtype=f32)).astype(f32)
    hh, ww = np.meshgrid(np.arange(H, dtype=f32), np.arange(W, dtype=f32), indexing="ij")
    ang = np.concatenate([np.zeros((H * W, dim_t // 2), dtype=f32),
                          hh.reshape(-1, 1) * hf, ww.reshape(-1, 1) * hf], axis=1).astype(f32)
    return np.cos(ang).astype(f32), np.sin(ang).astype(f32)


def timestep_embedding(sigma: float):
    """[1, 2048] = cat(cos(sigma f), sin(sigma f)), f_i = exp(-ln(1e4) i / 1024), in fp32
    (tools/reference.py:203-206). Note the model is fed sigma itself, not t * 1000."""
    half = D_MODEL // 2
    freqs = np.exp((f32(-math.log(10000)) * (np.arange(half, dtype=f32) / f32(half))).astype(f32)).astype(f32)
    t = (f32(sigma) * freqs).astype(f32)
    return np.concatenate([np.cos(t), np.sin(t)]).astype(f32)[None]


# ----------------------------------------------------------------------------- patches

def patchify(latent):
    """[16, h, w] + zero mask channel -> [L, 68] "(h w)(c m n)" (tools/reference.py:199-200)."""
    C, h, w = latent.shape
    Hp, Wp = h // 2, w // 2
    xin = np.concatenate([latent.astype(f32), np.zeros((1, h, w), dtype=f32)], 0)
    return xin.reshape(C + 1, Hp, 2, Wp, 2).transpose(1, 3, 0, 2, 4).reshape(Hp * Wp, (C + 1) * 4)


def unpatchify(o, h, w):
    """[L, 64] "(p1 p2 c)" -> [16, h, w] (tools/reference.py:249)."""
    Hp, Wp = h // 2, w // 2
    return o.reshape(Hp, Wp, 2, 2, 16).transpose(4, 0, 2, 1, 3).reshape(16, h, w)


# ----------------------------------------------------------------------------- DiT

def time_cond(W, sigma):
    """(temb, adaln_lora [1,6144], emb [1,2048]) (tools/reference.py:203-208)."""
    temb = timestep_embedding(sigma)
    adaln_lora = silu(temb @ W("t_embedder.1.linear_1.weight").T) @ W("t_embedder.1.linear_2.weight").T
    emb = rms_norm(temb, W("t_embedding_norm.weight"))
    return temb, adaln_lora.astype(f32), emb


def block_mod(W, p, emb, adaln_lora):
    """AdaLN-LoRA modulation -> (shift, scale, gate) (tools/reference.py:218-220)."""
    m = (silu(emb) @ W(p + ".1.weight").T) @ W(p + ".2.weight").T + adaln_lora
    return np.split(m.astype(f32), 3, axis=-1)


def _attn(W, p, xq, c, cos, sin, rope, key_len=None):
    """tools/reference.py:222-230."""
    Lq, Lk = xq.shape[0], c.shape[0]
    q = rms_norm((xq @ W(p + "q_proj.weight").T).reshape(Lq, HEADS, HEAD_DIM), W(p + "q_norm.weight")).transpose(1, 0, 2)
    k = rms_norm((c @ W(p + "k_proj.weight").T).reshape(Lk, HEADS, HEAD_DIM), W(p + "k_norm.weight")).transpose(1, 0, 2)
    v = (c @ W(p + "v_proj.weight").T).reshape(Lk, HEADS, HEAD_DIM).transpose(1, 0, 2)
    if rope:
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
    a = attention(q, k, v, key_len).transpose(1, 0, 2).reshape(Lq, D_MODEL)
    return a @ W(p + "output_proj.weight").T


def dit_block(W, i, x, ctx, emb, adaln_lora, cos, sin, key_len=None):
    """One transformer block, the body of tools/reference.py:232-242 (cos/sin already doubled to 128)."""
    p = f"blocks.{i}."
    sh, sc, g = block_mod(W, p + "adaln_modulation_self_attn", emb, adaln_lora)
    n = layer_norm(x) * (1 + sc) + sh
    x = x + g * _attn(W, p + "self_attn.", n, n, cos, sin, True)
    sh, sc, g = block_mod(W, p + "adaln_modulation_cross_attn", emb, adaln_lora)
    n = layer_norm(x) * (1 + sc) + sh
    x = x + g * _attn(W, p + "cross_attn.", n, ctx, cos, sin, False, key_len)
    sh, sc, g = block_mod(W, p + "adaln_modulation_mlp", emb, adaln_lora)
    n = layer_norm(x) * (1 + sc) + sh
    x = x + g * (gelu(n @ W(p + "mlp.layer1.weight").T) @ W(p + "mlp.layer2.weight").T)
    return x.astype(f32)


def dit_forward(W, latent, sigma, ctx, dump=None, n_blocks=N_BLOCKS, key_len=None):
    """Velocity [16, h, w] for latent [16, h, w] (tools/reference.py:194-249).

    W(name) -> fp32 array (dequantized). n_blocks < 28 runs a prefix of the stack (test speed).
    """
    C, h, w = latent.shape
    H, Wp = h // 2, w // 2
    x = (patchify(latent) @ W("x_embedder.proj.1.weight").T).astype(f32)
    temb, adaln_lora, emb = time_cond(W, sigma)
    if dump is not None:
        dump["dit_x_embed"] = x
        dump["dit_emb"] = emb
        dump["dit_adaln_lora"] = adaln_lora
    cos, sin = dit_rope(H, Wp)
    cos = np.concatenate([cos, cos], -1)
    sin = np.concatenate([sin, sin], -1)
    for i in range(n_blocks):
        x = dit_block(W, i, x, ctx, emb, adaln_lora, cos, sin, key_len)
        if dump is not None and i == 0:
            dump["dit_block0"] = x
    m = (silu(emb) @ W("final_layer.adaln_modulation.1.weight").T) @ W("final_layer.adaln_modulation.2.weight").T \
        + adaln_lora[:, : 2 * D_MODEL]
    sh, sc = np.split(m.astype(f32), 2, axis=-1)
    o = (layer_norm(x) * (1 + sc) + sh) @ W("final_layer.linear.weight").T
    return unpatchify(o.astype(f32), h, w)


# ----------------------------------------------------------------------------- sampling

def sigmas_simple(steps: int, shift: float):
    """ComfyUI "simple" schedule over the shift-3 flow table, rounded through fp32
    (tools/reference.py:300-303; app/samplers.js:16-23)."""
    table = [shift * t / (1 + (shift - 1) * t) for t in (np.arange(1, 1001) / 1000.0)]
    ss = 1000 / steps
    return [float(np.float32(table[-(1 + int(x * ss))])) for x in range(steps)] + [0.0]


def euler_sample(W, noise, ctx, steps, cfg=1.0, ctx_neg=None, n_blocks=N_BLOCKS, key_len=None, dump=None):
    """Deterministic Euler flow sampling with optional CFG (tools/reference.py:349-360)."""
    sig = sigmas_simple(steps, 3.0)
    x = (noise * f32(sig[0])).astype(f32)
    for i in range(steps):
        s = sig[i]
        v = dit_forward(W, x, s, ctx, dump=dump if i == 0 else None, n_blocks=n_blocks, key_len=key_len)
        if dump is not None and i == 0:
            dump["velocity0"] = v
        if ctx_neg is not None:
            vn = dit_forward(W, x, s, ctx_neg, n_blocks=n_blocks, key_len=key_len)
            v = vn + (v - vn) * f32(cfg)
        den = (x - v * f32(s)).astype(f32)
        if dump is not None and i == 0:
            dump["denoised0"] = den
        x = den if sig[i + 1] == 0 else (x + (x - den) / f32(s) * f32(sig[i + 1] - s)).astype(f32)
    return x


class DequantWeights:
    """W(name) over a dict of comfy_quant tensors, dequantizing quantized linears on access and
    caching the fp32 result (tools/reference.py:30-45 without the per-access cost)."""

    def __init__(self, tensors: dict, prefix: str = "", cache: bool = True):
        self.t = tensors
        self.prefix = prefix
        self.cache = {} if cache else None

    def __call__(self, name):
        if self.cache is not None and name in self.cache:
            return self.cache[name]
        k = self.prefix + name
        base = k[: -len("weight")] if k.endswith("weight") else None
        if base is not None and base + "comfy_quant" in self.t:
            parts = {s: self.t[base + s] for s in ("weight", "weight_scale", "weight_s_rel", "weight_s_channel", "weight_codebook", "comfy_quant") if base + s in self.t}
            w = dequantize(parts)
        else:
            w = np.asarray(self.t[k]).astype(f32)
        if self.cache is not None:
            self.cache[name] = w
        return w

    def has(self, name) -> bool:
        return self.prefix + name in self.t


class LoraMerged:
    """W(name) + sum_e scale_e * B_e @ A_e for matching linears (tools/reference.py:51-90).

    deltas: {module_name: [(scale, B [n, r], A [r, K])]} with module names as in the checkpoint
    (e.g. "blocks.0.self_attn.q_proj").
    """

    def __init__(self, base, deltas: dict):
        self.base = base
        self.deltas = deltas

    def __call__(self, name):
        w = self.base(name)
        if name.endswith(".weight"):
            for scale, B, A in self.deltas.get(name[: -len(".weight")], []):
                w = (w + f32(scale) * (B.astype(f32) @ A.astype(f32))).astype(f32)
        return w
