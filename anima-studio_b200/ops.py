"""The operator surface of the reference's app/gpu/ops.js, on the B200 kernels of libanima_b200.

Activations follow the reference's conventions (row-major, fp32 unless a fused path says
otherwise); names and argument meanings mirror ops.js, each function cites the line it stands in
for. Two B200-specific forms are added for the fused path the DiT uses:

  QuantRows   rotated + per-token quantized rows, x ~= scale * (hi + lo / 254) (lo optional);
              the "xr" input of a ConvRot linear in the reference (ops.js:48-54)
  layernorm_mod_quant / rotate_quant   produce QuantRows directly from the norm / the rotation

Everything runs on the current torch stream of the tensors' device; nothing falls back to the CPU.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import torch

from . import device as dev
from .device import ctx_for, ptr


@dataclass
class QuantRows:
    """Per-token quantized rotated activations [rows, cols]: x ~= scale[:, None] * (hi + lo / 254)."""

    hi: torch.Tensor
    lo: torch.Tensor | None
    scale: torch.Tensor

    @property
    def rows(self):
        return self.hi.shape[0]

    @property
    def cols(self):
        return self.hi.shape[1]

    @staticmethod
    def empty(rows: int, cols: int, planes: int = 2, device=None) -> "QuantRows":
        hi = torch.empty(rows, cols, dtype=torch.int8, device=device)
        lo = torch.empty(rows, cols, dtype=torch.int8, device=device) if planes == 2 else None
        return QuantRows(hi, lo, torch.empty(rows, dtype=torch.float32, device=device))

    def c(self) -> dev.QAct:
        return dev.QAct(self.rows, self.cols, self.hi.stride(0), self.hi.data_ptr(),
                        self.lo.data_ptr() if self.lo is not None else 0, self.scale.data_ptr())

    def dequant(self) -> torch.Tensor:
        """fp32 rows this encodes (for tests and debugging)."""
        x = self.hi.float()
        if self.lo is not None:
            x = x + self.lo.float() / 254.0
        return x * self.scale[:, None]


def _dt(t: torch.Tensor) -> int:
    return dev.DTYPE_CODE[t.dtype]


def _contig_rows(t: torch.Tensor):
    if t.dim() != 2 or t.stride(1) != 1:
        raise dev.AnimaError(1, "expected a 2-D tensor with contiguous rows")


# ----------------------------------------------------------------------------- rotation / norms

def rotate(x: torch.Tensor) -> torch.Tensor:
    """ConvRot input rotation, y = x H per 256 features (ops.js:38-44)."""
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.empty_like(x2, dtype=torch.float32)
    ctx_for(x).call("anima_rotate", ptr(x2), _dt(x2), x2.shape[0], x2.shape[1], x2.stride(0), ptr(y), dev.ANIMA_F32)
    return y.view(x.shape)


def rotate_quant(x: torch.Tensor, planes: int = 2, out: QuantRows | None = None, act: str | None = None) -> QuantRows:
    """rotate() fused with per-token quantization (input fp32/bf16/fp16 rows); act="gelu" applies
    the MLP activation first (for a layer1 GEMM that stored its pre-activation)."""
    _contig_rows(x)
    q = out or QuantRows.empty(x.shape[0], x.shape[1], planes, x.device)
    qa = q.c()
    if act:
        ctx_for(x).call("anima_act_rotate_quant", ptr(x), _dt(x), x.shape[0], x.shape[1], x.stride(0), dev.ACT[act],
                        C.byref(qa))
    else:
        ctx_for(x).call("anima_rotate_quant", ptr(x), _dt(x), x.shape[0], x.shape[1], x.stride(0), C.byref(qa))
    return q


def quant_rows(x: torch.Tensor, planes: int = 2, out: QuantRows | None = None) -> QuantRows:
    """Per-token quantization of already-rotated rows."""
    _contig_rows(x)
    q = out or QuantRows.empty(x.shape[0], x.shape[1], planes, x.device)
    qa = q.c()
    ctx_for(x).call("anima_quant_rows", ptr(x), _dt(x), x.shape[0], x.shape[1], x.stride(0), C.byref(qa))
    return q


def layernorm_mod(x: torch.Tensor, mod: torch.Tensor, shift_off: int, scale_off: int, cols: int,
                  rotate: bool = False, eps: float = 1e-6, out_dtype=torch.float32) -> torch.Tensor:
    """y = LN(x) * (1 + mod[scale_off:]) + mod[shift_off:] (+ ConvRot) (ops.js:129-137)."""
    rows = x.numel() // cols
    y = torch.empty(rows, cols, dtype=out_dtype, device=x.device)
    ctx_for(x).call("anima_layernorm_mod", ptr(x), rows, cols, ptr(mod), shift_off, scale_off, C.c_float(eps),
                    1 if rotate else 0, ptr(y), dev.DTYPE_CODE[out_dtype])
    return y


def layernorm_mod_quant(x: torch.Tensor, mod: torch.Tensor, shift_off: int, scale_off: int, cols: int,
                        planes: int = 2, eps: float = 1e-6, out: QuantRows | None = None) -> QuantRows:
    """layernorm_mod(rotate=True) fused with per-token quantization: the "xr" a ConvRot linear takes."""
    rows = x.numel() // cols
    q = out or QuantRows.empty(rows, cols, planes, x.device)
    qa = q.c()
    ctx_for(x).call("anima_layernorm_mod_quant", ptr(x), rows, cols, ptr(mod), shift_off, scale_off,
                    C.c_float(eps), C.byref(qa))
    return q


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, cols: int, eps: float = 1e-6, out=None,
            out_dtype=None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * w over rows of `cols` (ops.js:111-117)."""
    rows = x.numel() // cols
    y = out if out is not None else torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    ctx_for(x).call("anima_rmsnorm", ptr(x), _dt(x), rows, cols, ptr(weight), C.c_float(eps), ptr(y), _dt(y))
    return y


def qk_norm_rope(qkv: torch.Tensor, qn: torch.Tensor, kn: torch.Tensor, cs: torch.Tensor, L: int, H: int, D: int,
                 eps: float = 1e-6):
    """In-place per-head RMSNorm + RoPE on the q and k parts of qkv [L, 3 H D] (ops.js:140-145).
    cs: cos table [rows, D/2] followed by the sin table (rows = L or a divisor pattern)."""
    rows = cs.numel() // D
    ctx_for(qkv).call("anima_qk_norm_rope", ptr(qkv), _dt(qkv), L, H, D, qkv.stride(0), ptr(qn), ptr(kn), ptr(cs),
                      rows, C.c_float(eps))


def rope(x: torch.Tensor, cs: torch.Tensor, L: int, H: int, D: int, row_stride: int | None = None, col_off: int = 0):
    """In-place split-half RoPE on x viewed as [L, H, D] (ops.js:148-152)."""
    rows = cs.numel() // D
    ctx_for(x).call("anima_rope", ptr(x), _dt(x), L, H, D, row_stride or H * D, col_off, ptr(cs), rows)


def elementwise(op: str, a: torch.Tensor, b: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """silu | copy | add | silu_mul over fp32 elements (ops.js:154-160)."""
    code = {"copy": 0, "add": 1, "silu": 2, "silu_mul": 3}[op]
    y = out if out is not None else torch.empty_like(a)
    n = min(y.numel(), a.numel())
    ctx_for(a).call("anima_elementwise", code, ptr(a), ptr(b), ptr(y), n)
    return y


def conv3x3(x: torch.Tensor, W, h: int, w: int, up: bool = False, into: torch.Tensor | None = None) -> torch.Tensor:
    """NHWC 3x3 convolution, pad 1, of x [h w, cin] with W (bf16 OHWI as [N, 9 cin], + bias); up:
    nearest 2x upsample first; into: out += conv (ops.js:97-109, conv3x3 / conv3x3Into)."""
    H, Wd = (2 * h, 2 * w) if up else (h, w)
    out = into if into is not None else torch.empty(H * Wd, W.N, dtype=torch.float32, device=x.device)
    wc = W.c()
    ctx_for(x).call("anima_conv3x3", ptr(x), h, w, W.K // 9, C.byref(wc), 1 if up else 0, ptr(out),
                    1 if into is not None else 0)
    return out


def channel_norm(x: torch.Tensor, gamma: torch.Tensor, cols: int, silu: bool) -> torch.Tensor:
    """The Wan VAE's RMS_norm over channels, then SiLU (ops.js:120-126)."""
    y = torch.empty_like(x)
    ctx_for(x).call("anima_channel_norm", ptr(x), x.numel() // cols, cols, ptr(gamma), 1 if silu else 0, ptr(y))
    return y


def zero(t: torch.Tensor):
    """ops.zero (ops.js:89-93)."""
    ctx_for(t).call("anima_zero", ptr(t), t.numel() * t.element_size())


# ----------------------------------------------------------------------------- linears

def linear(x, W, *, out: torch.Tensor | None = None, resid: bool = False, gate: torch.Tensor | None = None,
           g_off: int = 0, act: str | None = None, add: torch.Tensor | None = None, out_dtype=torch.float32,
           mode: str = "store", qk=None, rope_cs: torch.Tensor | None = None, n_q: int = 0, eps: float = 1e-6,
           planes: int = 2, name: str | None = None, peer=None) -> torch.Tensor:
    """y = x @ W^T (+ bias) (+ add) (act); or out += gate[g_off + n] * y when resid (ops.js:48-66).

    x: QuantRows (rotated, quantized) for ConvRot weights, or an fp32 tensor (rotated and quantized
    here, like ops.linear rotating when no xr is given). LoRA side paths attached to W are added
    before the activation, as the reference does (ops.js:55-57).
    mode: "store" | "qkv" (per-head RMSNorm + RoPE on q/k heads, qk = (qn, kn)) |
          "head_norm" (per-head RMSNorm with qk[0]).
    peer (mode "qkv"): {"kv": [device addresses of every rank's gathered k|v buffer], "row0", "rows",
          "item_rows"}: the k|v columns go to those buffers over NVLink instead of to `out`
          (sharding.KVExchange; anima_linear_opts.peer_*).
    """
    from . import lora as lora_mod

    if W.kind in ("bf16", "f32"):
        return matmul(x, W, act=act, out=out, resid=resid, gate=gate, g_off=g_off)
    if not isinstance(x, QuantRows):
        x = rotate_quant(x.reshape(-1, W.K).contiguous(), planes)
    M = x.rows
    o = dev.LinearOpts()
    keep = None
    if W.lora:
        if lora_mod.PATH == "fused":
            keep = lora_mod.lora_epilogue(x, W, o)   # T B^T inside the GEMM epilogue (None: entries it
        if keep is None:                             # cannot take, which get an added delta)
            delta = lora_mod.lora_delta_tc(x, W) if lora_mod.PATH == "delta" else lora_mod.lora_delta(x, W)
            add = delta if add is None else add + delta
    if out is None:
        if resid:
            raise dev.AnimaError(1, "resid=True needs out")
        out = torch.empty(M, W.N, dtype=out_dtype, device=x.hi.device)
    o.act = dev.ACT[act]
    o.add = add.data_ptr() if add is not None else 0
    o.ld_add = add.stride(0) if add is not None else 0
    o.out_mode = dev.OUT_RESID if resid else {"store": dev.OUT_STORE, "qkv": dev.OUT_QKV_NORM_ROPE,
                                              "head_norm": dev.OUT_HEAD_NORM}[mode]
    o.out_dtype = _dt(out)
    o.out = out.data_ptr()
    o.ldo = out.stride(0)
    o.gate = gate.data_ptr() if gate is not None else 0
    o.gate_off = g_off
    if qk is not None:
        o.norm_q = qk[0].data_ptr()
        o.norm_k = qk[1].data_ptr() if len(qk) > 1 and qk[1] is not None else 0
    if rope_cs is not None:
        o.rope = rope_cs.data_ptr()
        o.rope_rows = rope_cs.numel() // 128
    o.n_q = n_q
    o.eps = eps
    if peer is not None:
        o.peer_count = len(peer["kv"])
        for r, a in enumerate(peer["kv"]):
            o.peer_kv[r] = a
        o.peer_row0, o.peer_rows, o.peer_item_rows = peer["row0"], peer["rows"], peer["item_rows"]
    qa = x.c()
    w = W.c()
    ctx_for(x.hi).call("anima_linear", C.byref(qa), C.byref(w), C.byref(o), tag=name, work=2.0 * M * W.N * W.K,
                       kernels=2 if W.kind == "w4" else 1)  # w4: the decode, then the GEMM
    del keep
    return out


def matmul(x: torch.Tensor, W, *, act: str | None = None, out: torch.Tensor | None = None, resid: bool = False,
           gate: torch.Tensor | None = None, g_off: int = 0, alpha: float = 1.0) -> torch.Tensor:
    """runMatmul for bf16/f32 weights (ops.js:14-33): small SIMT GEMM, fp32 accumulate."""
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    if out is None:
        if resid:
            raise dev.AnimaError(1, "resid=True needs out")
        out = torch.empty(M, W.N, dtype=torch.float32, device=x.device)
    w = W.c()
    ctx_for(x).call("anima_matmul", M, W.N, K, C.c_float(alpha), ptr(x2), x2.stride(0), C.byref(w), dev.ACT[act],
                    ptr(out), out.stride(0), 1 if resid else 0, ptr(gate), g_off)
    return out


# ----------------------------------------------------------------------------- attention

def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, Lq: int, Lk: int, H: int, D: int = 128,
              ldq: int | None = None, ldk: int | None = None, ldv: int | None = None, q_off: int = 0,
              k_off: int = 0, v_off: int = 0, batch: int = 1, q_bstride: int = 0, k_bstride: int = 0,
              v_bstride: int = 0, key_len: torch.Tensor | None = None, out: torch.Tensor | None = None,
              out_dtype=None, o_bstride: int | None = None, scale: float | None = None,
              name: str | None = None, noalloc: bool = False, group: int = 1, causal: bool = False) -> torch.Tensor:
    """Non-causal multi-head attention (ops.js:166-208): q [.., ldq] with head h at q_off + h D,
    k/v likewise; output [batch * Lq, H D]. q/k/v are bf16 or fp16; key_len (int32 [batch]) masks
    keys past each item's text length. noalloc: the entry point whose stream-K workspace is the
    library's static device array (no allocation; calls must not overlap). group: q heads per k/v
    head (GQA); causal: query i sees keys j <= i; with either, or D = 64, or fp32 q/k/v, the
    text-model kernel runs (ops.js:166-208 takes the same `group` and `causal`)."""
    ldq = ldq or H * D
    ldk = ldk or (H // max(group, 1)) * D
    ldv = ldv or (H // max(group, 1)) * D
    if out is None:
        out = torch.empty(batch * Lq, H * D, dtype=out_dtype or q.dtype, device=q.device)
    a = dev.AttentionArgs()
    a.batch, a.heads, a.head_dim, a.Lq, a.Lk = batch, H, D, Lq, Lk
    a.dtype = _dt(q)
    a.q, a.ldq, a.q_bstride, a.q_off = q.data_ptr(), ldq, q_bstride, q_off
    a.k, a.ldk, a.k_bstride, a.k_off = k.data_ptr(), ldk, k_bstride, k_off
    a.v, a.ldv, a.v_bstride, a.v_off = v.data_ptr(), ldv, v_bstride, v_off
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.o_bstride = o_bstride if o_bstride is not None else Lq * out.stride(0)
    a.out_dtype = _dt(out)
    a.key_len = key_len.data_ptr() if key_len is not None else 0
    a.scale = scale if scale is not None else 1.0 / math.sqrt(D)
    a.group, a.causal = int(group), 1 if causal else 0
    ctx_for(q).call("anima_attention_noalloc" if noalloc else "anima_attention", C.byref(a), tag=name,
                    work=4.0 * batch * Lq * Lk * D * H)
    return out


# ----------------------------------------------------------------------------- model glue

def patchify(latent: torch.Tensor) -> torch.Tensor:
    """[B, 16, h, w] -> [B (h/2)(w/2), 68] with the zero mask channel (dit.js:55-65)."""
    B, _, h, w = latent.shape
    out = torch.empty(B * (h // 2) * (w // 2), 68, dtype=torch.float32, device=latent.device)
    ctx_for(latent).call("anima_patchify", ptr(latent), B, h, w, ptr(out))
    return out


def unpatchify(o: torch.Tensor, B: int, h: int, w: int) -> torch.Tensor:
    """[B (h/2)(w/2), 64] -> [B, 16, h, w] (dit.js:68-78)."""
    out = torch.empty(B, 16, h, w, dtype=torch.float32, device=o.device)
    ctx_for(o).call("anima_unpatchify", ptr(o), B, h, w, ptr(out))
    return out


def timestep_embedding(sigmas: torch.Tensor) -> torch.Tensor:
    """[S] sigmas -> [S, 2048] sinusoidal embeddings (dit.js:41-51)."""
    out = torch.empty(sigmas.numel(), 2048, dtype=torch.float32, device=sigmas.device)
    ctx_for(sigmas).call("anima_timestep_embedding", ptr(sigmas), sigmas.numel(), ptr(out))
    return out


def euler_step(x: torch.Tensor, v: torch.Tensor, sigma: float, sigma_next: float, v_uncond=None, cfg: float = 1.0,
               den_out: torch.Tensor | None = None):
    """In place: CFG combine, x0 = x - sigma v, Euler step (pipeline.js:260-269, samplers.js:109-117)."""
    ctx_for(x).call("anima_euler_step", ptr(x), ptr(v), ptr(v_uncond), C.c_float(cfg), C.c_float(sigma),
                    C.c_float(sigma_next), x.numel(), ptr(den_out))
    return x


def lincomb(out: torch.Tensor, *terms) -> torch.Tensor:
    """out = sum of c * t over up to four (c, t) pairs of fp32 tensors with out's element count; out
    may be one of the t (the samplers' axpby, samplers.js:97-101)."""
    if not 1 <= len(terms) <= 4:
        raise ValueError("lincomb takes one to four (coefficient, tensor) terms")
    xs = [C.c_void_p(0)] * 4
    cs = (C.c_float * 4)(0.0, 0.0, 0.0, 0.0)
    for k, (c, t) in enumerate(terms):
        if t.dtype != torch.float32 or t.numel() != out.numel() or not t.is_contiguous():
            raise dev.AnimaError(1, "lincomb: terms must be contiguous fp32 tensors of out's size")
        xs[k] = ptr(t)
        cs[k] = float(c)
    ctx_for(out).call("anima_lincomb", ptr(out), out.numel(), *xs, cs)
    return out


def unpack_w4(packed: torch.Tensor, s_rel: torch.Tensor, codebook: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """4-bit codes -> int8-grid values [N, K], bit-exact with tools/quant.py:179-180."""
    out = torch.empty(N, K, dtype=torch.int8, device=packed.device)
    ctx_for(packed).call("anima_unpack_w4", ptr(packed), ptr(s_rel), ptr(codebook), N, K, ptr(out))
    return out
