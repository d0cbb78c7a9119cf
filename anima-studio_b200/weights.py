"""Linear weights in the ComfyUI comfy_quant layout, resident on the GPU (app/weights.js:118-189).

A Linear mirrors the reference's weight object {kind, N, K, buf, scale, srel, codebook, bias}:
  kind "i8"   int8 codes [N, K] + per-row weight_scale           (int8_tensorwise + convrot)
  kind "w4"   packed nibbles [N, K/2] + fp8 group scales [N, K/16] + codebook [16] +
              weight_s_channel (asym_w4a8_int8 + convrot), resident as stored: 0.5 byte a weight
  kind "bf16" / "f32"  unquantized weights (embedders, adaLN, final layer, LoRA A/B)
The reference decodes 4-bit weights inside its GEMM tile loader (app/gpu/gemm.js:141-158). Here
anima_linear decodes a W4 layer to its int8 grid (bit-exact, the arithmetic of anima_unpack_w4)
into a context-owned buffer just before the int8 tensor-core GEMM of that layer: at the DiT's
4096+ token rows every weight tile feeds 32+ row tiles, so decoding it once per call costs about
1/32 of decoding it in every CTA's shared-memory producer.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import device as dev
from . import quant


@dataclass
class Linear:
    kind: str
    N: int
    K: int
    data: torch.Tensor                    # int8 [N, K] (i8), packed uint8 [N, K/2] (w4) or bf16/f32 [N, K]
    scale: torch.Tensor | None = None     # fp32 [N]
    bias: torch.Tensor | None = None
    s_rel: torch.Tensor | None = None     # w4: fp8 bytes [N, K/16]
    codebook: torch.Tensor | None = None  # w4: fp32 [16]
    name: str = ""
    parts: list = field(default_factory=list)   # [(name, off, n)] of stacked linears
    lora: list = field(default_factory=list)    # attached LoRA entries (lora.attach_loras)

    @property
    def quantized(self) -> bool:
        return self.kind in ("i8", "w4")

    def c(self) -> dev.Weight:
        w = dev.Weight()
        w.kind = {"i8": dev.W_I8, "w4": dev.W_W4, "bf16": dev.W_BF16, "f32": dev.W_F32, "f16": dev.W_F16}[self.kind]
        w.N, w.K = self.N, self.K
        w.data = self.data.data_ptr()
        w.scale = self.scale.data_ptr() if self.scale is not None else 0
        w.bias = self.bias.data_ptr() if self.bias is not None else 0
        if self.kind == "w4":
            w.s_rel = self.s_rel.data_ptr()
            w.codebook = self.codebook.data_ptr()
        return w

    def grid(self) -> torch.Tensor:
        """The int8 values the tensor cores multiply: the codes (i8) or the decoded W4 grid."""
        if self.kind == "i8":
            return self.data
        if self.kind == "w4":
            from .ops import unpack_w4
            return unpack_w4(self.data, self.s_rel, self.codebook, self.N, self.K)
        raise ValueError(f"{self.name}: kind {self.kind} has no int8 grid")

    def nbytes(self) -> int:
        """Device bytes of the stored weight (codes, scales, bias)."""
        ts = (self.data, self.scale, self.bias, self.s_rel, self.codebook)
        return sum(t.numel() * t.element_size() for t in ts if t is not None)


def needs_rotation(W: Linear) -> bool:
    """ConvRot layers take rotated inputs (ops.js:35)."""
    return W.quantized


def linear_weights(tensors: dict, base: str, device="cuda") -> Linear:
    """<base>weight (+ comfy_quant companions, + <base>bias) -> Linear on `device` (weights.js:118-146)."""
    w = tensors[base + "weight"]
    bias = tensors.get(base + "bias")
    bias = bias.to(device=device, dtype=torch.float32).contiguous() if bias is not None else None
    meta = quant.meta_of(tensors, base)
    name = base[:-1] if base.endswith(".") else base
    if meta is not None:
        if not meta.get("convrot"):
            raise ValueError(f"{base}: only ConvRot-quantized linears are supported")
        if meta["format"] == "int8_tensorwise":
            return Linear("i8", w.shape[0], w.shape[1], w.to(device).contiguous(),
                          tensors[base + "weight_scale"].to(device=device, dtype=torch.float32).reshape(-1).contiguous(),
                          bias, name=name)
        if meta["format"] == "asym_w4a8_int8":
            N, K = w.shape[0], w.shape[1] * 2
            packed = w.view(torch.uint8).to(device).contiguous()
            srel = tensors[base + "weight_s_rel"].view(torch.uint8).to(device).contiguous()
            cb = tensors[base + "weight_codebook"].to(device=device, dtype=torch.float32).contiguous()
            sch = tensors[base + "weight_s_channel"].to(device=device, dtype=torch.float32).reshape(-1).contiguous()
            return Linear("w4", N, K, packed, sch, bias, s_rel=srel, codebook=cb, name=name)
        raise ValueError(f"unsupported quant format {meta['format']}")
    if w.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"expected a bf16/f32 weight for {base}, got {w.dtype}")
    N = w.shape[0]
    K = w.numel() // N
    kind = "bf16" if w.dtype == torch.bfloat16 else "f32"
    return Linear(kind, N, K, w.reshape(N, K).to(device).contiguous(), None, bias, name=name)


def vector(tensors: dict, name: str, device="cuda") -> torch.Tensor:
    """A 1-D parameter as fp32 on the device (weights.js:106-108)."""
    return tensors[name].to(device=device, dtype=torch.float32).contiguous()


def concat_linears(Ws: list[Linear]) -> Linear | None:
    """Stack linears sharing an input into one [sum N, K] weight, e.g. q, k, v -> qkv
    (weights.js:152-189). Rows are independent, so per-row scales concatenate; W4 rows stack with
    their fp8 group scales when every part has the same codebook (one codebook per decode, as in
    the reference)."""
    kind, K = Ws[0].kind, Ws[0].K
    if not all(w.kind == kind and w.K == K and w.bias is None for w in Ws):
        return None
    if kind == "w4" and not all(torch.equal(w.codebook, Ws[0].codebook) for w in Ws):
        return None
    out = Linear(kind, sum(w.N for w in Ws), K, torch.cat([w.data for w in Ws], 0).contiguous(),
                 torch.cat([w.scale for w in Ws]).contiguous() if Ws[0].scale is not None else None, None,
                 name="+".join(w.name for w in Ws))
    off = 0
    for w in Ws:
        out.parts.append((w.name, off, w.N))
        off += w.N
    if kind == "w4":
        out.s_rel = torch.cat([w.s_rel for w in Ws], 0).contiguous()
        out.codebook = Ws[0].codebook
    return out
