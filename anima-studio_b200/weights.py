"""Linear weights in the ComfyUI comfy_quant layout, resident on the GPU (app/weights.js:118-189).

A Linear mirrors the reference's weight object {kind, N, K, buf, scale, srel, codebook, bias}:
  kind "i8"   int8 codes [N, K] + per-row weight_scale           (int8_tensorwise + convrot)
  kind "w4"   decoded once at load to its int8-grid values [N, K] + weight_s_channel; the packed
              nibbles, fp8 group scales and codebook are kept (asym_w4a8_int8 + convrot)
  kind "bf16" / "f32"  unquantized weights (embedders, adaLN, final layer, LoRA A/B)
The reference decodes 4-bit weights inside its GEMM tile loader (app/gpu/gemm.js:141-158); here the
decode runs once per load on the GPU (anima_unpack_w4, bit-exact) and the int8 tensor-core GEMM
consumes the grid directly.
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
    data: torch.Tensor                    # int8 [N, K] (i8/w4 grid) or bf16/f32 [N, K]
    scale: torch.Tensor | None = None     # fp32 [N]
    bias: torch.Tensor | None = None
    packed: torch.Tensor | None = None    # w4: uint8 [N, K/2]
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
        w.kind = {"i8": dev.W_I8, "w4": dev.W_I8, "bf16": dev.W_BF16, "f32": dev.W_F32}[self.kind]
        w.N, w.K = self.N, self.K
        w.data = self.data.data_ptr()
        w.scale = self.scale.data_ptr() if self.scale is not None else 0
        w.bias = self.bias.data_ptr() if self.bias is not None else 0
        return w


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
            from .ops import unpack_w4
            grid = unpack_w4(packed, srel, cb, N, K)
            sch = tensors[base + "weight_s_channel"].to(device=device, dtype=torch.float32).reshape(-1).contiguous()
            return Linear("w4", N, K, grid, sch, bias, packed=packed, s_rel=srel, codebook=cb, name=name)
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
    (weights.js:152-189). Rows are independent, so per-row scales concatenate. Decoded W4 grids
    stack too (the reference additionally requires one shared codebook because it decodes in the
    GEMM; ours are decoded already, but the rule is kept so stacking means the same thing)."""
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
        out.packed = torch.cat([w.packed for w in Ws], 0)
        out.s_rel = torch.cat([w.s_rel for w in Ws], 0)
        out.codebook = Ws[0].codebook
    return out
