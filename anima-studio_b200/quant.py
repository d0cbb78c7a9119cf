"""Offline ConvRot quantizers producing the ComfyUI comfy_quant layout (torch, CPU or CUDA).

Restates the two weight formats of the reference's offline tool (tools/quant.py), which the
reference ports from comfy_kitchen's eager backend (not vendored, no pinned version):

  int8_tensorwise + convrot : per-output-row int8 of the Hadamard-rotated weight (quant.py:59-67)
  asym_w4a8_int8  + convrot : 4-bit codes into a 16-level codebook, fp8-e4m3 scale per group of
                              16, fp32 per-row scale, decoded on an int8 grid (quant.py:132-169)

These run once, offline, to build weights for tests and benchmarks; they are not on the denoising
path. tests/test_host.py checks them bit for bit against the reference's outputs (fixtures in
tests/golden/ written by the reference's own quantizers).
"""

from __future__ import annotations

import json
import math

import torch

CONVROT_GROUP = 256
W4_GROUP = 16
FIXED_LUT = (
    -0.980602, -0.794529, -0.638165, -0.500986, -0.377321, -0.263187, -0.155210, -0.050720,
    0.052541, 0.156985, 0.265284, 0.379533, 0.502636, 0.638953, 0.794876, 0.980671,
)
_ALS_ITERS = 2
_GATE_KURTOSIS = -0.1


def hadamard(size: int, device=None, dtype=torch.float32) -> torch.Tensor:
    """kron(H4, ..., H4) / sqrt(size) with H4 the regular symmetric 4x4 Hadamard (quant.py:30-38)."""
    if size < 4 or 4 ** round(math.log(size, 4)) != size:
        raise ValueError(f"size must be a power of 4, got {size}")
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=dtype, device=device)
    h = h4
    while h.shape[0] < size:
        h = torch.kron(h, h4)
    return h / math.sqrt(size)


def rotate(weight: torch.Tensor, group: int = CONVROT_GROUP) -> torch.Tensor:
    """weight @ H^T per contiguous group of input features (quant.py:41-45)."""
    n, k = weight.shape
    h = hadamard(group, weight.device)
    return (weight.float().reshape(n, k // group, group) @ h.T).reshape(n, k)


def comfy_meta(fmt: str, **extra) -> torch.Tensor:
    """The comfy_quant metadata tensor: JSON bytes as uint8 (quant.py:52-54)."""
    return torch.tensor(list(json.dumps({"format": fmt, **extra}).encode()), dtype=torch.uint8)


def quantize_int8_convrot(weight: torch.Tensor) -> dict:
    rot = rotate(weight)
    scale = (rot.abs().amax(dim=1, keepdim=True) / 127.0).clamp(min=1e-30)
    q = (rot / scale).round().clamp(-128, 127).to(torch.int8)
    return {
        "weight": q.contiguous(),
        "weight_scale": scale.float().contiguous(),
        "comfy_quant": comfy_meta("int8_tensorwise", convrot=True, convrot_groupsize=CONVROT_GROUP),
    }


def quantize_int8_rows(weight: torch.Tensor) -> dict:
    """Per-row int8 without rotation, the layout of embedding tables (rows are gathered, never
    multiplied; quant.py:70-78): scale = amax_row / 127, q = clamp(rne(w / scale), -128, 127)."""
    w = weight.float()
    scale = (w.abs().amax(dim=1, keepdim=True) / 127.0).clamp(min=1e-30)
    return {
        "weight": (w / scale).round().clamp(-128, 127).to(torch.int8).contiguous(),
        "weight_scale": scale.contiguous(),
        "comfy_quant": comfy_meta("int8_tensorwise"),
    }


def _nearest_level(x: torch.Tensor, levels: torch.Tensor) -> torch.Tensor:
    """Index of the nearest sorted level; ties go to the lower one (quant.py:88-95)."""
    last = levels.numel() - 1
    pos = torch.searchsorted(levels, x.contiguous())
    lo = (pos - 1).clamp(0, last)
    hi = pos.clamp(0, last)
    return torch.where((x - levels[hi]).abs() < (x - levels[lo]).abs(), hi, lo)


def _lloyd_codebook(normalized: torch.Tensor, levels=16, iterations=25, sample_size=300000) -> torch.Tensor:
    """Lloyd-Max fit on a fixed-seed subsample, quantile-initialised (quant.py:98-113)."""
    s = normalized.flatten()
    if s.numel() > sample_size:
        g = torch.Generator(device=s.device).manual_seed(0)
        s = s[torch.randint(0, s.numel(), (sample_size,), device=s.device, generator=g)]
    s = s.float()
    cb = torch.quantile(s, torch.linspace(0, 1, levels, device=s.device))
    for _ in range(iterations):
        nearest = (s.unsqueeze(-1) - cb).abs().argmin(-1)
        nxt = cb.clone()
        for i in range(levels):
            sel = nearest == i
            if sel.any():
                nxt[i] = s[sel].mean()
        cb = nxt
    return cb.contiguous()


def _choose_codebook(normalized: torch.Tensor) -> torch.Tensor:
    """FIXED_LUT when the excess kurtosis is <= -0.1, else a Lloyd fit (quant.py:116-124)."""
    x = normalized.flatten().float()
    if x.numel() > (1 << 19):
        g = torch.Generator(device=x.device).manual_seed(0)
        x = x[torch.randint(0, x.numel(), (1 << 19,), device=x.device, generator=g)]
    kurt = ((x - x.mean()) / (x.std() + 1e-9)).pow(4).mean() - 3.0
    if kurt.item() <= _GATE_KURTOSIS:
        return torch.tensor(FIXED_LUT, device=normalized.device, dtype=torch.float32)
    return _lloyd_codebook(normalized)


def quantize_w4a8(weight: torch.Tensor) -> dict:
    """asym_w4a8_int8 + convrot (quant.py:132-169): per-group scale refined by two alternating
    least-squares passes, fp8 group scales relative to a per-row scale, and a final code
    assignment against the int8-grid levels the kernels decode."""
    n, k = weight.shape
    groups = k // W4_GROUP
    gw = rotate(weight).view(n, groups, W4_GROUP)
    gscale = gw.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    codebook = _choose_codebook(gw / gscale)
    q = _nearest_level(gw / gscale, codebook)
    for _ in range(_ALS_ITERS):
        lv = codebook[q]
        gscale = ((gw * lv).sum(-1, keepdim=True) / (lv * lv).sum(-1, keepdim=True).clamp(min=1e-8)).clamp(min=1e-8)
        q = _nearest_level(gw / gscale, codebook)
    shifted = codebook[q] * gscale
    s_channel = (shifted.abs().amax(dim=(1, 2)) / 127.0).clamp(min=1e-8)
    s_rel = (gscale.squeeze(-1) / s_channel.unsqueeze(1)).float().to(torch.float8_e4m3fn)
    levels = (codebook.view(1, 1, -1) * s_rel.float().unsqueeze(-1)).round().clamp(-127, 127)
    target = (gw / s_channel.view(-1, 1, 1)).reshape(n * groups, W4_GROUP).contiguous()
    lvf = levels.reshape(n * groups, 16).contiguous()
    pos = torch.searchsorted(lvf, target)
    lo = (pos - 1).clamp(0, 15)
    hi = pos.clamp(0, 15)
    dlo = (target - torch.gather(lvf, 1, lo)).abs()
    dhi = (target - torch.gather(lvf, 1, hi)).abs()
    codes = torch.where(dhi < dlo, hi, lo).to(torch.int32).view(n, k)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    return {
        "weight": packed.contiguous(),
        "weight_s_rel": s_rel.contiguous(),
        "weight_s_channel": s_channel.float().contiguous(),
        "weight_codebook": codebook.float().contiguous(),
        "comfy_quant": comfy_meta("asym_w4a8_int8", group_size=W4_GROUP, convrot=True, convrot_groupsize=CONVROT_GROUP),
    }


def meta_of(tensors: dict, base: str) -> dict | None:
    """Parsed comfy_quant JSON of `<base>comfy_quant`, or None for an unquantized tensor."""
    t = tensors.get(base + "comfy_quant")
    if t is None:
        return None
    return json.loads(bytes(t.cpu().to(torch.uint8).tolist()).decode())
