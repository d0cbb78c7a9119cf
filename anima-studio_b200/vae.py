"""The Wan-2.1 VAE decoder (Qwen-Image): the denoised latent to an image, once per image
(app/models/vae.js:10-113; math of tools/reference.py:254-295), NHWC on the device.

The latent is de-normalised with the model's per-channel mean and std, a 1x1 conv, a 3x3 conv to
384 channels, two residual blocks around a single-head spatial attention (d = 384), then four
stages of residual blocks with a nearest 2x upsample + 3x3 conv between them (8x in all), and a
norm + SiLU + 3x3 conv to RGB clamped to [-1, 1] and mapped to [0, 1]. Residual blocks are
norm + SiLU -> conv -> norm + SiLU -> conv, plus the input (through a 1x1 conv when the channel
count changes); the conv adds its result into the shortcut (conv3x3Into).
"""

from __future__ import annotations

import torch

from . import ops
from .synthetic import LATENT_MEAN, LATENT_STD
from .weights import linear_weights, vector


class VAEDecoder:
    """Decoder weights on one GPU plus decode() (vae.js VAEDecoder.load / decode)."""

    def __init__(self, tensors, device="cuda"):
        dv = torch.device(device)
        self.device = dv
        lin = lambda base: linear_weights(tensors, base, dv)  # noqa: E731
        g = lambda name: vector(tensors, name, dv)  # noqa: E731

        def res(p):
            return {"n1": g(p + ".residual.0.gamma"), "c1": lin(p + ".residual.2."), "n2": g(p + ".residual.3.gamma"),
                    "c2": lin(p + ".residual.6."), "sc": lin(p + ".shortcut.") if p + ".shortcut.weight" in tensors else None}

        self.conv2 = lin("conv2.")
        self.conv1 = lin("decoder.conv1.")
        self.mid0 = res("decoder.middle.0")
        self.attn = {"norm": g("decoder.middle.1.norm.gamma"), "qkv": lin("decoder.middle.1.to_qkv."),
                     "proj": lin("decoder.middle.1.proj.")}
        self.mid2 = res("decoder.middle.2")
        self.ups = []
        for i in range(15):
            p = f"decoder.upsamples.{i}"
            if p + ".resample.1.weight" in tensors:
                self.ups.append({"up": lin(p + ".resample.1.")})
            else:
                self.ups.append({"res": res(p)})
        self.head_norm = g("decoder.head.0.gamma")
        self.head = lin("decoder.head.2.")
        self.mean = torch.tensor(LATENT_MEAN, dtype=torch.float32, device=dv)
        self.std = torch.tensor(LATENT_STD, dtype=torch.float32, device=dv)

    def _res(self, x, r, h, w):
        cin = x.shape[1]
        t = ops.channel_norm(x, r["n1"], cin, True)
        a = ops.conv3x3(t, r["c1"], h, w)
        t = ops.channel_norm(a, r["n2"], r["c1"].N, True)
        out = ops.matmul(x, r["sc"]) if r["sc"] is not None else x
        return ops.conv3x3(t, r["c2"], h, w, into=out)

    def decode(self, latent: torch.Tensor) -> torch.Tensor:
        """latent [16, h, w] in the model's normalised space -> image [3, 8h, 8w] in [0, 1]."""
        C, h, w = latent.shape
        z = latent.to(self.device, torch.float32) * self.std[:, None, None] + self.mean[:, None, None]
        x = ops.matmul(z.reshape(C, h * w).t().contiguous(), self.conv2)          # NHWC [h w, 16]
        x = ops.conv3x3(x, self.conv1, h, w)
        x = self._res(x, self.mid0, h, w)
        c = x.shape[1]                                                          # single-head attention, d = c
        n = ops.channel_norm(x, self.attn["norm"], c, False)
        qkv = ops.matmul(n, self.attn["qkv"])
        a = ops.attention(qkv, qkv, qkv, Lq=h * w, Lk=h * w, H=1, D=c, ldq=3 * c, ldk=3 * c, ldv=3 * c, q_off=0,
                          k_off=c, v_off=2 * c, out_dtype=torch.float32)
        ops.matmul(a, self.attn["proj"], out=x, resid=True)
        x = self._res(x, self.mid2, h, w)
        H, W = h, w
        for u in self.ups:
            if "up" in u:
                x = ops.conv3x3(x, u["up"], H, W, up=True)
                H, W = 2 * H, 2 * W
            else:
                x = self._res(x, u["res"], H, W)
        t = ops.channel_norm(x, self.head_norm, x.shape[1], True)
        rgb = ops.conv3x3(t, self.head, H, W)                                   # [H W, 3]
        return ((rgb.clamp(-1, 1) + 1) / 2).clamp(0, 1).t().reshape(3, H, W)
