"""numpy restatement of the reference's VAE decoder — TEST INFRASTRUCTURE ONLY.

vae_decode of tools/reference.py:254-295 (Wan-2.1 decoder on CHW arrays), with the weights given as
W(name) -> fp32 array and W.has(name). Pinned by tests/golden/vae_64.npz, which the reference's
own code wrote.
"""

from __future__ import annotations

import numpy as np

from .text_np import attention
from .ref_np import silu

f32 = np.float32


def conv(W, x, p):
    """3x3 (pad 1; OHWI weights) or 1x1 ([O, I]) convolution of x [C, h, w], plus bias."""
    w = W(p + ".weight")
    b = W(p + ".bias")
    C, h, wd = x.shape
    if w.ndim == 2:
        return (np.einsum("chw,oc->ohw", x, w) + b[:, None, None]).astype(f32)
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1)))
    # im2col in (ky, kx, ci) order, the OHWI weight's K order
    cols = np.stack([xp[:, ky:ky + h, kx:kx + wd] for ky in range(3) for kx in range(3)], 0)  # [9, C, h, w]
    cols = cols.transpose(2, 3, 0, 1).reshape(h * wd, 9 * C)
    y = cols @ w.reshape(w.shape[0], -1).T + b
    return y.T.reshape(-1, h, wd).astype(f32)


def norm(W, x, p):
    """F.normalize over channels * sqrt(C) * gamma (tools/reference.py:264-265)."""
    n = np.sqrt((x.astype(f32) ** 2).sum(0, keepdims=True, dtype=f32))
    return (x / np.maximum(n, f32(1e-12)) * f32(np.sqrt(x.shape[0])) * W(p + ".gamma")[:, None, None]).astype(f32)


def res(W, x, p):
    h = conv(W, silu(norm(W, x, p + ".residual.0")), p + ".residual.2")
    h = conv(W, silu(norm(W, h, p + ".residual.3")), p + ".residual.6")
    sc = conv(W, x, p + ".shortcut") if W.has(p + ".shortcut.weight") else x
    return (h + sc).astype(f32)


def attn_block(W, x, p):
    c, hh, ww = x.shape
    qkv = conv(W, norm(W, x, p + ".norm"), p + ".to_qkv")
    q, k, v = qkv.reshape(3, c, hh * ww).transpose(0, 2, 1)  # [hw, c] each
    a = attention(q[None], k[None], v[None])[0].T.reshape(c, hh, ww)
    return (conv(W, a, p + ".proj") + x).astype(f32)


def vae_decode(W, z):
    """z [16, h, w] de-normalised latent -> image [3, 8h, 8w] in [0, 1]."""
    x = conv(W, z.astype(f32), "conv2")
    x = conv(W, x, "decoder.conv1")
    x = res(W, x, "decoder.middle.0")
    x = attn_block(W, x, "decoder.middle.1")
    x = res(W, x, "decoder.middle.2")
    for i in range(15):
        p = f"decoder.upsamples.{i}"
        if W.has(p + ".resample.1.weight"):
            x = x.repeat(2, 1).repeat(2, 2)
            x = conv(W, x, p + ".resample.1")
        else:
            x = res(W, x, p)
    x = conv(W, silu(norm(W, x, "decoder.head.0")), "decoder.head.2")
    return ((np.clip(x, -1, 1) + 1) / 2).clip(0, 1).astype(f32)
