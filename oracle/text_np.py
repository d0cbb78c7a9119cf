"""numpy restatement of the reference's text conditioning — TEST INFRASTRUCTURE ONLY.

Qwen3-0.6B text encoder and LLM adapter of tools/reference.py:116-169 (with rope_cos_sin,
tools/reference.py:98-102, and causal attention, :109-111), on weights given as W(name) -> fp32
array (DequantWeights). Pinned by tests/golden/text_1024.npz, which the reference's own code wrote.
"""

from __future__ import annotations

import numpy as np

from .ref_np import gelu, layer_norm, rms_norm, rotate_half, silu  # noqa: F401

f32 = np.float32


def rope_cos_sin(L: int, head_dim: int, theta: float):
    """(cos, sin) [L, head_dim], the second half repeating the first (tools/reference.py:98-102)."""
    inv = (f32(1.0) / np.power(f32(theta), np.arange(0, head_dim, 2, dtype=f32) / f32(head_dim), dtype=f32)).astype(f32)
    f = (np.arange(L, dtype=f32)[:, None] * inv[None]).astype(f32)
    emb = np.concatenate([f, f], -1)
    return np.cos(emb).astype(f32), np.sin(emb).astype(f32)


def attention(q, k, v, causal=False):
    """softmax(q k^T / sqrt(D)) v per head, fp32 with max subtraction; q [H, Lq, D], k/v [H, Lk, D]."""
    H, Lq, D = q.shape
    out = np.empty((H, Lq, v.shape[-1]), dtype=f32)
    scale = f32(1.0 / np.sqrt(D))
    for h in range(H):
        s = (q[h].astype(f32) @ k[h].astype(f32).T) * scale
        if causal:
            s = np.where(np.tril(np.ones((Lq, k.shape[1]), dtype=bool)), s, -np.inf)
        s -= s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True, dtype=f32)
        out[h] = p @ v[h].astype(f32)
    return out


def qwen3(W, ids, n_layers=28):
    """Final hidden states [L, 1024] (tools/reference.py:116-136)."""
    x = W("model.embed_tokens.weight")[np.asarray(ids)].astype(f32)
    L = x.shape[0]
    cos, sin = rope_cos_sin(L, 128, 1e6)
    for i in range(n_layers):
        p = f"model.layers.{i}."
        h = rms_norm(x, W(p + "input_layernorm.weight"))
        q = (h @ W(p + "self_attn.q_proj.weight").T).reshape(L, 16, 128).transpose(1, 0, 2)
        k = (h @ W(p + "self_attn.k_proj.weight").T).reshape(L, 8, 128).transpose(1, 0, 2)
        v = (h @ W(p + "self_attn.v_proj.weight").T).reshape(L, 8, 128).transpose(1, 0, 2)
        q = rms_norm(q, W(p + "self_attn.q_norm.weight"))
        k = rms_norm(k, W(p + "self_attn.k_norm.weight"))
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        k = np.repeat(k, 2, axis=0)
        v = np.repeat(v, 2, axis=0)
        a = attention(q, k, v, causal=True).transpose(1, 0, 2).reshape(L, 2048)
        x = (x + a @ W(p + "self_attn.o_proj.weight").T).astype(f32)
        h = rms_norm(x, W(p + "post_attention_layernorm.weight"))
        g = h @ W(p + "mlp.gate_proj.weight").T
        u = h @ W(p + "mlp.up_proj.weight").T
        x = (x + (silu(g) * u) @ W(p + "mlp.down_proj.weight").T).astype(f32)
    return rms_norm(x, W("model.norm.weight")).astype(f32)


def llm_adapter(W, src, t5_ids, t5_weights=None, n_blocks=6):
    """T5-position context [512, 1024] from Qwen3 states src [Ls, 1024] (tools/reference.py:139-169)."""
    p0 = "llm_adapter."
    x = W(p0 + "embed.weight")[np.asarray(t5_ids)].astype(f32)
    Lt, Ls = x.shape[0], src.shape[0]
    cos_t, sin_t = rope_cos_sin(Lt, 64, 1e4)
    cos_s, sin_s = rope_cos_sin(Ls, 64, 1e4)

    def attn(p, xq, ctx, cq, sq, ck, sk):
        Lq, Lk = xq.shape[0], ctx.shape[0]
        q = rms_norm((xq @ W(p + "q_proj.weight").T).reshape(Lq, 16, 64), W(p + "q_norm.weight")).transpose(1, 0, 2)
        k = rms_norm((ctx @ W(p + "k_proj.weight").T).reshape(Lk, 16, 64), W(p + "k_norm.weight")).transpose(1, 0, 2)
        v = (ctx @ W(p + "v_proj.weight").T).reshape(Lk, 16, 64).transpose(1, 0, 2)
        q = q * cq + rotate_half(q) * sq
        k = k * ck + rotate_half(k) * sk
        return attention(q, k, v).transpose(1, 0, 2).reshape(Lq, 1024) @ W(p + "o_proj.weight").T

    for i in range(n_blocks):
        p = f"{p0}blocks.{i}."
        n = rms_norm(x, W(p + "norm_self_attn.weight"))
        x = (x + attn(p + "self_attn.", n, n, cos_t, sin_t, cos_t, sin_t)).astype(f32)
        x = (x + attn(p + "cross_attn.", rms_norm(x, W(p + "norm_cross_attn.weight")), src, cos_t, sin_t, cos_s,
                      sin_s)).astype(f32)
        h = rms_norm(x, W(p + "norm_mlp.weight"))
        h = gelu(h @ W(p + "mlp.0.weight").T + W(p + "mlp.0.bias"))
        x = (x + h @ W(p + "mlp.2.weight").T + W(p + "mlp.2.bias")).astype(f32)
    out = rms_norm(x @ W(p0 + "out_proj.weight").T + W(p0 + "out_proj.bias"), W(p0 + "norm.weight")).astype(f32)
    if t5_weights is not None:
        out = out * np.asarray(t5_weights, dtype=f32)[:, None]
    if out.shape[0] < 512:
        out = np.concatenate([out, np.zeros((512 - out.shape[0], out.shape[1]), f32)])
    return out
