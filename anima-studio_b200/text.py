"""The text conditioning in front of the DiT: the Qwen3-0.6B text encoder and the LLM adapter that
maps its hidden states onto T5-token positions (app/models/qwen3.js:9-79, app/models/dit.js:139-191;
math of tools/reference.py:116-169), on the B200 operators of libanima_b200.

Qwen3 runs its attention and MLP linears on the int8 tensor-core GEMM (ConvRot weights, inputs
rotated and quantized per token in two int8 planes, as the DiT's), per-head RMSNorm and split-half
RoPE (theta 1e6) on q and k, and causal attention with 16 query heads over 8 key/value heads. The
adapter's linears are bf16 (the published DiT file keeps them unquantized) on the CUDA-core GEMM,
with d = 64 attention (RoPE theta 1e4). Both run once per prompt; their outputs feed
AnimaDiT.prepare_context.
"""

from __future__ import annotations

import torch

from . import ops
from .synthetic import ADAPTER, QWEN3
from .weights import linear_weights, vector


def rope_table(L: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """cos [L, head_dim / 2] followed by sin, for positions 0..L-1 (tools/reference.py:98-102, the
    fp32 arithmetic of rope_cos_sin; its second half repeats the first, so half is kept)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    f = torch.arange(L, dtype=torch.float32)[:, None] * inv[None]
    return torch.cat([f.cos(), f.sin()], 0).contiguous().to(device)


class Qwen3:
    """Qwen3-0.6B: token ids -> final hidden states [L, 1024] (after the last RMSNorm)."""

    def __init__(self, tensors, device="cuda", precision: str = "a16", n_layers: int | None = None):
        dv = torch.device(device)
        self.device = dv
        self.planes = 2 if precision == "a16" else 1
        if n_layers is None:
            n_layers = 1 + max(int(k.split(".")[2]) for k in tensors if k.startswith("model.layers."))
        # per-row int8 table (quant.py:70-78): rows are gathered, value = q * weight_scale[row]
        self.embed_q = tensors["model.embed_tokens.weight"].to(dv)
        self.embed_s = tensors["model.embed_tokens.weight_scale"].to(dv, torch.float32).reshape(-1)
        lin = lambda base: linear_weights(tensors, base, dv)  # noqa: E731
        self.layers = []
        for i in range(n_layers):
            p = f"model.layers.{i}."
            self.layers.append({
                "ln1": vector(tensors, p + "input_layernorm.weight", dv),
                "ln2": vector(tensors, p + "post_attention_layernorm.weight", dv),
                "qn": vector(tensors, p + "self_attn.q_norm.weight", dv),
                "kn": vector(tensors, p + "self_attn.k_norm.weight", dv),
                "q": lin(p + "self_attn.q_proj."), "k": lin(p + "self_attn.k_proj."), "v": lin(p + "self_attn.v_proj."),
                "o": lin(p + "self_attn.o_proj."), "gate": lin(p + "mlp.gate_proj."), "up": lin(p + "mlp.up_proj."),
                "down": lin(p + "mlp.down_proj."),
            })
        self.norm = vector(tensors, "model.norm.weight", dv)

    def encode(self, ids) -> torch.Tensor:
        """qwen3.js encode / tools/reference.py qwen3: ids -> [L, 1024] fp32 on the device."""
        D, H, KH, HD = QWEN3["hidden"], QWEN3["heads"], QWEN3["kv_heads"], QWEN3["head_dim"]
        idx = torch.as_tensor(ids, dtype=torch.long).to(self.device)
        L = idx.numel()
        x = (self.embed_q[idx].float() * self.embed_s[idx][:, None]).contiguous()
        cs = rope_table(L, HD, QWEN3["theta"], self.device)
        for ly in self.layers:
            h = ops.rmsnorm(x, ly["ln1"], D)
            hq = ops.rotate_quant(h, self.planes)               # one rotation + quantization for q, k, v
            # q, k, v leave their norms / projections as fp16 for the tcgen05 attention (causal, 16 q
            # heads over 8 k/v heads); its softmax and output stay fp32
            f16 = torch.float16
            q = ops.rmsnorm(ops.linear(hq, ly["q"]), ly["qn"], HD, out_dtype=f16)
            k = ops.rmsnorm(ops.linear(hq, ly["k"]), ly["kn"], HD, out_dtype=f16)
            v = ops.linear(hq, ly["v"], out_dtype=f16)
            ops.rope(q, cs, L, H, HD)
            ops.rope(k, cs, L, KH, HD)
            a = ops.attention(q, k, v, Lq=L, Lk=L, H=H, D=HD, group=H // KH, causal=True, out_dtype=torch.float32)
            ops.linear(a, ly["o"], out=x, resid=True, planes=self.planes)
            h2q = ops.rotate_quant(ops.rmsnorm(x, ly["ln2"], D), self.planes)
            gu = ops.elementwise("silu_mul", ops.linear(h2q, ly["gate"]), ops.linear(h2q, ly["up"]))
            ops.linear(gu, ly["down"], out=x, resid=True, planes=self.planes)
        return ops.rmsnorm(x, self.norm, D)


class LLMAdapter:
    """The LLM adapter: Qwen3 hidden states + T5 token ids -> the DiT's text context [512, 1024]
    (tools/reference.py:139-169, app/models/dit.js:139-191): T5-token embeddings attend to
    themselves and to the Qwen3 states through 6 blocks, then a projection and RMSNorm, optional
    per-token weights, zero padding to 512 rows."""

    def __init__(self, tensors, device="cuda", n_blocks: int | None = None, prefix: str = "llm_adapter."):
        dv = torch.device(device)
        self.device = dv
        p0 = prefix
        if n_blocks is None:
            n_blocks = 1 + max(int(k[len(p0):].split(".")[1]) for k in tensors if k.startswith(p0 + "blocks."))
        self.embed = tensors[p0 + "embed.weight"].to(dv)
        lin = lambda base: linear_weights(tensors, base, dv)  # noqa: E731
        self.blocks = []
        for i in range(n_blocks):
            p = f"{p0}blocks.{i}."
            blk = {n: vector(tensors, p + n + ".weight", dv) for n in ("norm_self_attn", "norm_cross_attn", "norm_mlp")}
            for a in ("self_attn", "cross_attn"):
                blk[a] = {n: lin(f"{p}{a}.{n}.") for n in ("q_proj", "k_proj", "v_proj", "o_proj")}
                blk[a]["qn"] = vector(tensors, f"{p}{a}.q_norm.weight", dv)
                blk[a]["kn"] = vector(tensors, f"{p}{a}.k_norm.weight", dv)
            blk["mlp0"], blk["mlp2"] = lin(p + "mlp.0."), lin(p + "mlp.2.")
            self.blocks.append(blk)
        self.out_proj = lin(p0 + "out_proj.")
        self.norm = vector(tensors, p0 + "norm.weight", dv)

    def _attn(self, w, xq, ctx, cs_q, cs_k, x):
        """x += o_proj(attention(rope(rms(q)), rope(rms(k)), v)) (tools/reference.py:149-157)."""
        D, H, HD = ADAPTER["hidden"], ADAPTER["heads"], ADAPTER["head_dim"]
        Lq, Lk = xq.shape[0], ctx.shape[0]
        q = ops.rmsnorm(ops.matmul(xq, w["q_proj"]), w["qn"], HD)
        k = ops.rmsnorm(ops.matmul(ctx, w["k_proj"]), w["kn"], HD)
        v = ops.matmul(ctx, w["v_proj"])
        ops.rope(q, cs_q, Lq, H, HD)
        ops.rope(k, cs_k, Lk, H, HD)
        a = ops.attention(q, k, v, Lq=Lq, Lk=Lk, H=H, D=HD, out_dtype=torch.float32)
        ops.matmul(a, w["o_proj"], out=x, resid=True)

    def __call__(self, src: torch.Tensor, t5_ids, t5_weights=None, pad_to: int = 512) -> torch.Tensor:
        D, HD = ADAPTER["hidden"], ADAPTER["head_dim"]
        idx = torch.as_tensor(t5_ids, dtype=torch.long).to(self.device)
        x = self.embed[idx].float().contiguous()
        src = src.to(self.device, torch.float32).contiguous()
        Lt, Ls = x.shape[0], src.shape[0]
        cs_t = rope_table(Lt, HD, ADAPTER["theta"], self.device)
        cs_s = rope_table(Ls, HD, ADAPTER["theta"], self.device)
        for blk in self.blocks:
            n = ops.rmsnorm(x, blk["norm_self_attn"], D)
            self._attn(blk["self_attn"], n, n, cs_t, cs_t, x)
            n = ops.rmsnorm(x, blk["norm_cross_attn"], D)
            self._attn(blk["cross_attn"], n, src, cs_t, cs_s, x)
            h = ops.matmul(ops.rmsnorm(x, blk["norm_mlp"], D), blk["mlp0"], act="gelu")
            ops.matmul(h, blk["mlp2"], out=x, resid=True)
        out = ops.rmsnorm(ops.matmul(x, self.out_proj), self.norm, D)
        if t5_weights is not None:
            out = out * torch.as_tensor(t5_weights, dtype=torch.float32, device=self.device)[:, None]
        if out.shape[0] < pad_to:
            out = torch.cat([out, torch.zeros(pad_to - out.shape[0], D, device=self.device)])
        return out
