"""AnimaDiT: the 28-block Cosmos-Predict2 MiniTrainDIT denoiser on the B200 kernels
(app/models/dit.js:80-325; math of tools/reference.py:194-249).

Per block (x is the fp32 residual stream [B L, 2048], as in the reference):
  self-attention  LN+adaLN+ConvRot+quant -> qkv GEMM with per-head RMSNorm + RoPE in the epilogue
                  (bf16 q/k/v) -> tcgen05 flash attention -> ConvRot+quant -> o GEMM with the gated
                  residual in the epilogue
  cross-attention LN+adaLN+ConvRot+quant -> q GEMM with per-head RMSNorm -> attention against the
                  per-prompt K/V cache -> ConvRot+quant -> o GEMM + gated residual
  MLP             LN+adaLN+ConvRot+quant -> layer1 GEMM (+GELU epilogue, fp16) -> ConvRot+quant
                  -> layer2 GEMM + gated residual
Activations entering a ConvRot linear are per-token int8 planes (precision "a16": hi + lo/254,
two MMAs, ~16-bit; "a8": one plane, plain W8A8). Attention runs on fp16 q/k/v/P by default (same
tensor-core rate as bf16, 8x finer rounding of the probabilities); attn_dtype=torch.bfloat16 gives
the bf16 path. The modulation vectors for every sigma of a run
are computed in one batched pass (time_cond_batch), the reference's timeCond per pass.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .weights import Linear, concat_linears, linear_weights, vector

D = 2048
HEADS = 16
HD = 128
CTX_DIM = 1024
MLP = 8192


def rope_table(H: int, W: int) -> np.ndarray:
    """cos [H W, 64] followed by sin [H W, 64] of the 3D RoPE for one frame, computed in fp32 as
    the reference does (tools/reference.py:174-187; app/models/common.js:26-52): slots 0..21 are
    the temporal axis at t = 0, 22..42 height, 43..63 width, theta_hw = 1e4 * 4^(42/40)."""
    dim_h = HD // 6 * 2
    dim_t = HD - 2 * dim_h
    f32 = np.float32
    sp = (np.arange(0, dim_h, 2)[: dim_h // 2].astype(f32) / f32(dim_h)).astype(f32)
    h_theta = 10000.0 * 4.0 ** (dim_h / (dim_h - 2))
    hf = (f32(1.0) / np.power(f32(h_theta), sp, dtype=f32)).astype(f32)
    hh, ww = np.meshgrid(np.arange(H, dtype=f32), np.arange(W, dtype=f32), indexing="ij")
    ang = np.concatenate([np.zeros((H * W, dim_t // 2), f32), hh.reshape(-1, 1) * hf, ww.reshape(-1, 1) * hf], 1)
    return np.concatenate([np.cos(ang.astype(f32)), np.sin(ang.astype(f32))], 0).astype(f32)


@dataclass
class TimeCond:
    """Modulation vectors of one sigma: mods [3 * n_blocks + 1, 6144] (self, cross, mlp per block,
    then the final layer's [4096]) (dit.js:196-225)."""

    mods: torch.Tensor
    sigma: float

    def block(self, i):
        return self.mods[3 * i], self.mods[3 * i + 1], self.mods[3 * i + 2]

    @property
    def final(self):
        return self.mods[-1]


@dataclass
class Cond:
    """Per-prompt cross-attention keys/values for all blocks (dit.js:232-249): k (per-head
    RMSNormed) and v, each [B, Lk, 2048] in the attention dtype, plus optional key lengths."""

    k: list
    v: list
    Lk: int
    batch: int
    key_len: torch.Tensor | None = None

    @staticmethod
    def stack(conds: list["Cond"]) -> "Cond":
        """Batch several prompts (e.g. CFG's cond and uncond) into one Cond."""
        Lk = conds[0].Lk
        if not all(c.Lk == Lk for c in conds):
            raise ValueError("stacked contexts need the same length (pad them)")
        kl = None
        if any(c.key_len is not None for c in conds):
            kl = torch.cat([c.key_len if c.key_len is not None else
                            torch.full((c.batch,), Lk, dtype=torch.int32, device=c.k[0].device) for c in conds])
        return Cond([torch.cat([c.k[i] for c in conds]) for i in range(len(conds[0].k))],
                    [torch.cat([c.v[i] for c in conds]) for i in range(len(conds[0].v))], Lk,
                    sum(c.batch for c in conds), kl)


class AnimaDiT:
    """Weights resident on one GPU plus the forward pass (app/models/dit.js:80-129, 253-325)."""

    def __init__(self, tensors: dict, device="cuda", precision: str = "a16", attn_dtype=torch.float16,
                 n_blocks: int | None = None, seq=None):
        """seq: a sharding.SeqGroup to split every image's token rows over its ranks (sequence
        parallelism, the single-image latency mode); every rank holds all weights, calls forward()
        with the same inputs and gets the same velocity."""
        if precision not in ("a16", "a8"):
            raise ValueError("precision must be 'a16' (two int8 planes) or 'a8' (W8A8)")
        self.seq = seq if seq is not None and seq.world > 1 else None
        self.seq_exchange = "peer"
        self._exchanges = []
        self.device = torch.device(device)
        self.planes = 2 if precision == "a16" else 1
        self.precision = precision
        self.attn_dtype = attn_dtype
        if n_blocks is None:
            n_blocks = 1 + max(int(k.split(".")[1]) for k in tensors if k.startswith("blocks."))
        self.n_blocks = n_blocks
        dv = self.device
        lin = lambda base: linear_weights(tensors, base, dv)  # noqa: E731
        self.x_embed = lin("x_embedder.proj.1.")
        self.t1 = lin("t_embedder.1.linear_1.")
        self.t2 = lin("t_embedder.1.linear_2.")
        self.t_norm = vector(tensors, "t_embedding_norm.weight", dv)
        self.blocks = []
        mod_w1, mod_w2 = [], []
        for i in range(n_blocks):
            p = f"blocks.{i}."
            self_q, self_k, self_v = (lin(p + f"self_attn.{n}_proj.") for n in ("q", "k", "v"))
            qkv = concat_linears([self_q, self_k, self_v])
            if qkv is None:
                raise ValueError(f"block {i}: q/k/v cannot be stacked (formats differ)")
            blk = {
                "qkv": qkv, "self_o": lin(p + "self_attn.output_proj."),
                "self_qn": vector(tensors, p + "self_attn.q_norm.weight", dv),
                "self_kn": vector(tensors, p + "self_attn.k_norm.weight", dv),
                "cross_q": lin(p + "cross_attn.q_proj."), "cross_k": lin(p + "cross_attn.k_proj."),
                "cross_v": lin(p + "cross_attn.v_proj."), "cross_o": lin(p + "cross_attn.output_proj."),
                "cross_qn": vector(tensors, p + "cross_attn.q_norm.weight", dv),
                "cross_kn": vector(tensors, p + "cross_attn.k_norm.weight", dv),
                "l1": lin(p + "mlp.layer1."), "l2": lin(p + "mlp.layer2."),
            }
            for m in ("adaln_modulation_self_attn", "adaln_modulation_cross_attn", "adaln_modulation_mlp"):
                mod_w1.append(tensors[p + m + ".1.weight"])
                mod_w2.append(lin(p + m + ".2."))
            self.blocks.append(blk)
        mod_w1.append(tensors["final_layer.adaln_modulation.1.weight"])
        mod_w2.append(lin("final_layer.adaln_modulation.2."))
        self.rank = mod_w1[0].shape[0]
        # every modulation's first projection stacked: one GEMM per run instead of 85 GEMVs per pass
        self.mod_w1 = Linear("bf16", len(mod_w1) * self.rank, D,
                             torch.cat([w.to(torch.bfloat16) for w in mod_w1], 0).to(dv).contiguous(), name="mod_w1")
        self.mod_w2 = mod_w2
        self.final_linear = lin("final_layer.linear.")
        self._rope = {}
        self._bufs = {}

    def set_seq(self, seq, exchange: str = "peer") -> None:
        """Switch sequence parallelism on (a sharding.SeqGroup with world > 1) or off (None) for
        later forwards; the weights are the same either way. exchange: how self-attention's k|v
        reach the other ranks: "peer" (the qkv GEMM stores them into every rank's buffer over
        NVLink, then a device barrier) or "nccl" (a copy and an NCCL all-gather). Collective."""
        self._close_exchanges()
        self.seq = seq if seq is not None and seq.world > 1 else None
        self.seq_exchange = exchange
        self._bufs = {}
        self._rope = {}

    def _close_exchanges(self):
        for x in getattr(self, "_exchanges", []):
            x.close()
        self._exchanges = []

    @classmethod
    def from_file(cls, path: str, device="cuda", prefix: str = "model.diffusion_model.", **kw) -> "AnimaDiT":
        """A DiT from a comfy_quant safetensors checkpoint (SafeTensors.open + AnimaDiT.load,
        app/weights.js:29-41, app/models/dit.js:80-129); tensors stream from the mapped file to
        the device one by one."""
        from .checkpoint import open_dit

        tensors = open_dit(path, prefix)
        try:
            return cls(tensors, device, **kw)
        finally:
            tensors.release()
            tensors.st.close()

    # ------------------------------------------------------------------ time conditioning

    def time_cond_batch(self, sigmas) -> list[TimeCond]:
        """Modulations for every sigma at once (dit.js:196-225 per sigma, tools/reference.py:203-220)."""
        sig = torch.tensor([float(s) for s in sigmas], dtype=torch.float32, device=self.device)
        S = sig.numel()
        temb = ops.timestep_embedding(sig)
        h = ops.matmul(temb, self.t1, act="silu")
        adaln_lora = ops.matmul(h, self.t2)                      # [S, 6144]
        emb = ops.rmsnorm(temb, self.t_norm, D)
        semb = ops.elementwise("silu", emb)
        hh = ops.matmul(semb, self.mod_w1)                      # [S, n_mods * rank]
        n_mods = len(self.mod_w2)
        mods = torch.empty(S, n_mods, 3 * D, dtype=torch.float32, device=self.device)
        mods[:] = adaln_lora[:, None, :]                         # broadcast copy of the shared term
        for i, w2 in enumerate(self.mod_w2):
            hv = hh[:, i * self.rank:(i + 1) * self.rank]
            out = mods[:, i, :]
            ops.matmul(hv, w2, out=out, resid=True)              # mods += W2 (W1 silu(emb))
        return [TimeCond(mods[s], float(sigmas[s])) for s in range(S)]

    def time_cond(self, sigma: float) -> TimeCond:
        return self.time_cond_batch([sigma])[0]

    # ------------------------------------------------------------------ prompt conditioning

    def prepare_context(self, ctx: torch.Tensor, key_len=None) -> Cond:
        """Cross-attention K/V of every block for a context [B, Lk, 1024] or [Lk, 1024]
        (dit.js:232-249): k = RMSNorm_head(ctx_r Wk^T), v = ctx_r Wv^T, in the attention dtype."""
        if ctx.dim() == 2:
            ctx = ctx[None]
        B, Lk, _ = ctx.shape
        c2 = ctx.reshape(B * Lk, CTX_DIM).to(self.device, torch.float32).contiguous()
        cq = ops.rotate_quant(c2, self.planes)
        ks, vs = [], []
        for blk in self.blocks:
            k = torch.empty(B * Lk, D, dtype=self.attn_dtype, device=self.device)
            v = torch.empty(B * Lk, D, dtype=self.attn_dtype, device=self.device)
            ops.linear(cq, blk["cross_k"], out=k, mode="head_norm", qk=(blk["cross_kn"],))
            ops.linear(cq, blk["cross_v"], out=v)
            ks.append(k.view(B, Lk, D))
            vs.append(v.view(B, Lk, D))
        kl = None
        if key_len is not None:
            kl = torch.as_tensor(key_len, dtype=torch.int32).reshape(-1).to(self.device)
            if kl.numel() == 1 and B > 1:
                kl = kl.expand(B).contiguous()
        return Cond(ks, vs, Lk, B, kl)

    # ------------------------------------------------------------------ forward

    def rope(self, Hp: int, Wp: int, rows: tuple[int, int] | None = None) -> torch.Tensor:
        """cos then sin of the RoPE table for an Hp x Wp patch grid; rows = (lo, hi) keeps only
        those token rows (a sequence-parallel rank's slice), as [hi - lo, 64] cos then sin."""
        key = (Hp, Wp, rows)
        if key not in self._rope:
            t = rope_table(Hp, Wp)
            if rows is not None:
                L = Hp * Wp
                t = np.concatenate([t[rows[0]:rows[1]], t[L + rows[0]:L + rows[1]]], 0)
            self._rope[key] = torch.from_numpy(np.ascontiguousarray(t)).to(self.device)
        return self._rope[key]

    def _buffers(self, M: int, B: int = 1):
        """Activations of one forward over M = B x (local) L rows, reused across calls."""
        b = self._bufs.get((M, B))
        if b is None:
            dv = self.device
            b = {
                "qa": ops.QuantRows.empty(M, D, self.planes, dv),
                "qh": ops.QuantRows.empty(M, MLP, self.planes, dv),
                "qkv": torch.empty(M, 3 * D, dtype=self.attn_dtype, device=dv),
                "o": torch.empty(M, D, dtype=self.attn_dtype, device=dv),
                "q": torch.empty(M, D, dtype=self.attn_dtype, device=dv),
                "h": torch.empty(M, MLP, dtype=torch.float16, device=dv),
            }
            if self.seq:
                Lr = M // B
                if self.seq_exchange == "peer":
                    # every rank's k|v rows land in this rank's IPC-shared buffer [B, world * Lr, 4096];
                    # kept until set_seq (graphs captured on it may still be replayed)
                    from .sharding import KVExchange
                    x = KVExchange(self.seq, B, Lr, self.attn_dtype, dv)
                    self._exchanges.append(x)
                    b["kvx"], b["kv_all"] = x, x.kv
                else:
                    # this rank's k|v rows, then every rank's, per image: [B, world * Lr, 4096]
                    b["kv_mine"] = torch.empty(B, Lr, 2 * D, dtype=self.attn_dtype, device=dv)
                    b["kv_all"] = torch.empty(B, self.seq.world * Lr, 2 * D, dtype=self.attn_dtype, device=dv)
            self._bufs = {(M, B): b}
        return b

    def block(self, i: int, x: torch.Tensor, cond: Cond, tc: TimeCond, B: int, L: int, cs: torch.Tensor,
              bufs: dict):
        """One transformer block, in place on x [B L, 2048] (dit.js:261-314)."""
        """One transformer block, in place on x [B L, 2048] (dit.js:261-314). With sequence
        parallelism x, L and cs are this rank's rows; self-attention gathers k|v of all rows."""
        blk = self.blocks[i]
        m_self, m_cross, m_mlp = tc.block(i)
        qa, qh = bufs["qa"], bufs["qh"]
        # self-attention
        ops.layernorm_mod_quant(x, m_self, 0, D, D, out=qa)
        kvx = bufs.get("kvx")
        qkv = ops.linear(qa, blk["qkv"], out=bufs["qkv"], mode="qkv", qk=(blk["self_qn"], blk["self_kn"]),
                         rope_cs=cs, n_q=D, name="dit.self.qkv", peer=kvx.peer_args() if kvx else None)
        if self.seq:
            if kvx:
                kvx.barrier()        # every rank's k|v tiles have landed in bufs["kv_all"]
                kv = bufs["kv_all"]
            else:
                kv = self._gather_kv(qkv, B, L, bufs)
            Lk = kv.shape[1]
            a = ops.attention(qkv, kv, kv, Lq=L, Lk=Lk, H=HEADS, D=HD, ldq=3 * D, ldk=2 * D, ldv=2 * D, q_off=0,
                              k_off=0, v_off=D, batch=B, q_bstride=L * 3 * D, k_bstride=Lk * 2 * D,
                              v_bstride=Lk * 2 * D, out=bufs["o"], name="attn.self")
        else:
            a = ops.attention(qkv, qkv, qkv, Lq=L, Lk=L, H=HEADS, D=HD, ldq=3 * D, ldk=3 * D, ldv=3 * D, q_off=0,
                              k_off=D, v_off=2 * D, batch=B, q_bstride=L * 3 * D, k_bstride=L * 3 * D,
                              v_bstride=L * 3 * D, out=bufs["o"], name="attn.self")
        ops.rotate_quant(a, out=qa)
        ops.linear(qa, blk["self_o"], out=x, resid=True, gate=m_self, g_off=2 * D, name="dit.self.out")
        # cross-attention against the per-prompt keys/values
        ops.layernorm_mod_quant(x, m_cross, 0, D, D, out=qa)
        q = ops.linear(qa, blk["cross_q"], out=bufs["q"], mode="head_norm", qk=(blk["cross_qn"],), name="dit.cross.q")
        kb = cond.Lk * D if cond.batch == B else 0
        a = ops.attention(q, cond.k[i], cond.v[i], Lq=L, Lk=cond.Lk, H=HEADS, D=HD, batch=B, q_bstride=L * D,
                          k_bstride=kb, v_bstride=kb, key_len=cond.key_len, out=bufs["o"], name="attn.cross")
        ops.rotate_quant(a, out=qa)
        ops.linear(qa, blk["cross_o"], out=x, resid=True, gate=m_cross, g_off=2 * D, name="dit.cross.out")
        # MLP
        ops.layernorm_mod_quant(x, m_mlp, 0, D, D, out=qa)
        # GELU on layer1's fp32 accumulators in the GEMM epilogue (it has issue slots to spare), then
        # the fp16 hidden layer's ConvRot+quant
        h = ops.linear(qa, blk["l1"], out=bufs["h"], act="gelu", name="dit.mlp1")
        ops.rotate_quant(h, out=qh)
        ops.linear(qh, blk["l2"], out=x, resid=True, gate=m_mlp, g_off=2 * D, name="dit.mlp2")

    def _gather_kv(self, qkv: torch.Tensor, B: int, L: int, bufs: dict) -> torch.Tensor:
        """k|v of this rank's rows (columns 2048.. of the qkv output) gathered from every rank, per
        image, in global row order: [B, world * L, 4096]."""
        mine, allkv = bufs["kv_mine"], bufs["kv_all"]
        mine.copy_(qkv.view(B, L, 3 * D)[:, :, D:])
        for b in range(B):
            self.seq.all_gather(allkv[b], mine[b])
        return allkv

    def forward(self, latent: torch.Tensor, cond: Cond, tc: TimeCond, on_block=None) -> torch.Tensor:
        """Velocity [B, 16, h, w] for latents [B, 16, h, w] on the device (dit.js:253-325)."""
        if latent.dim() == 3:
            latent = latent[None]
        B, C, h, w = latent.shape
        Hp, Wp = h // 2, w // 2
        L = Hp * Wp
        patches = ops.patchify(latent.contiguous())                      # [B L, 68]
        rows = None
        if self.seq:
            rows = self.seq.span(L)
            L = rows[1] - rows[0]                                          # this rank's rows of each image
            patches = patches.view(B, Hp * Wp, 68)[:, rows[0]:rows[1]].reshape(B * L, 68)
        x = ops.matmul(patches, self.x_embed)                              # [B L, 2048] fp32 residual stream
        cs = self.rope(Hp, Wp, rows)
        bufs = self._buffers(B * L, B)
        for i in range(self.n_blocks):
            self.block(i, x, cond, tc, B, L, cs, bufs)
            if on_block is not None:
                on_block(i, x)
        n = ops.layernorm_mod(x, tc.final, 0, D, D)
        o = ops.matmul(n, self.final_linear)                              # [B L, 64] "(p1 p2 c)"
        if self.seq:
            parts = torch.empty(self.seq.world, B * L, 64, dtype=o.dtype, device=o.device)
            self.seq.all_gather(parts, o)
            o = parts.view(self.seq.world, B, L, 64).transpose(0, 1).reshape(B * Hp * Wp, 64)
        return ops.unpatchify(o, B, h, w)
