"""Work partitioning over the GPUs of one node.

Data parallelism (the throughput mode): images, seeds and CFG branches are independent, so each
rank denoises its own share with no collective on the data path (`seed_shard`); timings are
reduced with the maximum over ranks (`max_over_ranks`).

Head-sharded tensor parallelism (`TPGroup`, `shard_block`) for single-image latency:

The heads (and the MLP's 8192 hidden features) are split over P ranks of one node, one process
per GPU. Column-parallel linears keep the rows of their output features that belong to the
rank: qkv (the rank's q, k and v heads), cross q/k/v and MLP layer 1. Row-parallel linears keep
the matching input columns: self-attention and cross-attention out-projections and MLP layer 2.
Their partial outputs are summed with one NCCL all-reduce of the fp32 residual stream [B L, 2048]
after each of them, three per block. LayerNorm, the time conditioning, patch embedding and the
final layer run replicated on the full residual stream.

ConvRot keeps this exact: the rotation acts on groups of 256 input features, and every shard
boundary (2048 / P, 8192 / P for P in 2, 4, 8) falls on a group boundary, so a rank rotates and
quantizes its own slice. Each rank quantizes its slice with its own per-token scale, which is a
finer granularity than the unsharded run (results agree to the quantization noise, ~1e-4).
The weight codes and per-row scales are the unsharded ones: a row-parallel shard keeps the
full-row scale of each output row, and only rank 0 keeps the bias.

The gated residual is applied inside the GEMM epilogue: rank 0 adds gate * (y_0 + bias) to x,
the other ranks add gate * y_r to a zeroed x, and the all-reduce (sum) leaves
x + gate * (sum_r y_r + bias) on every rank.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .weights import Linear


def seed_shard(n_items: int, rank: int, world: int) -> range:
    """The contiguous block of item indices (images / seeds) rank `rank` of `world` owns; the
    blocks differ in size by at most one and cover 0..n_items-1 exactly once."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(n_items, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def max_over_ranks(value: float, device="cpu", group=None) -> float:
    """The maximum of a per-rank number over all ranks (1 process: the number itself)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


@dataclass
class TPGroup:
    """The ranks sharing one image: rank, world size and their torch.distributed group."""

    rank: int
    world: int
    group: object = None

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def span(self, n: int, unit: int = 1) -> tuple[int, int]:
        """[lo, hi) of this rank's share of n features, in whole units (heads, 256-groups)."""
        if n % (self.world * unit):
            raise ValueError(f"{n} features do not split into {self.world} shards of whole {unit}-blocks")
        step = n // self.world
        return self.rank * step, (self.rank + 1) * step


def shard_rows(W: Linear, lo: int, hi: int) -> Linear:
    """Output features [lo, hi) of W (a column-parallel shard)."""
    if not 0 <= lo < hi <= W.N:
        raise ValueError(f"{W.name}: rows [{lo}, {hi}) outside N = {W.N}")
    out = Linear(W.kind, hi - lo, W.K, W.data[lo:hi].contiguous(),
                 W.scale[lo:hi].contiguous() if W.scale is not None else None,
                 W.bias[lo:hi].contiguous() if W.bias is not None else None,
                 name=W.name)
    if W.kind == "w4":
        out.s_rel = W.s_rel[lo:hi].contiguous()
        out.codebook = W.codebook
    return out


def shard_cols(W: Linear, lo: int, hi: int, keep_bias: bool) -> Linear:
    """Input features [lo, hi) of W (a row-parallel shard). The shard must start and end on
    256-feature ConvRot groups; per-row scales stay those of the full rows."""
    if not (0 <= lo < hi <= W.K and lo % 256 == 0 and hi % 256 == 0):
        raise ValueError(f"{W.name}: columns [{lo}, {hi}) must be whole 256-groups inside K = {W.K}")
    data = W.data[:, lo // 2:hi // 2] if W.kind == "w4" else W.data[:, lo:hi]  # w4: two codes a byte
    out = Linear(W.kind, W.N, hi - lo, data.contiguous(), W.scale, W.bias if keep_bias else None, name=W.name)
    if W.kind == "w4":
        out.s_rel = W.s_rel[:, lo // 16:hi // 16].contiguous()
        out.codebook = W.codebook
    return out


def shard_stacked(W: Linear, tp: TPGroup, unit: int) -> Linear:
    """A stacked linear (e.g. q|k|v) with every part cut to this rank's share, re-stacked."""
    if not W.parts:
        raise ValueError(f"{W.name}: not a stacked linear")
    pieces, parts, off = [], [], 0
    for name, p_off, n in W.parts:
        lo, hi = tp.span(n, unit)
        piece = shard_rows(W, p_off + lo, p_off + hi)
        pieces.append(piece)
        parts.append((name, off, hi - lo))
        off += hi - lo
    out = Linear(W.kind, off, W.K, torch.cat([p.data for p in pieces], 0).contiguous(),
                 torch.cat([p.scale for p in pieces]).contiguous() if W.scale is not None else None,
                 None, name=W.name, parts=parts)
    if W.kind == "w4":
        out.s_rel = torch.cat([p.s_rel for p in pieces], 0).contiguous()
        out.codebook = W.codebook
    return out


def shard_block(blk: dict, tp: TPGroup, head_dim: int) -> dict:
    """One DiT block's linears cut to this rank (heads for attention, 256-groups for the MLP)."""
    out = dict(blk)
    out["qkv"] = shard_stacked(blk["qkv"], tp, head_dim)
    d_lo, d_hi = tp.span(blk["cross_q"].N, head_dim)
    out["cross_q"] = shard_rows(blk["cross_q"], d_lo, d_hi)
    out["cross_k"] = shard_rows(blk["cross_k"], d_lo, d_hi)
    out["cross_v"] = shard_rows(blk["cross_v"], d_lo, d_hi)
    o_lo, o_hi = tp.span(blk["self_o"].K, head_dim)
    out["self_o"] = shard_cols(blk["self_o"], o_lo, o_hi, keep_bias=tp.rank == 0)
    out["cross_o"] = shard_cols(blk["cross_o"], o_lo, o_hi, keep_bias=tp.rank == 0)
    f_lo, f_hi = tp.span(blk["l1"].N, 256)
    out["l1"] = shard_rows(blk["l1"], f_lo, f_hi)
    out["l2"] = shard_cols(blk["l2"], f_lo, f_hi, keep_bias=tp.rank == 0)
    return out
