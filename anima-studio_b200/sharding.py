"""Work partitioning over the GPUs of one node.

Data parallelism (the throughput mode): images, seeds and CFG branches are independent, so each
rank denoises its own share with no collective on the data path (`seed_shard`); timings are
reduced with the maximum over ranks (`max_over_ranks`).

Sequence parallelism (`SeqGroup`, the single-image latency mode): the image's L token rows are
split into P equal contiguous slices, one per rank of one node, and every rank holds the full
weights. Patch embedding, LayerNorm + adaLN, every linear, the cross-attention (the text K/V are
the same on all ranks), the MLP, the gated residuals and the final layer are row-local: rank r
runs them on its rows [r L/P, (r+1) L/P) with no communication. Self-attention is the one
exchange: each rank's queries attend to the keys and values of all L rows, so after the qkv GEMM
every rank's k|v rows are gathered into a full [L, 4096] k|v buffer (16 MiB fp16 at 1024^2, one
all-gather per block); keys enter the softmax in global row order, so the result is the
one-GPU attention's. At the end the final layer's [L/P, 64] rows are gathered (1 MiB) and every
rank unpatchifies the same velocity and takes the same Euler step. The RoPE table a rank uses is
its slice of rows of the full table.

This replaces head sharding, which needed three all-reduces of the fp32 residual stream (32 MiB
each) per block and ran LayerNorm and quantization replicated on every rank.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch



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
class SeqGroup:
    """The ranks sharing one image's token rows: rank, world size and their torch.distributed
    group (None = the default group)."""

    rank: int
    world: int
    group: object = None

    def span(self, n: int) -> tuple[int, int]:
        """[lo, hi) of this rank's share of n rows (n must split evenly)."""
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} of world {self.world}")
        if n % self.world:
            raise ValueError(f"{n} token rows do not split into {self.world} equal slices")
        step = n // self.world
        return self.rank * step, (self.rank + 1) * step

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> torch.Tensor:
        """out [world * rows, ...] <- every rank's inp [rows, ...] in rank order."""
        import torch.distributed as dist

        dist.all_gather_into_tensor(out, inp, group=self.group)
        return out
