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


class _DeviceArray:
    """__cuda_array_interface__ over a raw device allocation, for a torch view of it."""

    def __init__(self, addr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (addr, False),
                                         "version": 3, "strides": None}


class KVExchange:
    """The k|v exchange of sequence parallelism over peer memory, for images of `rows` local token
    rows: every rank owns a gathered k|v buffer [B, world * rows, 4096] and a flag array, shared
    with the other ranks by CUDA IPC. The qkv GEMM of each rank stores its k|v tiles into every
    rank's buffer through its mappings (ops.linear(..., peer=self.peer_args())), then barrier()
    (anima_peer_barrier) orders those writes before any rank's attention reads `self.kv`.
    Construction and close() are collective: every rank of the group calls them in the same order."""

    def __init__(self, seq: SeqGroup, B: int, rows: int, dtype: torch.dtype, device):
        import ctypes as C

        import torch.distributed as dist

        from . import device as dev

        self.seq, self.B, self.rows = seq, B, rows
        index = torch.device(device).index
        self.ctx = dev.Context.get(torch.cuda.current_device() if index is None else index)
        esz = torch.tensor([], dtype=dtype).element_size()
        nbytes = B * seq.world * rows * 4096 * esz
        mine, handles = [], []
        for size in (nbytes, 64):  # the k|v buffer, then the barrier flags (world <= 8 words)
            addr, h = C.c_void_p(), C.create_string_buffer(64)
            self.ctx.call("anima_ipc_alloc", size, C.byref(addr), h)
            mine.append(addr.value)
            handles.append(h.raw)
        everyone = [None] * seq.world
        dist.all_gather_object(everyone, handles, group=seq.group)
        self.kv_addr, self.flag_addr, self.opened = [], [], []
        for r, (hk, hf) in enumerate(everyone):
            if r == seq.rank:
                self.kv_addr.append(mine[0])
                self.flag_addr.append(mine[1])
                continue
            for h, dst in ((hk, self.kv_addr), (hf, self.flag_addr)):
                addr = C.c_void_p()
                self.ctx.call("anima_ipc_open", h, C.byref(addr))
                dst.append(addr.value)
                self.opened.append(addr.value)
        self.own = mine
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        typestr = "<f2" if dtype == torch.float16 else "<i2"
        kv = torch.as_tensor(_DeviceArray(mine[0], (B, seq.world * rows, 4096), typestr), device=device)
        self.kv = kv if dtype == torch.float16 else kv.view(dtype)
        g = dev.PeerGroup()
        g.rank, g.world, g.timeout_us = seq.rank, seq.world, 0
        for r in range(seq.world):
            g.flags[r] = self.flag_addr[r]
        g.counter = self.counter.data_ptr()
        self._group = g

    def peer_args(self) -> dict:
        lo, _ = self.seq.span(self.seq.world * self.rows)
        return {"kv": list(self.kv_addr), "row0": lo, "rows": self.rows, "item_rows": self.seq.world * self.rows}

    def barrier(self):
        import ctypes as C

        self.ctx.call("anima_peer_barrier", C.byref(self._group))

    def close(self):
        """Unmap the other ranks' buffers, then free this rank's (collective)."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.seq.group)
        for a in self.opened:
            self.ctx.call("anima_ipc_close", a)
        dist.barrier(group=self.seq.group)
        for a in self.own:
            self.ctx.call("anima_ipc_free", a)
        self.opened, self.own = [], []
