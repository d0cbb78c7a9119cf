"""Multi-GPU partitioning logic on the CPU: data-parallel seed shards and timing reduction, and the
head-sharded tensor-parallel weight split, exercised with world-size-2 `gloo` process groups.

The tensor-parallel checks run the oracle's fp32 math (dequantized ConvRot weights) on each rank's
shard and sum the partial products with the same all-reduce the GPU path uses; the result must
equal the unsharded product. The CUDA kernels themselves are covered by the GPU tests."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from conftest import pkg


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world=2):
    port = _free_port()
    mp.spawn(fn, args=(world, port), nprocs=world, join=True)


def _init(rank, world, port):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    return dist


def _convrot_linear(seed, N, K, parts=None):
    """An int8 ConvRot Linear (CPU tensors) and its dequantized fp32 weight."""
    quant, W = pkg("quant"), pkg("weights")
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    t = quant.quantize_int8_convrot(w)
    lin = W.Linear("i8", N, K, t["weight"].contiguous(), t["weight_scale"].reshape(-1).float().contiguous(),
                   torch.randn(N, generator=g) * 0.1, name="lin")
    if parts:
        lin.parts = parts
        lin.bias = None
    deq = oracle.dequantize_int8_convrot(t["weight"].numpy(), t["weight_scale"].numpy())
    return lin, deq


def test_seed_shards_cover_every_item_once():
    sh = pkg("sharding")
    for n in (1, 7, 64):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in sh.seed_shard(n, r, world)]
            assert got == list(range(n))
            sizes = [len(sh.seed_shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_shards_reassemble():
    sh = pkg("sharding")
    lin, _ = _convrot_linear(1, 512, 1024)
    for world in (2, 4):
        rows = [sh.shard_rows(lin, r * 512 // world, (r + 1) * 512 // world) for r in range(world)]
        assert torch.equal(torch.cat([s.data for s in rows]), lin.data)
        assert torch.equal(torch.cat([s.scale for s in rows]), lin.scale)
        cols = [sh.shard_cols(lin, r * 1024 // world, (r + 1) * 1024 // world, keep_bias=r == 0) for r in range(world)]
        assert torch.equal(torch.cat([s.data for s in cols], 1), lin.data)
        assert all(torch.equal(s.scale, lin.scale) for s in cols)
        assert cols[0].bias is not None and all(s.bias is None for s in cols[1:])
    with pytest.raises(ValueError):
        sh.shard_cols(lin, 0, 100, keep_bias=True)  # not a whole ConvRot group
    with pytest.raises(ValueError):
        sh.TPGroup(0, 3).span(2048, 128)            # 16 heads do not split three ways


def _dp_worker(rank, world, port):
    dist = _init(rank, world, port)
    sh = pkg("sharding")
    assert sh.max_over_ranks(1.5 + rank) == 1.5 + world - 1
    mine = list(sh.seed_shard(64, rank, world))
    t = torch.zeros(64)
    t[mine] = 1
    dist.all_reduce(t)
    assert torch.equal(t, torch.ones(64))
    dist.destroy_process_group()


def test_data_parallel_helpers_gloo():
    _spawn(_dp_worker)


def _tp_worker(rank, world, port):
    dist = _init(rank, world, port)
    sh = pkg("sharding")
    tp = sh.TPGroup(rank, world, None)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((33, 2048)).astype(np.float32)

    # row-parallel (out-projection): input features split, partial products summed, bias once
    lin, deq = _convrot_linear(3, 256, 2048)
    lo, hi = tp.span(2048, 128)
    shard = sh.shard_cols(lin, lo, hi, keep_bias=rank == 0)
    part_deq = oracle.dequantize_int8_convrot(shard.data.numpy(), shard.scale.numpy())
    y = x[:, lo:hi] @ part_deq.T
    if shard.bias is not None:
        y = y + shard.bias.numpy()
    yt = tp.all_reduce(torch.from_numpy(np.ascontiguousarray(y)))
    ref = x @ deq.T + lin.bias.numpy()
    assert np.abs(yt.numpy() - ref).max() <= 1e-4 * np.abs(ref).max()

    # column-parallel stacked q|k|v: each part cut to this rank's heads
    qkv, deq3 = _convrot_linear(5, 3 * 512, 2048, parts=[("q", 0, 512), ("k", 512, 512), ("v", 1024, 512)])
    s3 = sh.shard_stacked(qkv, tp, 128)
    assert s3.N == 3 * 512 // world and [p[2] for p in s3.parts] == [512 // world] * 3
    got = x @ oracle.dequantize_int8_convrot(s3.data.numpy(), s3.scale.numpy()).T
    full = x @ deq3.T
    h0, h1 = tp.span(512, 128)
    want = np.concatenate([full[:, o + h0:o + h1] for o in (0, 512, 1024)], 1)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_split_gloo(world):
    _spawn(_tp_worker, world)
