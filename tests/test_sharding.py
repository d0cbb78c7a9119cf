"""Multi-GPU partitioning logic on the CPU, with world-size-2 `gloo` process groups: data-parallel
seed shards and timing reduction, and the sequence-parallel split of one image's token rows.

The sequence-parallel check runs the oracle's fp32 math (dequantized ConvRot weights) the way the
GPU path splits it: each rank computes every row-local part of a DiT block on its own rows, and
gathers k and v of all rows for self-attention with the same all-gather; its rows must equal the
one-process block. The CUDA kernels themselves are covered by the GPU tests."""

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


def test_seed_shards_cover_every_item_once():
    sh = pkg("sharding")
    for n in (1, 7, 64):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in sh.seed_shard(n, r, world)]
            assert got == list(range(n))
            sizes = [len(sh.seed_shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_seq_spans():
    sh = pkg("sharding")
    for world in (1, 2, 4, 8):
        spans = [sh.SeqGroup(r, world).span(4096) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 4096
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        sh.SeqGroup(0, 3).span(4096)   # 4096 rows do not split three ways
    with pytest.raises(ValueError):
        sh.SeqGroup(2, 2).span(64)


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


def _seq_block(W, i, x, ctx, emb, adaln_lora, cos, sin, seq):
    """oracle.dit_block with the token rows split over the ranks: x, cos, sin are this rank's rows;
    self-attention's k and v are gathered from every rank in rank (= row) order."""
    import torch.distributed as dist

    O = oracle
    p = f"blocks.{i}."
    H, HD = 16, 128

    def gather(t):
        parts = [torch.empty_like(torch.from_numpy(t)) for _ in range(seq.world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(t)))
        return torch.cat(parts).numpy()

    L = x.shape[0]
    sh, sc, g = O.block_mod(W, p + "adaln_modulation_self_attn", emb, adaln_lora)
    n = O.layer_norm(x) * (1 + sc) + sh
    a = p + "self_attn."
    q = O.rms_norm((n @ W(a + "q_proj.weight").T).reshape(L, H, HD), W(a + "q_norm.weight")).transpose(1, 0, 2)
    k = O.rms_norm((n @ W(a + "k_proj.weight").T).reshape(L, H, HD), W(a + "k_norm.weight")).transpose(1, 0, 2)
    v = (n @ W(a + "v_proj.weight").T).reshape(L, H, HD).transpose(1, 0, 2)
    q = q * cos + O.rotate_half(q) * sin
    k = k * cos + O.rotate_half(k) * sin
    k_all = gather(k.transpose(1, 0, 2).astype(np.float32)).transpose(1, 0, 2)
    v_all = gather(v.transpose(1, 0, 2).astype(np.float32)).transpose(1, 0, 2)
    o = O.attention(q, k_all, v_all).transpose(1, 0, 2).reshape(L, H * HD)
    x = x + g * (o @ W(a + "output_proj.weight").T)
    sh, sc, g = O.block_mod(W, p + "adaln_modulation_cross_attn", emb, adaln_lora)
    n = O.layer_norm(x) * (1 + sc) + sh
    from oracle import ref_np

    x = x + g * ref_np._attn(W, p + "cross_attn.", n, ctx, cos, sin, False)
    sh, sc, g = O.block_mod(W, p + "adaln_modulation_mlp", emb, adaln_lora)
    n = O.layer_norm(x) * (1 + sc) + sh
    return (x + g * (O.gelu(n @ W(p + "mlp.layer1.weight").T) @ W(p + "mlp.layer2.weight").T)).astype(np.float32)


def _seq_worker(rank, world, port):
    dist = _init(rank, world, port)
    sh, syn = pkg("sharding"), pkg("synthetic")
    seq = sh.SeqGroup(rank, world, None)
    t = oracle.to_numpy(syn.global_tensors(3))
    t.update(oracle.to_numpy(syn.block_tensors(3, 0, "int8", 28, direct=True)))
    W = oracle.DequantWeights(t)
    Hp, Wp = 4, 8
    L = Hp * Wp
    x = syn.randn(3, "x", (L, 2048)).numpy()
    ctx = syn.randn(3, "ctx", (40, 1024)).numpy()
    _, adaln_lora, emb = oracle.time_cond(W, 0.7)
    cos, sin = oracle.dit_rope(Hp, Wp)
    cos, sin = np.concatenate([cos, cos], -1), np.concatenate([sin, sin], -1)
    full = oracle.dit_block(W, 0, x, ctx, emb, adaln_lora, cos, sin)
    lo, hi = seq.span(L)
    mine = _seq_block(W, 0, x[lo:hi], ctx, emb, adaln_lora, cos[lo:hi], sin[lo:hi], seq)
    err = np.abs(mine - full[lo:hi]).max() / np.abs(full[lo:hi]).max()
    assert err < 1e-5, err
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sequence_parallel_block_gloo(world):
    _spawn(_seq_worker, world)
