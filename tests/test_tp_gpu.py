"""Head-sharded tensor parallelism on 2 GPUs (NCCL): the sharded forward must match the one-GPU
forward of the same weights. Each rank quantizes its own slice of the attention output and the
MLP hidden with its own per-token scale, so the two runs differ by quantization noise only."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import pkg

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    syn, ditm, sh, pl = pkg("synthetic"), pkg("dit"), pkg("sharding"), pkg("pipeline")
    tensors = syn.dit_tensors(31, "int8", 2)
    ctx = syn.randn(31, "ctx", (77, 1024)).cuda()
    noise = syn.randn(31, "noise", (1, 16, 32, 32)).cuda()
    dit = ditm.AnimaDiT(tensors, "cuda", n_blocks=2, tp=sh.TPGroup(rank, world, None))
    cond = dit.prepare_context(ctx)
    tc = dit.time_cond(0.8)
    v_tp = dit.forward(noise * 0.8, cond, tc)
    lat_tp = pl.denoise_loop(dit, noise, cond, 2)
    torch.cuda.synchronize()
    if rank == 0:
        ref = ditm.AnimaDiT(tensors, "cuda", n_blocks=2)
        cref = ref.prepare_context(ctx)
        v_1 = ref.forward(noise * 0.8, cref, ref.time_cond(0.8))
        lat_1 = pl.denoise_loop(ref, noise, cref, 2)
        np.savez(out_path, v_tp=v_tp.cpu().numpy(), v_1=v_1.cpu().numpy(), lat_tp=lat_tp.cpu().numpy(),
                 lat_1=lat_1.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_matches_single_gpu(tmp_path):
    out = str(tmp_path / "tp.npz")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = np.load(out)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    assert rel(r["v_tp"], r["v_1"]) < 1e-3
    assert rel(r["lat_tp"], r["lat_1"]) < 1e-3
