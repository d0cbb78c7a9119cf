"""Sequence parallelism on 2 GPUs: one image's token rows split over the ranks, k|v of all rows
exchanged for self-attention, either by the qkv GEMM storing its k|v tiles into every rank's buffer
over NVLink (peer memory, device barrier) or by an NCCL all-gather; both must deliver the same
k|v. The split forward must match the one-GPU forward of the same weights (the same kernels on
fewer rows) and the reference's own 28-block forward + 2 Euler steps at a 16x16 latent
(tests/golden/forward_int8_16x16.npz)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import GOLDEN, pkg

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
    g = dict(np.load(os.path.join(GOLDEN, "forward_int8_16x16.npz")))
    seed = int(g["seed"])
    tensors = syn.dit_tensors(seed, "int8", 28, direct=True)
    ctx = torch.cat([syn.randn(seed, "golden.ctx", (256, 1024)), torch.zeros(256, 1024)]).cuda()
    noise = torch.from_numpy(g["noise"])[None].cuda()
    seq = sh.SeqGroup(rank, world, None)
    dit = ditm.AnimaDiT(tensors, "cuda", seq=seq)       # k|v exchanged over peer memory
    cond = dit.prepare_context(ctx)
    sig = pl.sigmas_simple(2, 3.0)
    x0 = (noise * np.float32(sig[0])).contiguous()
    v_sp = dit.forward(x0, cond, dit.time_cond(sig[0]))
    lat_sp = pl.denoise_loop(dit, noise, cond, 2)
    # the graphed sampler with the qkv GEMMs' peer stores and the device barriers captured
    gs = pl.GraphedSampler(dit, cond, 2, 1, 16, 16)
    lat_graph = gs.run(noise).clone()
    lat_graph2 = gs.run(noise).clone()   # replays are repeatable (the barrier epochs live on the device)
    del gs
    dit.set_seq(seq, "nccl")                             # the same exchange through NCCL
    v_nccl = dit.forward(x0, cond, dit.time_cond(sig[0]))
    torch.cuda.synchronize()
    pkg("device").Context.get(rank).sync()
    dit.set_seq(None)
    if rank == 0:
        cref = dit.prepare_context(ctx)
        v_1 = dit.forward(x0, cref, dit.time_cond(sig[0]))
        lat_1 = pl.denoise_loop(dit, noise, cref, 2)
        np.savez(out_path, v_sp=v_sp.cpu().numpy(), v_1=v_1.cpu().numpy(), lat_sp=lat_sp.cpu().numpy(),
                 lat_1=lat_1.cpu().numpy(), lat_graph=lat_graph.cpu().numpy(), lat_graph2=lat_graph2.cpu().numpy(),
                 v_nccl=v_nccl.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_matches_single_gpu_and_reference(tmp_path):
    out = str(tmp_path / "sp.npz")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = np.load(out)
    g = np.load(os.path.join(GOLDEN, "forward_int8_16x16.npz"))
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    print(f"sp2 vs 1 GPU: velocity {rel(r['v_sp'], r['v_1']):.2e} latent {rel(r['lat_sp'], r['lat_1']):.2e}; "
          f"vs reference: velocity {rel(r['v_sp'][0], g['velocity0']):.2e} latent {rel(r['lat_sp'][0], g['latent_final']):.2e}")
    assert rel(r["v_sp"], r["v_1"]) < 1e-4
    assert rel(r["lat_sp"], r["lat_1"]) < 1e-4
    assert rel(r["lat_graph"], r["lat_sp"]) < 1e-6
    assert np.array_equal(r["lat_graph2"], r["lat_graph"])
    assert np.array_equal(r["v_nccl"], r["v_sp"])       # both exchanges deliver the same k|v
    assert rel(r["v_sp"][0], g["velocity0"]) < 3e-3
    assert rel(r["lat_sp"][0], g["latent_final"]) < 3e-3
