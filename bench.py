"""Benchmark: DiT denoise steps/s at 1024^2 (4096 tokens) on 1..8 B200.

A step is one denoising step of the Turbo configuration: one 28-block INT8-ConvRot DiT forward at
1024x1024 (latent 16x128x128, L = 4096 tokens) plus the Euler update, batch 1, no CFG, the text
context a seeded 256x1024 N(0,1) block zero-padded to 512 rows as the reference does. Weights are
synthetic (N(0, 0.02) quantized with the reference's ConvRot int8 quantizer); inputs seeded.

  python bench.py [--gpus N --steps K --warmup W]           this implementation
  python bench.py --impl reference [...]                    the reference's algorithm on the CPU

Multi-GPU: one process per GPU (torchrun), each rank denoises its own image (data parallel, no
collective on the data path); the reported value is the whole job's steps/s, timed on the device
as the max over ranks.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DiT denoise steps/sec at 1024^2 (4096 tokens), 28-block INT8 ConvRot DiT"
WORKLOAD = ("BASELINE configs[2]: Turbo DiT, 28 blocks, INT8 ConvRot weights, 1024x1024 (latent 16x128x128, "
            "4096 tokens), batch 1 per GPU, Euler steps, no CFG, context 256x1024 zero-padded to 512 rows")


def pkg(sub):
    return importlib.import_module("anima-studio_b200." + sub)


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def traffic_from_profile():
    """Per-launch DRAM bytes of the mlp1 GEMM from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "gemm_i8_mlp1_L4096.md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    def __init__(self, index: int):
        self.path = os.path.join("/tmp", f"anima_clocks_{os.getpid()}.csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.close()
        rows = [r.split(", ") for r in open(self.path).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows), "reasons": sorted(reasons)}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------- reference arm (CPU)

def host_threads():
    """Threads for the CPU arms: every core this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its ranks, which would otherwise throttle BLAS to one thread)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def blas_on_all_cores(cores):
    """Lift the BLAS/OpenMP thread limits to `cores` whatever the environment says; returns the
    threadpoolctl context (kept alive by the caller) or None."""
    import torch

    torch.set_num_threads(cores)
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=cores)
    except ImportError:
        return None


def run_reference(args, world, rank):
    """The reference's algorithm (tools/reference.py, restated in numpy as oracle/) on the host
    cores. A step of this arm is one bounded sample of the workload: one of the 28 DiT blocks at
    L = 4096, so ms_per_step x steps is the timed region; `value` converts it to the metric's unit
    (DiT denoising steps/s = 1 / (28 x block time)). Under torchrun only rank 0 runs (the host's
    cores do the whole job whatever the GPU count); the other ranks exit without work."""
    if rank != 0:
        return
    import oracle
    from oracle import to_numpy as to_np

    cores = host_threads()
    limits = blas_on_all_cores(cores)  # noqa: F841  (holds the thread limits for the run)
    syn = pkg("synthetic")
    seed, Hp = 1234, 64
    L = Hp * Hp
    t = to_np(syn.global_tensors(seed))
    t.update(to_np(syn.block_tensors(seed, 0, "int8", 28, direct=True)))
    W = oracle.DequantWeights(t)
    ctx = np.concatenate([syn.randn(seed, "ctx", (256, 1024)).numpy(), np.zeros((256, 1024), np.float32)])
    x = syn.randn(seed, "x", (L, 2048)).numpy()
    _, adaln_lora, emb = oracle.time_cond(W, 0.9)
    cos, sin = oracle.dit_rope(Hp, Hp)
    cos, sin = np.concatenate([cos, cos], -1), np.concatenate([sin, sin], -1)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.dit_block(W, 0, x, ctx, emb, adaln_lora, cos, sin)
        times.append(time.perf_counter() - t0)
    timed = times[args.warmup:]
    region_s = sum(timed)
    block_s = region_s / len(timed)
    v = 1.0 / (28 * block_s)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": block_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": L, "blocks": 28,
                       "step_of_this_arm": "one bounded sample: one DiT block at L=4096 (1/28 of a denoising step); "
                                           "value = 1 / (28 x ms_per_step) denoising steps/s",
                       "timed_region_s": region_s, "samples_timed": len(timed),
                       "host": f"{cores} threads on the host's cores, rank 0 only"},
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": cores, "kind": "port",
                             "sample": f"{len(timed)} x one DiT block at L=4096 ({block_s:.2f} s each, "
                                       f"{region_s:.1f} s timed), x28 blocks per denoising step; numpy restatement of "
                                       "tools/reference.py (fp32, BLAS threads = cores)"},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- this implementation

def cpu_baseline_sample(seconds_budget=25.0):
    """The oracle port timed on the host cores on a bounded sample (one block at L=4096)."""
    import oracle
    from oracle import to_numpy as to_np

    cores = host_threads()
    limits = blas_on_all_cores(cores)  # noqa: F841
    syn = pkg("synthetic")
    seed, Hp = 1234, 64
    t = to_np(syn.global_tensors(seed))
    t.update(to_np(syn.block_tensors(seed, 0, "int8", 28, direct=True)))
    W = oracle.DequantWeights(t)
    ctx = np.concatenate([syn.randn(seed, "ctx", (256, 1024)).numpy(), np.zeros((256, 1024), np.float32)])
    x = syn.randn(seed, "x", (Hp * Hp, 2048)).numpy()
    _, adaln_lora, emb = oracle.time_cond(W, 0.9)
    cos, sin = oracle.dit_rope(Hp, Hp)
    cos, sin = np.concatenate([cos, cos], -1), np.concatenate([sin, sin], -1)
    oracle.dit_block(W, 0, x, ctx, emb, adaln_lora, cos, sin)  # warm (dequantized weights cached)
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.dit_block(W, 0, x, ctx, emb, adaln_lora, cos, sin)
        n += 1
        if time.perf_counter() - t0 > seconds_budget / 2 or n >= 3:
            break
    block_s = (time.perf_counter() - t0) / n
    return {"value": 1.0 / (28 * block_s), "unit": "steps/s", "cores": cores, "kind": "port",
            "sample": f"{n} x one DiT block at L=4096 ({block_s:.2f} s each), x28 blocks per step; numpy restatement "
                      "of tools/reference.py, fp32, BLAS on all host cores"}


def measure_int8_peak(torch):
    """Dense int8 tensor-core throughput of cuBLASLt (torch._int_mm, 8192^3), as the int8
    roofline denominator (MEASURED_PEAKS.json has only bf16)."""
    n = 8192
    a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def kernel_case(args):
    """One kernel of the 1024^2 workload in isolation (for ncu captures and kernel timing):
    mlp1  the 2048->8192 block linear (M=4096, two activation planes, GELU, fp16 out)
    mlp2  the 8192->2048 block linear with the gated residual
    qkv   the 2048->6144 qkv linear with the per-head RMSNorm + RoPE epilogue
    attn  self-attention, 16 heads x 4096 tokens x d=128 (fp16 q/k/v in the qkv layout)
    xattn cross-attention, 4096 queries x 512 context rows (k|v stacked per row), 16 heads
    ln    LayerNorm + adaLN + ConvRot + two-plane quantization of [4096, 2048]
    gelu  GELU + ConvRot + quantization of the fp16 MLP hidden [4096, 8192]
    rotq  ConvRot + quantization of the fp16 attention output [4096, 2048]
    rotq8k  ConvRot + quantization of the fp16 MLP hidden after GELU [4096, 8192]
    xembed / final  the fp32 SIMT GEMMs of the patch embedding (68 -> 2048) and the final layer (2048 -> 64)"""
    import torch

    syn, ditm, ops, W = pkg("synthetic"), pkg("dit"), pkg("ops"), pkg("weights")
    dev = pkg("device")
    torch.manual_seed(0)
    M = 4096
    planes = 2 if args.precision == "a16" else 1

    def lin(N, K):
        q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
        return W.Linear("i8", N, K, q, torch.full((N,), 1e-3, device="cuda"))

    if args.kernel in ("mlp1", "mlp2", "qkv", "oproj"):
        N, K = {"mlp1": (8192, 2048), "mlp2": (2048, 8192), "qkv": (6144, 2048), "oproj": (2048, 2048)}[args.kernel]
        w = lin(N, K)
        qa = ops.rotate_quant(torch.randn(M, K, device="cuda"), planes)
        if args.kernel == "mlp1":
            out = torch.empty(M, N, dtype=torch.float16 if args.out == "f16" else torch.float32, device="cuda")
            act = None if args.act == "none" else args.act
            fn = lambda: ops.linear(qa, w, out=out, act=act)  # noqa: E731
        elif args.kernel in ("mlp2", "oproj"):
            out = torch.zeros(M, N, device="cuda")
            gate = torch.randn(6144, device="cuda")
            fn = lambda: ops.linear(qa, w, out=out, resid=True, gate=gate, g_off=4096)  # noqa: E731
        else:
            out = torch.empty(M, N, dtype=torch.float16, device="cuda")
            nq, nk = torch.ones(128, device="cuda"), torch.ones(128, device="cuda")
            cs = torch.from_numpy(ditm.rope_table(64, 64)).cuda()
            fn = lambda: ops.linear(qa, w, out=out, mode="qkv", qk=(nq, nk), rope_cs=cs, n_q=2048)  # noqa: E731
        work, unit = 2.0 * M * N * K, "TOPS"
    elif args.kernel == "w4":
        # a W4A8 2048 -> 8192 linear: the per-call decode of the packed weight, then the int8 GEMM
        quant = pkg("quant")
        q = quant.quantize_w4a8(torch.randn(8192, 2048, device="cuda") * 0.02)
        w = W.linear_weights({"l." + k: v for k, v in q.items()}, "l.", "cuda")
        qa = ops.rotate_quant(torch.randn(M, 2048, device="cuda"), planes)
        out = torch.empty(M, 8192, dtype=torch.float16, device="cuda")
        fn = lambda: ops.linear(qa, w, out=out)  # noqa: E731
        work, unit = 2.0 * M * 8192 * 2048, "TOPS"
    elif args.kernel == "attn":
        dt = torch.float16 if args.attn == "f16" else torch.bfloat16
        qkv = torch.randn(M, 6144, device="cuda").to(dt)
        out = torch.empty(M, 2048, dtype=dt, device="cuda")
        fn = lambda: ops.attention(qkv, qkv, qkv, Lq=M, Lk=M, H=16, ldq=6144, ldk=6144, ldv=6144, q_off=0,  # noqa: E731
                                   k_off=2048, v_off=4096, out=out)
        work, unit = 4.0 * M * M * 128 * 16, "TFLOP/s"
    elif args.kernel == "xattn":
        # cross-attention of one DiT block: 4096 queries against the 512-row (zero-padded) context
        dt = torch.float16 if args.attn == "f16" else torch.bfloat16
        q = torch.randn(M, 2048, device="cuda").to(dt)
        kv = torch.randn(512, 4096, device="cuda").to(dt)
        out = torch.empty(M, 2048, dtype=dt, device="cuda")
        fn = lambda: ops.attention(q, kv, kv, Lq=M, Lk=512, H=16, ldk=4096, ldv=4096, k_off=0, v_off=2048,  # noqa: E731
                                   out=out)
        work, unit = 4.0 * M * 512 * 128 * 16, "TFLOP/s"
    elif args.kernel == "ln":
        x = torch.randn(M, 2048, device="cuda")
        mod = torch.randn(6144, device="cuda") * 0.5
        q = ops.QuantRows.empty(M, 2048, planes, "cuda")
        fn = lambda: ops.layernorm_mod_quant(x, mod, 0, 2048, 2048, out=q)  # noqa: E731
        work, unit = M * 2048 * (4 + planes) + M * 4, "GB/s"
    elif args.kernel in ("xembed", "final"):
        N, K = (2048, 68) if args.kernel == "xembed" else (64, 2048)
        a = torch.randn(M, K, device="cuda")
        w = W.Linear("bf16", N, K, (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16), None)
        out = torch.empty(M, N, device="cuda")
        fn = lambda: ops.matmul(a, w, out=out)  # noqa: E731
        work, unit = 2.0 * M * N * K, "TFLOP/s"
    elif args.kernel == "vae":
        # the Wan-2.1 decoder on a 128x128 latent -> one 1024x1024 image (once per image)
        dec = pkg("vae").VAEDecoder(syn.vae_tensors(1), "cuda")
        lat = torch.randn(16, 128, 128, device="cuda")
        fn = lambda: dec.decode(lat)  # noqa: E731
        work, unit = 1.0, "images/s"
    elif args.kernel == "te":
        # Qwen3-0.6B (28 int8 layers) on 512 tokens, then the LLM adapter on 512 T5 tokens
        text = pkg("text")
        te = text.Qwen3(syn.te_tensors(1, 28, 4096, direct=True), "cuda")
        ad = text.LLMAdapter(syn.adapter_tensors(1, 6, 4096), "cuda")
        ids = torch.randint(0, 4096, (512,)).tolist()
        fn = lambda: ad(te.encode(ids), ids)  # noqa: E731
        work, unit = 1.0, "prompts/s"
    elif args.kernel in ("gelu", "rotq", "rotq8k"):
        K = 2048 if args.kernel == "rotq" else 8192
        h = torch.randn(M, K, device="cuda").half()
        q = ops.QuantRows.empty(M, K, planes, "cuda")
        act = "gelu" if args.kernel == "gelu" else None
        fn = lambda: ops.rotate_quant(h, planes, out=q, act=act)  # noqa: E731
        work, unit = M * K * (2 + planes) + M * 4, "GB/s"
    else:
        raise SystemExit(f"unknown kernel case {args.kernel}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    # each sample times `batch` back-to-back launches replayed from a CUDA graph, so short kernels
    # are not measured with the host's per-call latency (Python, ctypes, launch); the VAE and text
    # encoder cases, which read sizes back to the host, run eagerly. Inputs stay L2-resident
    # between launches when they fit.
    graph = None
    if not args.no_graph and args.kernel not in ("vae", "te"):
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=side):
            for _ in range(args.batch):
                fn()
        torch.cuda.current_stream().wait_stream(side)
    ts = []
    for _ in range(args.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.batch):
                fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) / args.batch)
    dev.Context.get(0).sync()
    ms = statistics.median(ts)
    rate = work / (ms * 1e-3) / {"GB/s": 1e9, "images/s": 1.0, "prompts/s": 1.0}.get(unit, 1e12)
    print(json.dumps({"kernel": args.kernel, "precision": args.precision, "attn": args.attn, "graph": graph is not None,
                      "ms_median": ms,
                      "ms_min": min(ts), "rate": rate, "unit": unit, "reps": args.reps}), flush=True)


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def time_graphed(gs, noise, steps, warmup, world):
    """Replay a GraphedSampler's captured steps in order (restarting from the noise after the last
    one): `warmup` untimed steps, then `steps` timed with CUDA events on the replay stream between
    device synchronizations and barriers; returns the max over ranks in ms."""
    import torch

    sh = pkg("sharding")
    n = len(gs.graphs)
    gs.start(noise)

    def step(i):
        j = i % n
        gs.replay(j)
        if j == n - 1:
            gs.start(noise)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(warmup + i)
    e1.record()
    torch.cuda.synchronize()
    _barrier(world)
    return sh.max_over_ranks(e0.elapsed_time(e1), "cuda")


def step_profile(dit, fn, peaks):
    """One eager pass of fn() with CUDA events around every linear and attention launch: ms and
    achieved rate per op family (int8 TOPS for the linears, TFLOP/s for attention)."""
    dev = pkg("device")
    with dev.KernelTimer({"anima_linear", "anima_attention"}) as kt:
        fn()
    summ = kt.summary()
    out = {}
    for name, unit in (("anima_linear", "TOPS"), ("anima_attention", "TFLOP/s")):
        ms = sum(v[1] for k, v in summ.items() if k[0] == name)
        work = sum(v[2] for k, v in summ.items() if k[0] == name)
        rate = work / (ms * 1e-3) / 1e12 if ms else None
        out[name.replace("anima_", "")] = {"ms": ms, "rate": rate, "unit": unit}
    if out["attention"]["rate"] and peaks.get("bf16_tflops"):
        out["attention"]["frac_of_bf16_peak"] = out["attention"]["rate"] / peaks["bf16_tflops"]
    return out


def measure_cfg(dit, seed, res, cfg, steps, warmup, world, rank, peaks, int8_peak=None):
    """BASELINE configs[4] on this model: classifier-free guidance (cond and a negative context as
    one batch of 2 per image), Euler over the base model's 30-step schedule, res x res; each rank
    denoises its own image (its first seed of the 64), no collective on the data path."""
    import torch

    syn, pl = pkg("synthetic"), pkg("pipeline")
    lat = res // 8
    pad = torch.zeros(256, 1024)
    cond = dit.prepare_context(torch.cat([syn.randn(seed, "ctx", (256, 1024)), pad]).cuda())
    uncond = dit.prepare_context(torch.cat([syn.randn(seed, "ctx_neg", (256, 1024)), pad]).cuda())
    image = pkg("sharding").seed_shard(64, rank, world)[0] if world <= 64 else rank
    noise = syn.randn(seed + image, "noise", (1, 16, lat, lat)).cuda()
    gs = pl.GraphedSampler(dit, cond, 30, 1, lat, lat, cfg=cfg, uncond=uncond, capture=min(8, 30))
    ms = time_graphed(gs, noise, steps, warmup, world)
    del gs
    both = pkg("dit").Cond.stack([cond, uncond])
    tc = dit.time_cond(pl.sigmas_simple(30, 3.0)[0])
    x2 = torch.cat([noise, noise])
    prof = step_profile(dit, lambda: dit.forward(x2, both, tc), peaks)
    if int8_peak and prof["linear"]["rate"]:
        prof["linear"]["frac_of_int8_peak"] = prof["linear"]["rate"] / int8_peak
    steps_per_s = world * steps / (ms * 1e-3)
    tokens = (lat // 2) ** 2
    return {"res": res, "tokens": tokens, "rows_per_gemm": 2 * tokens, "cfg": cfg, "steps_per_image": 30,
            "steps_per_s": steps_per_s, "images_per_s": steps_per_s / 30, "ms_per_step": ms / steps,
            "steps_timed_per_rank": steps, "job": f"64 seeded images split over {world} rank(s); rate from "
            f"{steps} timed steps per rank", "per_op": prof}


def measure_seq(dit, seed, steps, warmup, world, rank, exchange="peer"):
    """One image denoised by all ranks together: its 4096 token rows split over the ranks
    (sequence parallelism, one k|v all-gather per block), Euler 8-step schedule, CUDA graph per
    step with the all-gathers captured in it. Returns the single-image rate."""
    import torch

    syn, pl, sh = pkg("synthetic"), pkg("pipeline"), pkg("sharding")
    dit.set_seq(sh.SeqGroup(rank, world, None), exchange)
    try:
        cond = dit.prepare_context(torch.cat([syn.randn(seed, "ctx", (256, 1024)), torch.zeros(256, 1024)]).cuda())
        noise = syn.randn(seed, "noise", (1, 16, 128, 128)).cuda()   # the same image on every rank
        gs = pl.GraphedSampler(dit, cond, 8, 1, 128, 128)
        ms = time_graphed(gs, noise, steps, warmup, world)
        del gs
    finally:
        dit.set_seq(None)
    how = ("the qkv GEMM stores its k|v tiles into every rank's buffer over NVLink, then a device barrier"
           if exchange == "peer" else "a copy and an NCCL all-gather")
    return {"workload": "one 1024x1024 image, 28 INT8 ConvRot blocks, token rows split over the ranks; k|v of all "
                        f"rows (fp16, 16 MiB) exchanged once per block: {how}; CUDA graph per step",
            "exchange": exchange, "n_gpus": world,
            "steps_per_s": steps / (ms * 1e-3), "ms_per_step": ms / steps, "steps": steps, "scaling": "strong"}


def one_plane_probe(dit, cond, tc):
    """The one-plane (W8A8, precision "a8") form of the 2048->8192 linear, where the north star's
    int8 tensor-core fraction is defined, and what that precision does to one DiT block at
    L = 4096: the block output's relative L2 distance from the default two-plane path (itself
    within ~3e-4 of the reference at this size)."""
    import torch

    ops, syn = pkg("ops"), pkg("synthetic")
    M, K = 4096, 2048
    w = dit.blocks[0]["l1"]
    x = syn.randn(7, "probe.x", (M, K)).cuda()
    q1 = ops.rotate_quant(x, 1)
    out = torch.empty(M, w.N, dtype=torch.float16, device="cuda")
    for _ in range(3):
        ops.linear(q1, w, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        ops.linear(q1, w, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    res = {}
    xb = syn.randn(7, "probe.block", (M, 2048)).cuda()
    cs = dit.rope(64, 64)
    for planes in (2, 1):
        dit.planes, dit._bufs = planes, {}
        y = xb.clone()
        dit.block(0, y, cond, tc, 1, M, cs, dit._buffers(M))
        res[planes] = y
    dit.planes, dit._bufs = 2, {}
    err = float((res[1] - res[2]).norm() / res[2].norm())
    return {"launch_ms": ms, "achieved": 2.0 * M * w.N * K / (ms * 1e-3) / 1e12, "block_rel_l2_vs_a16": err}


def load_model(args, seed, fmt="int8"):
    import torch

    syn, ditm = pkg("synthetic"), pkg("dit")
    tensors = syn.dit_tensors(seed, fmt, 28, device="cuda", direct=fmt != "int8")
    dit = ditm.AnimaDiT(tensors, "cuda", precision=args.precision,
                        attn_dtype=torch.bfloat16 if args.attn == "bf16" else torch.float16)
    del tensors
    torch.cuda.empty_cache()
    return dit


def init_dist(world, local):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))


def run_tp(args, world, rank, local):
    """--tp: the single-image latency run alone (sequence parallel over the --gpus ranks)."""
    import torch.distributed as dist

    init_dist(world, local)
    dit = load_model(args, 1234)
    clocks = ClockSampler(local)
    r = measure_seq(dit, 1234, args.steps, args.warmup, world, rank)
    clk = clocks.stop()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": "DiT denoise steps/sec at 1024^2 (4096 tokens) for one image, sequence parallel",
            "value": r["steps_per_s"], "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "BASELINE configs[4] latency run: " + r["workload"], "parallelism": f"sp{world}",
                       "precision": args.precision, "attention": args.attn}, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_cfg(args, world, rank, local):
    """--cfg: the configs[4] CFG run alone at --res (seeds split over the ranks, weak scaling)."""
    import torch.distributed as dist

    init_dist(world, local)
    dit = load_model(args, 1234)
    peaks = load_peaks()
    clocks = ClockSampler(local)
    r = measure_cfg(dit, 1234, args.res, args.cfg, args.steps, args.warmup, world, rank, peaks)
    clk = clocks.stop()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": f"DiT denoise steps/sec with CFG (batch 2 per image) at {args.res}^2 ({r['tokens']} tokens)",
            "value": r["steps_per_s"], "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"BASELINE configs[4]: base model, INT8 ConvRot, cfg {args.cfg} with a negative "
                                   f"context (cond and uncond as one batch of 2), Euler 30 steps per image, "
                                   f"{args.res}x{args.res}", **r, "launch": "CUDA graph per step",
                       "parallelism": f"dp{world}", "precision": args.precision, "attention": args.attn},
            "clocks": clk}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default=None, help="time one kernel case instead (mlp1|mlp2|qkv|oproj|w4|attn|xattn|ln|gelu|rotq|xembed|final|vae|te)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=10, help="kernel cases: launches per timed sample")
    ap.add_argument("--act", default="gelu", help="kernel case mlp1: epilogue activation (gelu|none)")
    ap.add_argument("--out", default="f16", help="kernel case mlp1: output dtype (f16|f32)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="anima", choices=["anima", "reference"])
    ap.add_argument("--precision", default="a16", choices=["a16", "a8"])
    ap.add_argument("--attn", default="f16", choices=["bf16", "f16"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch kernels from Python per step (kernel cases: per launch) instead of CUDA graphs")
    ap.add_argument("--cfg", type=float, default=None,
                    help="BASELINE configs[4]: guidance scale with a negative context (batch 2 per image), 30 steps")
    ap.add_argument("--res", type=int, default=1024, help="with --cfg: image side (1024 or 1536)")
    ap.add_argument("--tp", action="store_true",
                    help="single-image latency alone: token rows split over the --gpus ranks (sequence parallel)")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the configs[4] measurements the default line carries (cfg; tp at N > 1)")
    ap.add_argument("--fmt", default="int8", choices=["int8", "mixed"],
                    help="DiT weights: int8 (configs[2]) or W4A8 'mixed', blocks 2-27 W4A8 (configs[3])")
    ap.add_argument("--lora", type=int, default=0,
                    help="rank of a LoRA on q/k/v and both MLP linears of every block (configs[3]: 32); the "
                         "line then also carries the step time without it (the LoRA overhead)")
    args = ap.parse_args()
    world, rank, local = setup_dist()
    if args.kernel:
        return kernel_case(args)
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if args.tp:
        return run_tp(args, world, rank, local)
    if args.cfg is not None:
        return run_cfg(args, world, rank, local)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = pkg("device")
    syn, ditm, ops, pl = pkg("synthetic"), pkg("dit"), pkg("ops"), pkg("pipeline")

    headline = args.fmt == "int8" and not args.lora
    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and headline:
        cpu_base = cpu_baseline_sample()  # before any CUDA work (keeps BLAS threads off the GPU feeder)

    seed = 1234
    # int8: Gaussian weights through the reference's int8 ConvRot quantizer (on the GPU); mixed: the
    # stored formats drawn directly (W4 codes and fp8 group scales), the decode and GEMM cost the same
    tensors = syn.dit_tensors(seed, args.fmt, 28, device="cuda", direct=args.fmt != "int8")
    dit = ditm.AnimaDiT(tensors, "cuda", precision=args.precision,
                        attn_dtype=torch.bfloat16 if args.attn == "bf16" else torch.float16)
    del tensors
    torch.cuda.empty_cache()
    Linear = pkg("weights").Linear
    weight_bytes = sum(w.nbytes() for blk in dit.blocks for w in blk.values() if isinstance(w, Linear))
    ctx = torch.cat([syn.randn(seed, "ctx", (256, 1024)), torch.zeros(256, 1024)]).cuda()
    cond = dit.prepare_context(ctx)
    sig = pl.sigmas_simple(8, 3.0)
    tcs = dit.time_cond_batch(sig[:-1])
    noise = syn.randn(seed + rank, "noise", (1, 16, 128, 128)).cuda()
    x = noise * sig[0]
    lora_info = None
    if args.lora:
        # the same steps without the LoRA first (graphed), for the overhead the reference quotes
        # (README.md:153: ~+20% per step)
        g0 = pl.GraphedSampler(dit, cond, 8, 1, 128, 128)
        g0.start(noise)
        for i in range(3):
            g0.replay(i)
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        for i in range(16):
            g0.replay(i % 8)
        b1.record()
        torch.cuda.synchronize()
        base_ms = b0.elapsed_time(b1) / 16
        del g0
        lora = pkg("lora")
        targets = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.layer1", "mlp.layer2")
        lt = syn.lora_tensors(seed, targets, rank=args.lora, std=0.01, n_blocks=28, alpha=float(args.lora))
        reg = lora.linear_registry(dit.blocks)
        lo = lora.load_lora(lt, reg, device="cuda")
        lora.attach_loras([reg], [(lo, 1.0)])
        lora_info = {"rank": args.lora, "modules": lo.matched, "targets": list(targets),
                     "ms_per_step_without_lora": base_ms}
    graphed = None
    if not args.no_graph:
        graphed = pl.GraphedSampler(dit, cond, 8, 1, 128, 128)
        graphed.start(noise)

    def step(i):
        j = i % 8
        if graphed is not None:
            graphed.replay(j)
            if j == 7:  # next image: restart from the noise
                graphed.start(noise)
            return
        v = dit.forward(x, cond, tcs[j])
        ops.euler_step(x, v, sig[j], sig[j + 1])
        if j == 7:
            x.copy_(noise * sig[0])

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    launches0 = dev.Context.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = dev.Context.launches - launches0
    ms_max = pkg("sharding").max_over_ranks(e0.elapsed_time(e1), "cuda")
    value = world * args.steps / (ms_max * 1e-3)

    # Per-kernel durations: an instrumented replay of the same steps (CUDA events around each
    # launch on the launching stream), for the roofline of the dominant kernel.
    with dev.KernelTimer({"anima_linear", "anima_attention"}) as kt:
        xr = noise * sig[0]
        for i in range(min(args.steps, 8)):  # eager launches, so each kernel is bracketed by events
            j = i % 8
            v = dit.forward(xr, cond, tcs[j])
            ops.euler_step(xr, v, sig[j], sig[j + 1])
    summ = kt.summary()
    replay_steps = min(args.steps, 8)

    # e2e through the public step API with host buffers: each step uploads the latent from pinned
    # host memory, runs the DiT and the Euler update, and reads the new latent back.
    e2e = None
    if not args.no_e2e:
        xh = torch.empty(1, 16, 128, 128, pin_memory=True)
        xh.copy_(x.cpu())
        xd = graphed.x if graphed is not None else torch.empty_like(x)

        def e2e_step(j):
            xd.copy_(xh, non_blocking=True)
            if graphed is not None:
                graphed.replay(j)
            else:
                v = dit.forward(xd, cond, tcs[j])
                ops.euler_step(xd, v, sig[j], sig[j + 1])
            xh.copy_(xd, non_blocking=True)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for i in range(args.steps):
            e2e_step(i % 8)
        f1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        barrier()
        et = pkg("sharding").max_over_ranks(max(f0.elapsed_time(f1), wall * 1e3), "cuda")
        nbytes = xh.numel() * 4
        e2e = {"value": world * args.steps / (et * 1e-3), "unit": "steps/s",
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
               "api": "per step: pinned host latent -> device, pipeline.GraphedSampler step (AnimaDiT.forward + "
                      "euler_step as one CUDA graph), latent -> pinned host (the reference's per-pass host round trip, "
                      "dit.js:256,322)"}

    peaks = load_peaks()
    # BASELINE configs[4] on every run (all ranks, same order): the CFG sweep at 1024^2 and 1536^2
    # (each rank its own image), and with more than one rank the single-image sequence-parallel run
    subs = {}
    if headline and not args.no_sub:
        graphed = None  # the headline graphs are done; free their pool before the larger shapes
        torch.cuda.empty_cache()
        subs["cfg"] = [measure_cfg(dit, seed, res, 4.5, n, 3, world, rank, peaks)
                       for res, n in ((1024, 12), (1536, 6))]
        if world > 1:
            subs["tp"] = measure_seq(dit, seed, 16, 3, world, rank)
            subs["tp"]["nccl_exchange"] = measure_seq(dit, seed, 16, 3, world, rank, "nccl")
    a8 = one_plane_probe(dit, cond, tcs[0]) if rank == 0 and headline and args.precision == "a16" else None
    int8_peak = measure_int8_peak(torch) if rank == 0 else None
    dist.destroy_process_group() if world > 1 else None
    if rank != 0:
        return
    for c in subs.get("cfg", []):
        lin = c["per_op"]["linear"]
        if int8_peak and lin["rate"]:
            lin["frac_of_int8_peak"] = lin["rate"] / int8_peak

    # roofline of the dominant kernel: the int8 GEMM over all its launches in a step, and the
    # north star's 2048->8192 linear (mlp1) alone
    lin = {k: v for k, v in summ.items() if k[0] == "anima_linear"}
    lin_n = sum(v[0] for v in lin.values())
    lin_ms = sum(v[1] for v in lin.values())
    lin_work = sum(v[2] for v in lin.values())
    att = {k: v for k, v in summ.items() if k[0] == "anima_attention"}
    att_ms = sum(v[1] for v in att.values())
    att_work = sum(v[2] for v in att.values())
    mlp1 = summ.get(("anima_linear", "dit.mlp1"), (1, 0.0, 0.0))
    step_ms_replay = None
    planes = 2 if args.precision == "a16" else 1
    achieved = lin_work / (lin_ms * 1e-3) / 1e12 if lin_ms else 0.0
    traffic = traffic_from_profile()
    mlp1_n = max(mlp1[0], 1)
    mlp1_ms = mlp1[1] / mlp1_n
    mlp1_work = mlp1[2] / mlp1_n
    mlp1_ach = mlp1_work / (mlp1_ms * 1e-3) / 1e12 if mlp1_ms else 0.0
    roof = {"kernel": "gemm_i8_kernel, the 2048->8192 block linear (dit.mlp1): M=4096 N=8192 K=2048",
            "bound": "tensor", "achieved": mlp1_ach, "peak": int8_peak, "unit": "TOPS",
            "frac": mlp1_ach / int8_peak if int8_peak else None,
            "peak_source": "measured: cuBLASLt int8 GEMM 8192^3 (torch._int_mm) on this GPU (MEASURED_PEAKS.json has no int8 entry)",
            "traffic": traffic,
            "launch_ms": mlp1_ms, "work_per_launch": mlp1_work,
            "hw_ops_frac": planes * mlp1_ach / int8_peak if int8_peak else None,
            "all_linears": {"achieved_tops": achieved, "frac": achieved / int8_peak if int8_peak else None,
                            "launches_per_step": lin_n / replay_steps, "ms_per_step": lin_ms / replay_steps},
            "attention": {"ms_per_step": att_ms / replay_steps,
                          "achieved_tflops": att_work / (att_ms * 1e-3) / 1e12 if att_ms else None,
                          "peak_bf16_tflops": peaks.get("bf16_tflops"),
                          "frac": (att_work / (att_ms * 1e-3) / 1e12) / peaks["bf16_tflops"]
                          if att_ms and peaks.get("bf16_tflops") else None},
            "per_op_ms_per_step": {f"{k[0].replace('anima_', '')}:{k[1]}": round(v[1] / replay_steps, 3)
                                   for k, v in sorted(summ.items(), key=lambda kv: -kv[1][1])},
            "one_plane": dict(a8, frac=a8["achieved"] / int8_peak if int8_peak else None) if a8 else None,
            "note": "achieved = algorithmic 2MNK ops per launch / CUDA-event time per launch, measured on the "
                    "launching stream in an instrumented replay of the timed steps; a16 runs two int8 MMAs per "
                    "product, so its frac is capped at 0.5 by construction and hw_ops_frac = planes x frac; "
                    "one_plane = the same linear with one int8 activation plane (W8A8, the north star's int8 "
                    "figure), timed alone, with its DiT-block error against the a16 path; traffic = DRAM bytes per "
                    "launch from the ncu capture in profiles/gemm_i8_mlp1_L4096.md"}
    metric, workload = METRIC, WORKLOAD
    if not headline:
        metric = ("DiT denoise steps/sec at 1024^2 (4096 tokens), 28-block W4A8-mixed ConvRot DiT"
                  + (f" + rank-{args.lora} LoRA" if args.lora else ""))
        workload = ("BASELINE configs[3]: W4A8 'mixed' DiT (blocks 1 and 28 INT8, blocks 2-27 4-bit codes with fp8 "
                    "group scales, decoded per linear into the int8 GEMM), ConvRot, 1024x1024, batch 1 per GPU, "
                    "Euler steps, context 256x1024 zero-padded to 512 rows"
                    + (f"; rank-{args.lora} LoRA (A, B ~ N(0, 0.01)) on q/k/v and both MLP linears of every block"
                       if args.lora else ""))
    if lora_info:
        lora_info["overhead"] = (ms_max / args.steps) / lora_info["ms_per_step_without_lora"] - 1.0
    line = {"metric": metric, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": workload, "fmt": args.fmt, "lora": lora_info,
                       "block_weight_bytes": weight_bytes, "tokens": 4096, "blocks": 28, "batch_per_gpu": 1,
                       "launch": "CUDA graph per step" if graphed is not None else "eager",
                       "precision": args.precision, "attention": args.attn, "ctx_rows": 512,
                       "parallelism": f"dp{world}", "images_per_s": value / 8,
                       "l2": "inputs larger than L2: 1.5 GB of int8 weights stream through every step"},
            "roofline": roof, "cpu_baseline": cpu_base, "e2e": e2e, **subs,
            "gpu_launches": launches, "gpu_launches_per_step": launches / args.steps, "clocks": clk}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
