"""Euler flow sampling with optional classifier-free guidance, on the device
(app/pipeline.js:225-294 denoise/CFG glue, app/samplers.js:16-23 and 104-117; the math of
tools/reference.py:300-360).

The reference runs the sampler on the CPU and round-trips the latent through the host on every
DiT pass (dit.js:256, 322); here the latent stays on the GPU for the whole run, the modulation
vectors of every step are computed up front, and CFG's two passes run as one batch of 2.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import ops
from .dit import AnimaDiT, Cond


def sigmas_simple(steps: int, shift: float = 3.0) -> list[float]:
    """ComfyUI "simple" schedule over the shift-3 flow table, each sigma rounded to fp32
    (app/samplers.js:8-23, tools/reference.py:300-303)."""
    table = [shift * t / (1 + (shift - 1) * t) for t in (np.arange(1, 1001) / 1000.0)]
    ss = 1000 / steps
    return [float(np.float32(table[-(1 + int(x * ss))])) for x in range(steps)] + [0.0]


def sigmas_beta(steps: int, shift: float = 3.0, alpha: float = 0.6, beta: float = 0.6) -> list[float]:
    """ComfyUI "beta" scheduler over the same flow table (app/samplers.js:81-93): timestep
    t_i = round(999 * ppf(1 - i / steps)) of the Beta(0.6, 0.6) distribution, repeated timesteps
    dropped, so it can return fewer than `steps` steps. The Beta quantile comes from scipy's
    regularized incomplete beta inverse; the reference bisects its own CDF to the same value."""
    from scipy.special import betaincinv

    table = [float(np.float32(shift * t / (1 + (shift - 1) * t))) for t in (np.arange(1, 1001) / 1000.0)]
    out, last = [], -1
    for i in range(steps):
        p = 1 - i / steps
        q = 1.0 if p >= 1 else float(betaincinv(alpha, beta, p))
        t = int(np.floor(q * 999 + 0.5))  # JavaScript Math.round
        if t != last:
            out.append(table[t])
        last = t
    return out + [0.0]


SCHEDULERS = {"simple": sigmas_simple, "beta": sigmas_beta}
SAMPLERS = ("euler", "euler_a", "dpmpp_2m", "er_sde")


def sample(name: str, denoise, x: torch.Tensor, sigmas: list, seed: int = 0, shift: float = 3.0,
           on_step=None) -> torch.Tensor:
    """The reference's flow samplers on the device (app/samplers.js:104-218): euler, euler_a
    (sample_euler_ancestral_RF, eta 1), dpmpp_2m and er_sde (VP ER-SDE-Solver-3). x is the fp32
    latent on the device (updated in place), denoise(x, sigma, i) returns the x0 prediction as a
    new device tensor. Every update is one linear combination on the device (ops.lincomb); the
    stochastic samplers draw their noise from a CPU torch.Generator seeded with `seed` (the
    reference seeds a torch-compatible generator of its own the same way, samplers.js:104-106)."""
    if name not in SAMPLERS:
        raise ValueError(f"unknown sampler {name} (one of {', '.join(SAMPLERS)})")
    gen = torch.Generator().manual_seed(int(seed))

    def noise():
        return torch.randn(x.numel(), generator=gen).reshape(x.shape).to(x.device)

    n = len(sigmas) - 1
    if name == "er_sde":
        sg = list(sigmas)
        if sg[0] >= 1:
            sg[0] = float(np.float32(shift * (1 - 1e-4) / (1 + (shift - 1) * (1 - 1e-4))))
        lam = [0.0 if v == 0 else v / (1 - v) for v in sg]
    else:
        sg = sigmas
    scaler = lambda v: v * (math.exp(v ** 0.3) + 10)  # noqa: E731
    old = old_d = None
    for i in range(n):
        s, s1 = sg[i], sg[i + 1]
        den = denoise(x, s, i)
        if s1 == 0:
            x.copy_(den)
        elif name == "euler":
            ops.lincomb(x, (s1 / s, x), (1 - s1 / s, den))
        elif name == "euler_a":
            sigma_down = s1 * (s1 / s)
            alpha_ip1, alpha_down = 1 - s1, 1 - s1 * (s1 / s)
            renoise = math.sqrt(s1 * s1 - sigma_down * sigma_down * alpha_ip1 * alpha_ip1 / (alpha_down * alpha_down))
            r, k = sigma_down / s, alpha_ip1 / alpha_down
            ops.lincomb(x, (k * r, x), (k * (1 - r), den), (renoise, noise()))
        elif name == "dpmpp_2m":
            h = math.log(s) - math.log(s1)
            ratio, c = s1 / s, -math.expm1(-h)
            if old is None:
                ops.lincomb(x, (ratio, x), (c, den))
            else:
                r = (math.log(sg[i - 1]) - math.log(s)) / h
                ops.lincomb(x, (ratio, x), (c * (1 + 1 / (2 * r)), den), (-c / (2 * r), old))
        else:  # er_sde
            ls, lt = lam[i], lam[i + 1]
            alpha_s, alpha_t = s / ls, s1 / lt
            r = scaler(lt) / scaler(ls)
            a, b = alpha_t / alpha_s * r, alpha_t * (1 - r)
            stage = min(3, i + 1)
            if stage == 1:
                ops.lincomb(x, (a, x), (b, den))
            else:
                dt = lt - ls
                step = -dt / 200
                s_ = su = 0.0
                for p in range(200):
                    pos = lt + p * step
                    sp = scaler(pos)
                    s_ += 1 / sp
                    su += (pos - ls) / sp
                s_ *= step
                su *= step
                d_d = torch.empty_like(x)
                inv = 1 / (ls - lam[i - 1])
                ops.lincomb(d_d, (inv, den), (-inv, old))
                c2 = alpha_t * (dt + s_ * scaler(lt))
                if stage == 2:
                    ops.lincomb(x, (a, x), (b, den), (c2, d_d))
                else:
                    # x += c2 dD + c3 dU with dU = 2 (dD - old_dD) / (ls - lam[i-2])
                    c3 = alpha_t * (dt * dt / 2 + su * scaler(lt))
                    w = 2 / (ls - lam[i - 2])
                    ops.lincomb(x, (a, x), (b, den), (c2 + c3 * w, d_d), (-c3 * w, old_d))
                old_d = d_d
            nz = math.sqrt(max(0.0, lt * lt - ls * ls * r * r))
            if nz > 0:
                ops.lincomb(x, (1.0, x), (alpha_t * nz, noise()))
        old = den
        if on_step is not None:
            on_step(i, x, den)
    return x


def dit_denoiser(dit: AnimaDiT, cond: Cond, cfg: float = 1.0, uncond: Cond | None = None):
    """denoise(x, sigma, i) for `sample`: the DiT velocity with CFG as one batch of 2, combined as
    uncond + cfg (cond - uncond), and x0 = x - sigma v (pipeline.js:245-269)."""
    guided = uncond is not None and cfg != 1.0
    both = Cond.stack([cond, uncond]) if guided else cond
    tcs = {}

    def denoise(x, sigma, i):
        tc = tcs.get(sigma)
        if tc is None:
            tc = tcs[sigma] = dit.time_cond(sigma)
        den = torch.empty_like(x)
        if guided:
            B = x.shape[0]
            v2 = dit.forward(torch.cat([x, x]), both, tc)
            ops.lincomb(den, (1.0, x), (-sigma * cfg, v2[:B].contiguous()), (-sigma * (1 - cfg), v2[B:].contiguous()))
        else:
            ops.lincomb(den, (1.0, x), (-sigma, dit.forward(x, cond, tc)))
        return den

    return denoise


def denoise_loop(dit: AnimaDiT, noise: torch.Tensor, cond: Cond, steps: int, cfg: float = 1.0,
                 uncond: Cond | None = None, shift: float = 3.0, on_step=None) -> torch.Tensor:
    """Run `steps` Euler steps from noise [B, 16, h, w] (device) and return the final latent.

    x = noise * sigma_0; each step v = DiT(x) (CFG: v = vn + cfg (v - vn)), x0 = x - sigma v,
    x <- x0 if sigma' = 0 else x + (x - x0) / sigma * (sigma' - sigma)."""
    sig = sigmas_simple(steps, shift)
    tcs = dit.time_cond_batch(sig[:-1])
    x = (noise.to(dit.device, torch.float32) * np.float32(sig[0])).contiguous()
    B = x.shape[0]
    guided = uncond is not None and cfg != 1.0
    both = Cond.stack([cond, uncond]) if guided else cond
    for i in range(steps):
        s, s1 = sig[i], sig[i + 1]
        if guided:
            v2 = dit.forward(torch.cat([x, x]), both, tcs[i])
            ops.euler_step(x, v2[:B].contiguous(), s, s1, v_uncond=v2[B:].contiguous(), cfg=cfg)
        else:
            v = dit.forward(x, cond, tcs[i])
            ops.euler_step(x, v, s, s1)
        if on_step is not None:
            on_step(i, x)
    return x


class GraphedSampler:
    """The denoising loop captured as CUDA graphs, one per step (forward + CFG + Euler update), so a
    step replays ~400 kernel launches without host work in between. The latent lives in a static
    device buffer; load() copies a new starting latent in (x = noise * sigma_0 is done by the
    caller or by start()). Graphs share one memory pool and are replayed in order. Each replay adds
    the number of library kernels its capture enqueued to device.Context.launches."""

    def __init__(self, dit: AnimaDiT, cond: Cond, steps: int, batch: int, h: int, w: int, cfg: float = 1.0,
                 uncond: Cond | None = None, shift: float = 3.0, capture: int | None = None):
        """capture: graph only the first `capture` steps (a benchmark that replays those), else all."""
        self.dit, self.steps = dit, steps
        self.sig = sigmas_simple(steps, shift)
        self.tcs = dit.time_cond_batch(self.sig[:-1])
        self.guided = uncond is not None and cfg != 1.0
        self.cond = Cond.stack([cond, uncond]) if self.guided else cond
        self.cfg = cfg
        self.x = torch.zeros(batch, 16, h, w, dtype=torch.float32, device=dit.device)
        self.B = batch
        self.pool = None
        self.graphs = []
        stream = torch.cuda.Stream(device=dit.device)
        stream.wait_stream(torch.cuda.current_stream(dit.device))
        with torch.cuda.stream(stream):
            self._step(0)  # warm-up outside capture: kernel attributes, buffers, tensor maps
        torch.cuda.current_stream(dit.device).wait_stream(stream)
        torch.cuda.synchronize(dit.device)
        self.x.zero_()
        self.launches = []  # library kernels in each captured step
        from .device import Context
        for i in range(steps if capture is None else min(capture, steps)):
            g = torch.cuda.CUDAGraph()
            n0 = Context.launches
            with torch.cuda.graph(g, pool=self.pool, stream=stream):
                self._step(i)
            self.launches.append(Context.launches - n0)
            self.pool = g.pool()
            self.graphs.append(g)
        torch.cuda.synchronize(dit.device)
        # the graphs read and write the model's activation buffers by address: keep them alive even
        # if the model later runs another shape (which replaces its buffer set)
        self._keep = list(dit._bufs.values())

    def _step(self, i: int):
        s, s1 = self.sig[i], self.sig[i + 1]
        if self.guided:
            v2 = self.dit.forward(torch.cat([self.x, self.x]), self.cond, self.tcs[i])
            ops.euler_step(self.x, v2[: self.B].contiguous(), s, s1, v_uncond=v2[self.B:].contiguous(), cfg=self.cfg)
        else:
            v = self.dit.forward(self.x, self.cond, self.tcs[i])
            ops.euler_step(self.x, v, s, s1)

    def start(self, noise: torch.Tensor):
        """x <- noise * sigma_0 (the first Euler state)."""
        self.x.copy_(noise.to(self.x.device, torch.float32) * np.float32(self.sig[0]))

    def replay(self, i: int):
        from .device import Context
        self.graphs[i].replay()
        Context.launches += self.launches[i]

    def run(self, noise: torch.Tensor) -> torch.Tensor:
        if len(self.graphs) != self.steps:
            raise RuntimeError("run() needs every step captured (capture=None)")
        self.start(noise)
        for g in self.graphs:
            g.replay()
        return self.x


def generate(dit: AnimaDiT, noise, ctx, steps: int = 8, cfg: float = 1.0, ctx_neg=None, key_len=None,
             key_len_neg=None, shift: float = 3.0, sampler: str = "euler", scheduler: str = "simple",
             seed: int = 0) -> np.ndarray:
    """The public end-to-end call: host noise [B, 16, h, w] and text context(s) [Lk, 1024] in,
    final latent out on the host (pipeline.js:225-294 without the text encoder and VAE).
    sampler: euler | euler_a | dpmpp_2m | er_sde; scheduler: simple | beta; seed feeds the
    stochastic samplers' noise."""
    noise_d = torch.as_tensor(noise).to(dit.device, non_blocking=True)
    cond = dit.prepare_context(torch.as_tensor(ctx).to(dit.device, non_blocking=True), key_len)
    uncond = None
    if ctx_neg is not None and cfg != 1.0:
        uncond = dit.prepare_context(torch.as_tensor(ctx_neg).to(dit.device, non_blocking=True), key_len_neg)
    if sampler == "euler" and scheduler == "simple":
        x = denoise_loop(dit, noise_d, cond, steps, cfg, uncond, shift)   # fused CFG + Euler kernel
    else:
        if scheduler not in SCHEDULERS:
            raise ValueError(f"unknown scheduler {scheduler} (simple or beta)")
        sig = SCHEDULERS[scheduler](steps, shift)
        x = (noise_d.to(torch.float32) * np.float32(sig[0])).contiguous()
        x = sample(sampler, dit_denoiser(dit, cond, cfg, uncond), x, sig, seed=seed, shift=shift)
    return x.cpu().numpy()
