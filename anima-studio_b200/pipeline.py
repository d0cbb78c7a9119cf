"""Euler flow sampling with optional classifier-free guidance, on the device
(app/pipeline.js:225-294 denoise/CFG glue, app/samplers.js:16-23 and 104-117; the math of
tools/reference.py:300-360).

The reference runs the sampler on the CPU and round-trips the latent through the host on every
DiT pass (dit.js:256, 322); here the latent stays on the GPU for the whole run, the modulation
vectors of every step are computed up front, and CFG's two passes run as one batch of 2.
"""

from __future__ import annotations

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
                 uncond: Cond | None = None, shift: float = 3.0):
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
        for i in range(steps):
            g = torch.cuda.CUDAGraph()
            n0 = Context.launches
            with torch.cuda.graph(g, pool=self.pool, stream=stream):
                self._step(i)
            self.launches.append(Context.launches - n0)
            self.pool = g.pool()
            self.graphs.append(g)
        torch.cuda.synchronize(dit.device)

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
        self.start(noise)
        for g in self.graphs:
            g.replay()
        return self.x


def generate(dit: AnimaDiT, noise, ctx, steps: int = 8, cfg: float = 1.0, ctx_neg=None, key_len=None,
             key_len_neg=None, shift: float = 3.0) -> np.ndarray:
    """The public end-to-end call: host noise [B, 16, h, w] and text context(s) [Lk, 1024] in,
    final latent out on the host (pipeline.js:225-294 without the text encoder and VAE)."""
    noise_d = torch.as_tensor(noise).to(dit.device, non_blocking=True)
    cond = dit.prepare_context(torch.as_tensor(ctx).to(dit.device, non_blocking=True), key_len)
    uncond = None
    if ctx_neg is not None and cfg != 1.0:
        uncond = dit.prepare_context(torch.as_tensor(ctx_neg).to(dit.device, non_blocking=True), key_len_neg)
    x = denoise_loop(dit, noise_d, cond, steps, cfg, uncond, shift)
    return x.cpu().numpy()
