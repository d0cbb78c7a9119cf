"""The reference's flow samplers (euler, euler_a, dpmpp_2m, er_sde) and schedulers (simple, beta)
on the device, against the CPU restatement of app/samplers.js (oracle/samplers_np.py): first with
an analytic elementwise denoiser (checks the update arithmetic and the noise stream exactly), then
with a 2-block DiT against the numpy oracle forward."""

import numpy as np
import pytest
import torch

import oracle
from oracle import samplers_np
from tests._util import rel_l2, to_np
from tests.conftest import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _noise_fn(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda n: torch.randn(n, generator=g).numpy()


@pytest.mark.parametrize("sampler", ["euler", "euler_a", "dpmpp_2m", "er_sde"])
@pytest.mark.parametrize("scheduler", ["simple", "beta"])
def test_sampler_arithmetic(sampler, scheduler):
    pl = pkg("pipeline")
    sig = pl.SCHEDULERS[scheduler](8, 3.0)
    x0 = torch.randn(1, 16, 32, 32, generator=torch.Generator().manual_seed(3))
    x = (x0 * np.float32(sig[0])).contiguous()

    def den_dev(xd, s, i):
        return (torch.tanh(xd) * (1 - s) + 0.05 * s).contiguous()

    def den_ref(xn, s, i):
        return (np.tanh(xn.astype(np.float64)) * (1 - s) + 0.05 * s).astype(np.float32)

    out = pl.sample(sampler, den_dev, x.to(DEV), sig, seed=11).cpu().numpy()
    ref = samplers_np.sample(sampler, den_ref, x.numpy(), sig, _noise_fn(11))
    assert rel_l2(out, ref) < 1e-5


@pytest.mark.parametrize("sampler,scheduler", [("er_sde", "beta"), ("dpmpp_2m", "simple"), ("euler_a", "beta")])
def test_sampler_with_dit_matches_oracle(sampler, scheduler):
    syn, ditm, pl = pkg("synthetic"), pkg("dit"), pkg("pipeline")
    seed = 41
    t = syn.dit_tensors(seed, "int8", 2)
    ctx = syn.randn(seed, "ctx", (64, 1024)).numpy()
    noise = syn.randn(seed, "noise", (1, 16, 16, 16)).numpy()
    sig = pl.SCHEDULERS[scheduler](4, 3.0)
    dit = ditm.AnimaDiT(t, DEV, n_blocks=2)
    cond = dit.prepare_context(torch.from_numpy(ctx).to(DEV))
    x = torch.from_numpy(noise * np.float32(sig[0])).to(DEV).contiguous()
    out = pl.sample(sampler, pl.dit_denoiser(dit, cond), x, sig, seed=5).cpu().numpy()

    W = oracle.DequantWeights(to_np(t))

    def den_ref(xn, s, i):
        v = oracle.dit_forward(W, xn[0], s, ctx, n_blocks=2)
        return (xn - v[None] * np.float32(s)).astype(np.float32)

    ref = samplers_np.sample(sampler, den_ref, (noise * np.float32(sig[0])).astype(np.float32), sig, _noise_fn(5))
    assert rel_l2(out, ref) < 3e-3
