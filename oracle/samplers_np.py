"""CPU restatement of the reference's flow-matching samplers and the beta scheduler
(app/samplers.js:24-218), test infrastructure only: the checker for pipeline.sample and
pipeline.sigmas_beta.

Latents are fp32 arrays; every update is computed in float64 and stored in fp32, as the
reference computes in JavaScript numbers and stores into Float32Arrays. `denoise(x, sigma, i)`
returns the x0 prediction, and `noise(n)` draws the sampler's Gaussian noise (the reference seeds
its own generator with the run's seed, samplers.js:104-106).

Parity: unpinned against the JavaScript itself (no JS runtime here); the restatement follows the
file line by line.
"""

from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def _time_shift(shift, t):
    return shift * t / (1 + (shift - 1) * t)


def sigma_table(shift):
    """samplers.js:8-13: 1000 fp32-rounded sigmas."""
    return [float(f32(_time_shift(shift, i / 1000))) for i in range(1, 1001)]


def _ln_gamma(z):
    """Lanczos approximation, g = 7 (samplers.js:26-36)."""
    c = [0.99999999999980993, 676.5203681218851, -1259.1392167224028, 771.32342877765313,
         -176.61502916214059, 12.507343278686905, -0.13857109526572012, 9.9843695780195716e-6,
         1.5056327351493116e-7]
    if z < 0.5:
        return math.log(math.pi / math.sin(math.pi * z)) - _ln_gamma(1 - z)
    z -= 1
    x = c[0]
    for i in range(1, 9):
        x += c[i] / (z + i)
    t = z + 7.5
    return 0.5 * math.log(2 * math.pi) + (z + 0.5) * math.log(t) - t + math.log(x)


def _betacf(a, b, x):
    """Continued fraction of the incomplete beta function (samplers.js:38-60)."""
    FPMIN = 1e-300
    c, d = 1.0, 1 - (a + b) * x / (a + 1)
    if abs(d) < FPMIN:
        d = FPMIN
    d = 1 / d
    h = d
    for m in range(1, 301):
        m2 = 2 * m
        aa = m * (b - m) * x / ((a - 1 + m2) * (a + m2))
        d = 1 + aa * d
        d = FPMIN if abs(d) < FPMIN else d
        c = 1 + aa / c
        c = FPMIN if abs(c) < FPMIN else c
        d = 1 / d
        h *= d * c
        aa = -(a + m) * (a + b + m) * x / ((a + m2) * (a + 1 + m2))
        d = 1 + aa * d
        d = FPMIN if abs(d) < FPMIN else d
        c = 1 + aa / c
        c = FPMIN if abs(c) < FPMIN else c
        d = 1 / d
        de = d * c
        h *= de
        if abs(de - 1) < 1e-15:
            break
    return h


def _beta_cdf(x, a, b):
    """samplers.js:62-68."""
    if x <= 0:
        return 0.0
    if x >= 1:
        return 1.0
    lbt = _ln_gamma(a + b) - _ln_gamma(a) - _ln_gamma(b) + a * math.log(x) + b * math.log(1 - x)
    if x < (a + 1) / (a + b + 2):
        return math.exp(lbt) * _betacf(a, b, x) / a
    return 1 - math.exp(lbt) * _betacf(b, a, 1 - x) / b


def _beta_ppf(p, a, b):
    """Bisection, 100 halvings (samplers.js:70-79)."""
    if p <= 0:
        return 0.0
    if p >= 1:
        return 1.0
    lo, hi = 0.0, 1.0
    for _ in range(100):
        mid = (lo + hi) / 2
        if _beta_cdf(mid, a, b) < p:
            lo = mid
        else:
            hi = mid
    return (lo + hi) / 2


def sigmas_beta(steps, shift, alpha=0.6, beta=0.6):
    """ComfyUI "beta" scheduler with repeated timesteps dropped (samplers.js:83-93)."""
    table = sigma_table(shift)
    out, last = [], -1
    for i in range(steps):
        t = math.floor(_beta_ppf(1 - i / steps, alpha, beta) * 999 + 0.5)  # Math.round
        if t != last:
            out.append(table[t])
        last = t
    return out + [0.0]


def _axpby(a, x, b, y):
    return (a * x.astype(np.float64) + b * y.astype(np.float64)).astype(f32)


def sample(name, denoise, x, sigmas, noise, shift=3.0):
    """samplers.js:104-218 (euler, euler_a = sample_euler_ancestral_RF with eta 1, dpmpp_2m,
    er_sde = VP ER-SDE-Solver-3 for flow models). Returns the final latent."""
    x = np.asarray(x, dtype=f32)
    n = len(sigmas) - 1
    if name == "euler":
        for i in range(n):
            s, s1 = sigmas[i], sigmas[i + 1]
            den = denoise(x, s, i)
            x = den if s1 == 0 else _axpby(s1 / s, x, 1 - s1 / s, den)
        return x
    if name == "euler_a":
        for i in range(n):
            s, s1 = sigmas[i], sigmas[i + 1]
            den = denoise(x, s, i)
            if s1 == 0:
                x = den
                continue
            sigma_down = s1 * (s1 / s)
            alpha_ip1 = 1 - s1
            alpha_down = 1 - sigma_down
            renoise = math.sqrt(s1 * s1 - sigma_down * sigma_down * alpha_ip1 * alpha_ip1 / (alpha_down * alpha_down))
            r = sigma_down / s
            x = _axpby(r, x, 1 - r, den)
            eps = noise(x.size).reshape(x.shape)
            k = alpha_ip1 / alpha_down
            x = (k * x.astype(np.float64) + eps.astype(np.float64) * renoise).astype(f32)
        return x
    if name == "dpmpp_2m":
        t = lambda v: -math.log(v)  # noqa: E731
        old = None
        for i in range(n):
            s, s1 = sigmas[i], sigmas[i + 1]
            den = denoise(x, s, i)
            if s1 == 0:
                x = den
            else:
                h = t(s1) - t(s)
                ratio = s1 / s
                c = -math.expm1(-h)
                if old is None:
                    x = _axpby(ratio, x, c, den)
                else:
                    h_last = t(s) - t(sigmas[i - 1])
                    r = h_last / h
                    dd = _axpby(1 + 1 / (2 * r), den, -1 / (2 * r), old)
                    x = _axpby(ratio, x, c, dd)
            old = den
        return x
    if name == "er_sde":
        sg = list(sigmas)
        if sg[0] >= 1:
            sg[0] = float(f32(_time_shift(shift, 1 - 1e-4)))
        lam = [0.0 if v == 0 else v / (1 - v) for v in sg]
        scaler = lambda v: v * (math.exp(v ** 0.3) + 10)  # noqa: E731
        P = 200
        old = old_d = None
        for i in range(n):
            den = denoise(x, sg[i], i)
            stage = min(3, i + 1)
            if sg[i + 1] == 0:
                x = den
            else:
                ls, lt = lam[i], lam[i + 1]
                alpha_s, alpha_t = sg[i] / ls, sg[i + 1] / lt
                r = scaler(lt) / scaler(ls)
                x = _axpby(alpha_t / alpha_s * r, x, alpha_t * (1 - r), den)
                if stage >= 2:
                    dt = lt - ls
                    step = -dt / P
                    s_ = su = 0.0
                    for p in range(P):
                        pos = lt + p * step
                        sp = scaler(pos)
                        s_ += 1 / sp
                        su += (pos - ls) / sp
                    s_ *= step
                    su *= step
                    d_d = _axpby(1 / (ls - lam[i - 1]), den, -1 / (ls - lam[i - 1]), old)
                    c2 = alpha_t * (dt + s_ * scaler(lt))
                    x = (x.astype(np.float64) + c2 * d_d.astype(np.float64)).astype(f32)
                    if stage >= 3:
                        d_u = _axpby(2 / (ls - lam[i - 2]), d_d, -2 / (ls - lam[i - 2]), old_d)
                        c3 = alpha_t * (dt * dt / 2 + su * scaler(lt))
                        x = (x.astype(np.float64) + c3 * d_u.astype(np.float64)).astype(f32)
                    old_d = d_d
                nz = math.sqrt(max(0.0, lt * lt - ls * ls * r * r))
                if nz > 0:
                    eps = noise(x.size).reshape(x.shape)
                    x = (x.astype(np.float64) + alpha_t * eps.astype(np.float64) * nz).astype(f32)
            old = den
        return x
    raise ValueError(f"unknown sampler {name}")
