"""Generate the golden fixtures of tests/golden/ from the reference's own Python code.

Runs only where the reference checkout exists (it imports tools/quant.py and tools/reference.py
from REF: --ref, or the ANIMA_REFERENCE environment variable). Inputs come from the package's
seeded synthetic generator, so the tests can rebuild identical inputs without the reference. Usage:

    python tests/golden/make_golden.py --ref /path/to/anima-studio [--only small|full]

The full-size fixtures (--only full: 28 blocks at 1024^2, eleven reference forwards) take about
ten minutes on 8 CPU cores and ~20 GB of host memory.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def load_ref(ref):
    sys.path.insert(0, os.path.join(ref, "tools"))
    quant = importlib.import_module("quant")
    spec = importlib.util.spec_from_file_location("anima_reference", os.path.join(ref, "tools", "reference.py"))
    R = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(R)
    R.DEV = "cpu"
    return quant, R


def np_of(d):
    out = {}
    for k, v in d.items():
        if isinstance(v, torch.Tensor):
            if v.dtype == torch.float8_e4m3fn:
                v = v.view(torch.uint8)
            elif v.dtype == torch.bfloat16:
                v = v.float()
            v = v.cpu().numpy()
        out[k] = v
    return out


class RefWeights:
    """Duck-typed tools/reference.py Weights over an in-memory comfy_quant dict; block tensors are
    built on first access (one block at a time) to bound memory. cache=True keeps every block and
    its dequantized weights instead (many full-size forwards over the same checkpoint): the values
    are the same as dequantizing on every access, as the reference's Weights does."""

    def __init__(self, quant, make_block, globals_, cache=False):
        self.quant = quant
        self.make_block = make_block
        self.t = dict(globals_)
        self.block = None
        self.cache = cache
        self.built = set()
        self.deq = {}
        self.prefix = ""
        self.keys = _KeyView(self)

    def _ensure(self, name):
        if name.startswith("blocks."):
            i = int(name.split(".")[1])
            if self.cache:
                if i not in self.built:
                    self.t.update(self.make_block(i))
                    self.built.add(i)
            elif self.block != i:
                self.t = {k: v for k, v in self.t.items() if not k.startswith("blocks.")}
                self.t.update(self.make_block(i))
                self.block = i

    def __call__(self, name):
        if name in self.deq:
            return self.deq[name]
        self._ensure(name)
        base = name[: -len("weight")] if name.endswith("weight") else None
        if base is not None and base + "comfy_quant" in self.t:
            t = {s: self.t[base + s] for s in ("weight", "weight_scale", "weight_s_rel", "weight_s_channel", "weight_codebook", "comfy_quant") if base + s in self.t}
            w = self.quant.dequantize(t)
        else:
            w = self.t[name].float()
        if self.cache:
            self.deq[name] = w
        return w

    def has(self, name):
        self._ensure(name)
        return name in self.t


class _KeyView:
    """`name in W.keys` for the reference's LoraMerged (it copies base.keys)."""

    def __init__(self, w):
        self.w = w

    def __contains__(self, name):
        return self.w.has(name)


def full_size_fixtures(quant, R, syn):
    """BASELINE's headline configuration and its two neighbours at full size (1024^2: a 128x128
    latent, L = 4096 tokens), run through the reference's own dit_forward, Euler loop, CFG combine
    (tools/reference.py:194-249, 345-360) and LoraMerged (tools/reference.py:51-90). Each fixture
    keeps the velocity of the first pass, the final latent, and every 32nd token row of the residual
    stream after block 0 (128 of 4096 rows, to bound the file); the tests rebuild the noise from its
    seed with the reference's generator (torch_cpu_noise) and the weights from their seeds."""
    import tempfile

    from safetensors.torch import save_file

    rows = slice(0, 4096, 32)
    pad = torch.zeros(256, 1024)

    # (a) the headline: 28 INT8 ConvRot blocks, 8 Euler steps (sigmas_simple(8, 3)), no CFG
    seed = 41
    Wf = RefWeights(quant, lambda i: syn.block_tensors(seed, i, "int8", 28, direct=True), syn.global_tensors(seed),
                    cache=True)
    ctx = torch.cat([syn.randn(seed, "golden.ctx", (256, 1024)), pad])
    noise = R.torch_cpu_noise(seed, (1, 16, 1, 128, 128))[0, :, 0]
    sig = R.sigmas_simple(8, 3.0)
    xx = noise * sig[0]
    dump, v0 = {}, None
    for i in range(8):
        s = sig[i]
        v = R.dit_forward(Wf, xx, s, ctx, dump if i == 0 else None)
        if i == 0:
            v0 = v.clone()
        den = xx - v * s
        xx = den if sig[i + 1] == 0 else xx + (xx - den) / s * (sig[i + 1] - s)
        print(f"headline step {i + 1}/8", flush=True)
    np.savez_compressed(os.path.join(HERE, "forward_int8_1024.npz"), seed=seed, noise_sum=np.float64(noise.double().sum()),
                        velocity0=v0.numpy(), latent_final=xx.numpy(),
                        dit_block0_rows=dump["dit_block0"][rows].numpy(), rows_step=32)

    # (b) CFG: the base model's 30-step schedule, first step, cfg 4.5 with a negative context
    ctx_neg = torch.cat([syn.randn(seed, "golden.ctx_neg", (256, 1024)), pad])
    sig30 = R.sigmas_simple(30, 3.0)
    x0 = noise * sig30[0]
    v = R.dit_forward(Wf, x0, sig30[0], ctx)
    vn = R.dit_forward(Wf, x0, sig30[0], ctx_neg)
    vg = vn + (v - vn) * 4.5
    den = x0 - vg * sig30[0]
    x1 = x0 + (x0 - den) / sig30[0] * (sig30[1] - sig30[0])
    np.savez_compressed(os.path.join(HERE, "cfg_int8_1024.npz"), seed=seed, cfg=4.5, velocity_guided=vg.numpy(),
                        latent_step1=x1.numpy())
    print("cfg done", flush=True)
    del Wf

    # (c) W4A8 "mixed" (blocks 1..26 W4A8) + rank-32 LoRA on q/k/v and the MLP, one step
    seed = 43
    targets = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.layer1", "mlp.layer2")
    lt = syn.lora_tensors(seed, targets, rank=32, std=0.01, n_blocks=28, alpha=16.0)
    base = RefWeights(quant, lambda i: syn.block_tensors(seed, i, "mixed", 28, direct=True), syn.global_tensors(seed),
                      cache=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "lora.safetensors")
        save_file({k: v.contiguous() for k, v in lt.items()}, path)
        Wm = R.LoraMerged(base, [(path, 0.9)])
        ctx = torch.cat([syn.randn(seed, "golden.ctx", (256, 1024)), pad])
        noise = R.torch_cpu_noise(seed, (1, 16, 1, 128, 128))[0, :, 0]
        sig = R.sigmas_simple(8, 3.0)
        dump = {}
        v = R.dit_forward(Wm, noise * sig[0], sig[0], ctx, dump)
    np.savez_compressed(os.path.join(HERE, "forward_mixed_lora_1024.npz"), seed=seed, strength=0.9, alpha=16.0,
                        noise_sum=np.float64(noise.double().sum()), velocity0=v.numpy(),
                        dit_block0_rows=dump["dit_block0"][rows].numpy(), rows_step=32)
    print("mixed + LoRA done", flush=True)


def text_fixtures(quant, R, syn):
    """The text conditioning through the reference's own qwen3 and llm_adapter
    (tools/reference.py:116-169): a 28-layer INT8 ConvRot Qwen3 and the 6-block bf16 adapter with
    synthetic weights (vocabularies cut to 4096 rows: the ids stay below), 77 Qwen3 tokens and 60
    T5 tokens drawn from a seeded generator. Keeps the ids, the Qwen3 hidden states and the
    adapter's first 60 rows (the rest is zero padding to 512)."""
    seed, vocab = 51, 4096
    g = torch.Generator().manual_seed(seed)
    qids = torch.randint(0, vocab, (77,), generator=g).tolist()
    tids = torch.randint(0, vocab, (60,), generator=g).tolist()
    Wte = RefWeights(quant, lambda i: {}, syn.te_tensors(seed, 28, vocab, direct=True))
    hs = R.qwen3(Wte, qids)
    Wad = RefWeights(quant, lambda i: {}, syn.adapter_tensors(seed, 6, vocab))
    ctx = R.llm_adapter(Wad, hs, tids)
    assert ctx.shape == (512, 1024) and float(ctx[60:].abs().max()) == 0.0
    np.savez_compressed(os.path.join(HERE, "text_1024.npz"), seed=seed, vocab=vocab, qwen_ids=np.array(qids),
                        t5_ids=np.array(tids), hidden=hs.numpy(), ctx60=ctx[:60].numpy())
    print("text done", flush=True)


def vae_fixtures(quant, R, syn):
    """The reference's own vae_decode (tools/reference.py:254-295) on a synthetic Wan-2.1 decoder
    (the published channel layout), an 8x8 latent in the model's normalised space -> a 64x64
    image. vae_decode takes the de-normalised latent, as generate passes it (reference.py:368-370)."""
    seed = 61
    latent = syn.randn(seed, "golden.vae.latent", (16, 8, 8))
    Wv = RefWeights(quant, lambda i: {}, syn.vae_tensors(seed))
    mean = torch.tensor(R.LATENT_MEAN)[:, None, None]
    std = torch.tensor(R.LATENT_STD)[:, None, None]
    img = R.vae_decode(Wv, latent * std + mean)
    np.savez_compressed(os.path.join(HERE, "vae_64.npz"), seed=seed, latent=latent.numpy(), image=img.numpy())
    print("vae done", img.shape, flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ANIMA_REFERENCE"))
    ap.add_argument("--only", choices=["small", "full", "text", "vae"], default=None,
                    help="small: sections 1-5 (L = 64 and the quantizers); full: the 1024^2 fixtures; "
                         "text: the Qwen3 + LLM adapter fixture; vae: the VAE decoder fixture")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or ANIMA_REFERENCE")
    quant, R = load_ref(args.ref)
    sys.path.insert(0, ROOT)
    syn = importlib.import_module("anima-studio_b200.synthetic")
    torch.set_grad_enabled(False)
    if args.only == "full":
        full_size_fixtures(quant, R, syn)
        return
    if args.only == "text":
        text_fixtures(quant, R, syn)
        return
    if args.only == "vae":
        vae_fixtures(quant, R, syn)
        return

    # 1. int8 ConvRot quantizer + dequantizer (tools/quant.py:59-67, 81-83)
    w = syn.randn(1, "golden.int8", (64, 512), "cpu", 0.02)
    q = quant.quantize_int8_convrot(w)
    np.savez_compressed(os.path.join(HERE, "quant_int8.npz"), w=w.numpy(), weight=q["weight"].numpy(),
                        weight_scale=q["weight_scale"].numpy(), comfy_quant=q["comfy_quant"].numpy(),
                        deq=quant.dequantize(q).numpy())

    # 2. W4A8 quantizer (FIXED_LUT path and Lloyd-fit path) + decode (tools/quant.py:132-182)
    spikes = torch.zeros(64, 512)
    g = torch.Generator().manual_seed(7)
    idx = torch.randint(0, 512, (64, 24), generator=g)
    spikes.scatter_(1, idx, torch.randn(64, 24, generator=g))
    spikes += 0.01 * torch.randn(64, 512, generator=g)
    cases = {"w4_gauss": syn.randn(2, "golden.w4", (128, 1024), "cpu", 0.02),
             "w4_fit": quant.rotate(spikes) * 0.02}  # rotate() is an involution: the rotated weight is sparse
    for name, w in cases.items():
        q = quant.quantize_w4a8(w)
        ones = dict(q, weight_s_channel=torch.ones_like(q["weight_s_channel"]))
        grid = torch.round(quant.rotate(quant.dequantize_w4a8(ones)))  # undo the rotation: the int8 grid
        np.savez_compressed(os.path.join(HERE, f"quant_{name}.npz"), w=w.numpy(), grid=grid.numpy(),
                            deq=quant.dequantize(q).numpy(), **np_of(q))

    # 3. RoPE tables, time embedding path, sigma schedules (tools/reference.py:174-187, 300-303)
    ropes = {}
    for H, W in ((8, 8), (16, 12), (64, 64)):
        c, s = R.dit_rope(H, W)
        ropes[f"cos_{H}x{W}"], ropes[f"sin_{H}x{W}"] = c.numpy(), s.numpy()
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **ropes)
    sig = {f"simple_{n}": np.array(R.sigmas_simple(n, 3.0), dtype=np.float64) for n in (1, 2, 8, 30)}
    np.savez_compressed(os.path.join(HERE, "sigmas.npz"), **sig)

    # 4. one block at L=64 (8x8 patches) with quantized-Gaussian int8 weights: the body of the
    #    reference's block loop (tools/reference.py:232-242) run with its own helpers
    seed = 11
    Wb = RefWeights(quant, lambda i: syn.block_tensors(seed, i, "int8", 28), syn.global_tensors(seed))
    L = 64
    x = syn.randn(seed, "golden.x", (L, 2048))
    ctx256 = syn.randn(seed, "golden.ctx", (256, 1024))
    ctx = torch.nn.functional.pad(ctx256, (0, 0, 0, 256))  # zero-padded to 512 rows as the reference does
    sigma = 0.9
    half = 1024
    freqs = torch.exp(-np.log(10000) * torch.arange(half).float() / half)
    temb = sigma * freqs
    temb = torch.cat([temb.cos(), temb.sin()])[None]
    adaln_lora = torch.nn.functional.silu(temb @ Wb("t_embedder.1.linear_1.weight").T) @ Wb("t_embedder.1.linear_2.weight").T
    emb = R.rms_norm(temb, Wb("t_embedding_norm.weight"))
    cos, sin = R.dit_rope(8, 8)
    cos, sin = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)

    def mod(p):
        m = torch.nn.functional.silu(emb) @ Wb(p + ".1.weight").T @ Wb(p + ".2.weight").T + adaln_lora
        return m.chunk(3, -1)

    def attn(p, xq, c, rope):
        Lq, Lk = xq.shape[0], c.shape[0]
        qq = R.rms_norm((xq @ Wb(p + "q_proj.weight").T).view(Lq, 16, 128), Wb(p + "q_norm.weight")).transpose(0, 1)
        kk = R.rms_norm((c @ Wb(p + "k_proj.weight").T).view(Lk, 16, 128), Wb(p + "k_norm.weight")).transpose(0, 1)
        vv = (c @ Wb(p + "v_proj.weight").T).view(Lk, 16, 128).transpose(0, 1)
        if rope:
            qq = qq * cos + R.rotate_half(qq) * sin
            kk = kk * cos + R.rotate_half(kk) * sin
        return R.attention(qq, kk, vv).transpose(0, 1).reshape(Lq, 2048) @ Wb(p + "output_proj.weight").T

    p = "blocks.0."
    xb = x.clone()
    sh, sc, gt = mod(p + "adaln_modulation_self_attn")
    n = R.layer_norm(xb) * (1 + sc) + sh
    xb = xb + gt * attn(p + "self_attn.", n, n, True)
    x_self = xb.clone()
    sh, sc, gt = mod(p + "adaln_modulation_cross_attn")
    n = R.layer_norm(xb) * (1 + sc) + sh
    xb = xb + gt * attn(p + "cross_attn.", n, ctx, False)
    x_cross = xb.clone()
    sh, sc, gt = mod(p + "adaln_modulation_mlp")
    n = R.layer_norm(xb) * (1 + sc) + sh
    xb = xb + gt * (torch.nn.functional.gelu(n @ Wb(p + "mlp.layer1.weight").T) @ Wb(p + "mlp.layer2.weight").T)
    np.savez_compressed(os.path.join(HERE, "block0_L64.npz"), seed=seed, sigma=sigma, x=x.numpy(), ctx256=ctx256.numpy(),
                        temb=temb.numpy(), adaln_lora=adaln_lora.numpy(), emb=emb.numpy(),
                        x_self=x_self.numpy(), x_cross=x_cross.numpy(), out=xb.numpy())

    # 5. the full 28-block reference forward + 2-step Euler at a 16x16 latent (L = 64), with
    #    directly drawn int8 weights (and W4A8 "mixed"), through tools/reference.py's own
    #    dit_forward and its Euler loop (tools/reference.py:194-249, 345-360)
    for fmt in ("int8", "mixed"):
        seed = 21
        Wf = RefWeights(quant, lambda i, fmt=fmt: syn.block_tensors(seed, i, fmt, 28, direct=True), syn.global_tensors(seed))
        noise = R.torch_cpu_noise(seed, (1, 16, 1, 16, 16))[0, :, 0]
        ctx = torch.nn.functional.pad(syn.randn(seed, "golden.ctx", (256, 1024)), (0, 0, 0, 256))
        sig = R.sigmas_simple(2, 3.0)
        xx = noise * sig[0]
        dump = {}
        v0 = None
        for i in range(2):
            s = sig[i]
            v = R.dit_forward(Wf, xx, s, ctx, dump if i == 0 else None)
            if i == 0:
                v0 = v.clone()
            den = xx - v * s
            if i == 0:
                dump["denoised0"] = den
            xx = den if sig[i + 1] == 0 else xx + (xx - den) / s * (sig[i + 1] - s)
        np.savez_compressed(os.path.join(HERE, f"forward_{fmt}_16x16.npz"), seed=seed, noise=noise.numpy(),
                            velocity0=v0.numpy(), latent_final=xx.numpy(), **{k: t.numpy() for k, t in dump.items()})
        print("forward", fmt, "done", flush=True)
    if args.only is None:
        full_size_fixtures(quant, R, syn)
        text_fixtures(quant, R, syn)
        vae_fixtures(quant, R, syn)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
