"""Seeded synthetic DiT checkpoints in the reference's comfy_quant layout.

The real Anima weights are not available here, so tests and benchmarks build a checkpoint with the
2B MiniTrainDIT shapes (tools/reference.py:194-249): block linears N(0, 0.02) quantized with the
ConvRot quantizers (quant.py), everything else bf16 N(0, 0.02), norm weights 1 + N(0, 0.02).
The "mixed" precision follows the reference's asset builder: W4A8 for blocks 1..n-2, INT8 for the
first and last block (tools/build_assets.py:118-120).

Every tensor draws from its own generator seeded with (seed, crc32(name)), so any subset of a
checkpoint can be rebuilt independently and identically on any machine (CPU generator) or on the
same GPU model (CUDA generator).

AdaLN-LoRA rank and the t_embedder widths are not fixed by the reference's source (they come from
checkpoint shapes); these use rank 256 and 2048 -> 2048 -> 6144.
"""

from __future__ import annotations

import math
import zlib

import torch

from . import quant

D = 2048
HEADS = 16
HEAD_DIM = 128
MLP = 8192
CTX_DIM = 1024
ADALN_RANK = 256
N_BLOCKS = 28

QUANTIZED = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.output_proj",
             "cross_attn.q_proj", "cross_attn.k_proj", "cross_attn.v_proj", "cross_attn.output_proj",
             "mlp.layer1", "mlp.layer2")


def block_linear_shapes() -> dict:
    """[N, K] of every quantized linear of one block (module suffix -> shape)."""
    return {
        "self_attn.q_proj": (D, D), "self_attn.k_proj": (D, D), "self_attn.v_proj": (D, D),
        "self_attn.output_proj": (D, D),
        "cross_attn.q_proj": (D, D), "cross_attn.k_proj": (D, CTX_DIM), "cross_attn.v_proj": (D, CTX_DIM),
        "cross_attn.output_proj": (D, D),
        "mlp.layer1": (MLP, D), "mlp.layer2": (D, MLP),
    }


def _gen(seed: int, name: str, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFF)
    return g


def randn(seed: int, name: str, shape, device="cpu", std: float = 1.0) -> torch.Tensor:
    return torch.randn(shape, generator=_gen(seed, name, device), device=device, dtype=torch.float32) * std


def block_format(fmt: str, block: int, n_blocks: int) -> str:
    """'int8' or 'w4a8' for one block under fmt in {'int8', 'w4a8', 'mixed'}."""
    if fmt == "int8":
        return "int8"
    if fmt in ("w4a8", "mixed"):
        return "w4a8" if 0 < block < n_blocks - 1 else "int8"
    raise ValueError(f"unknown weight format {fmt}")


def quantized_linear(seed: int, name: str, shape, fmt: str, device="cpu", std: float = 0.02) -> dict:
    """comfy_quant tensors for one linear, keyed by suffix ('weight', 'weight_scale', ...)."""
    w = randn(seed, name, shape, device, std)
    q = quant.quantize_int8_convrot(w) if fmt == "int8" else quant.quantize_w4a8(w)
    return q


def direct_linear(seed: int, name: str, shape, fmt: str, device="cpu", std: float = 0.02) -> dict:
    """Quantized tensors drawn directly in the stored format, skipping the quantizer (cheap on a
    CPU for whole 28-block checkpoints): int8 codes ~ round(N(0, 40)), per-row scales near
    std/40; w4 codes uniform, fp8 group scales in [100, 130), FIXED_LUT codebook."""
    n, k = shape
    g = _gen(seed, name, device)
    if fmt == "int8":
        q = (torch.randn(shape, generator=g, device=device) * 40).round().clamp(-127, 127).to(torch.int8)
        s = (std / 40) * (1 + 0.1 * torch.rand((n, 1), generator=g, device=device))
        return {"weight": q, "weight_scale": s.float(),
                "comfy_quant": quant.comfy_meta("int8_tensorwise", convrot=True, convrot_groupsize=quant.CONVROT_GROUP)}
    codes = torch.randint(0, 16, (n, k), generator=g, device=device, dtype=torch.int32)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    s_rel = (100 + 30 * torch.rand((n, k // quant.W4_GROUP), generator=g, device=device)).to(torch.float8_e4m3fn)
    s_ch = (std * 2.5 / 127) * (1 + 0.1 * torch.rand((n,), generator=g, device=device))
    return {"weight": packed.contiguous(), "weight_s_rel": s_rel.contiguous(), "weight_s_channel": s_ch.float(),
            "weight_codebook": torch.tensor(quant.FIXED_LUT, dtype=torch.float32, device=device),
            "comfy_quant": quant.comfy_meta("asym_w4a8_int8", group_size=quant.W4_GROUP, convrot=True,
                                            convrot_groupsize=quant.CONVROT_GROUP)}


def block_tensors(seed: int, i: int, fmt: str = "int8", n_blocks: int = N_BLOCKS, device="cpu",
                  direct: bool = False) -> dict:
    """All tensors of block i, keyed by checkpoint name (without the model.diffusion_model. prefix).

    direct=True draws the quantized linears in their stored format (direct_linear) instead of
    quantizing Gaussian weights."""
    p = f"blocks.{i}."
    out = {}
    bfmt = block_format(fmt, i, n_blocks)
    make = direct_linear if direct else quantized_linear
    for mod, shape in block_linear_shapes().items():
        for suffix, t in make(seed, p + mod, shape, bfmt, device).items():
            out[p + mod + "." + suffix] = t
    for a in ("self_attn", "cross_attn"):
        for nrm in ("q_norm", "k_norm"):
            n = p + f"{a}.{nrm}.weight"
            out[n] = (1 + randn(seed, n, (HEAD_DIM,), device, 0.02)).to(torch.bfloat16)
    for m in ("adaln_modulation_self_attn", "adaln_modulation_cross_attn", "adaln_modulation_mlp"):
        n1, n2 = p + m + ".1.weight", p + m + ".2.weight"
        out[n1] = randn(seed, n1, (ADALN_RANK, D), device, 0.02).to(torch.bfloat16)
        out[n2] = randn(seed, n2, (3 * D, ADALN_RANK), device, 0.02).to(torch.bfloat16)
    return out


def global_tensors(seed: int, device="cpu") -> dict:
    """Non-block tensors: embedders, time conditioning, final layer."""
    out = {}

    def bf(name, shape, std=0.02):
        out[name] = randn(seed, name, shape, device, std).to(torch.bfloat16)

    bf("x_embedder.proj.1.weight", (D, 68))
    bf("t_embedder.1.linear_1.weight", (D, D))
    bf("t_embedder.1.linear_2.weight", (3 * D, D))
    out["t_embedding_norm.weight"] = (1 + randn(seed, "t_embedding_norm.weight", (D,), device, 0.02)).to(torch.bfloat16)
    bf("final_layer.adaln_modulation.1.weight", (ADALN_RANK, D))
    bf("final_layer.adaln_modulation.2.weight", (2 * D, ADALN_RANK))
    bf("final_layer.linear.weight", (64, D))
    return out


def dit_tensors(seed: int, fmt: str = "int8", n_blocks: int = N_BLOCKS, device="cpu", direct: bool = False) -> dict:
    """A full synthetic checkpoint (n_blocks blocks) as a flat name -> tensor dict."""
    out = global_tensors(seed, device)
    for i in range(n_blocks):
        out.update(block_tensors(seed, i, fmt, n_blocks, device, direct))
    return out


def lora_tensors(seed: int, targets, rank: int = 32, std: float = 0.01, n_blocks: int = N_BLOCKS,
                 alpha: float | None = None) -> dict:
    """PEFT-named LoRA (diffusion_model.<module>.lora_A/B.weight), fp32 N(0, std) A and B.

    targets: module suffixes inside each block, e.g. ("self_attn.q_proj", "mlp.layer1").
    """
    shapes = block_linear_shapes()
    out = {}
    for i in range(n_blocks):
        for t in targets:
            N, K = shapes[t]
            mod = f"diffusion_model.blocks.{i}.{t}"
            out[mod + ".lora_A.weight"] = randn(seed, mod + ".A", (rank, K), "cpu", std)
            out[mod + ".lora_B.weight"] = randn(seed, mod + ".B", (N, rank), "cpu", std)
            if alpha is not None:
                out[mod + ".alpha"] = torch.tensor(float(alpha))
    return out


# ----------------------------------------------------------------------------- text models
# Qwen3-0.6B (app/models/qwen3.js:7) and the LLM adapter (tools/reference.py:139-169). The
# published files keep Qwen3's attention and MLP linears quantized (int8 ConvRot or W4A8), its
# embedding table as per-row int8, and the adapter in bf16 (tools/build_assets.py:66-69, 130-157).
QWEN3 = {"layers": 28, "hidden": 1024, "heads": 16, "kv_heads": 8, "head_dim": 128, "mlp": 3072, "vocab": 151936,
         "theta": 1e6}
ADAPTER = {"blocks": 6, "hidden": 1024, "heads": 16, "head_dim": 64, "mlp": 4096, "vocab": 32128, "theta": 1e4}


def te_tensors(seed: int, n_layers: int = QWEN3["layers"], vocab: int = QWEN3["vocab"], fmt: str = "int8",
               device="cpu", direct: bool = False) -> dict:
    """A synthetic Qwen3 text-encoder file (names as the reference's te asset): linears N(0, 0.02)
    quantized with the ConvRot quantizers (direct=True: drawn in the stored format, see
    direct_linear), the embedding N(0, 1) as per-row int8, norm weights 1 + N(0, 0.02) in bf16.
    vocab may be cut down for tests (ids must stay below it)."""
    D, HD = QWEN3["hidden"], QWEN3["head_dim"]
    shapes = {"self_attn.q_proj": (QWEN3["heads"] * HD, D), "self_attn.k_proj": (QWEN3["kv_heads"] * HD, D),
              "self_attn.v_proj": (QWEN3["kv_heads"] * HD, D), "self_attn.o_proj": (D, QWEN3["heads"] * HD),
              "mlp.gate_proj": (QWEN3["mlp"], D), "mlp.up_proj": (QWEN3["mlp"], D), "mlp.down_proj": (D, QWEN3["mlp"])}
    out = {}
    for k, v in quant.quantize_int8_rows(randn(seed, "te.embed", (vocab, D), device)).items():
        out["model.embed_tokens." + k] = v
    for i in range(n_layers):
        p = f"model.layers.{i}."
        for mod, shape in shapes.items():
            make = direct_linear if direct else quantized_linear
            for k, v in make(seed, p + mod, shape, fmt if fmt == "int8" else "w4a8", device).items():
                out[p + mod + "." + k] = v
        for n, size in (("input_layernorm", D), ("post_attention_layernorm", D), ("self_attn.q_norm", HD),
                        ("self_attn.k_norm", HD)):
            name = p + n + ".weight"
            out[name] = (1 + randn(seed, name, (size,), device, 0.02)).to(torch.bfloat16)
    out["model.norm.weight"] = (1 + randn(seed, "model.norm.weight", (D,), device, 0.02)).to(torch.bfloat16)
    return out


def adapter_tensors(seed: int, n_blocks: int = ADAPTER["blocks"], vocab: int = ADAPTER["vocab"], device="cpu") -> dict:
    """A synthetic LLM adapter (the "llm_adapter." tensors of the DiT file), all bf16: linears
    N(0, 0.02), biases N(0, 0.02), the T5-vocabulary embedding N(0, 1), norms 1 + N(0, 0.02)."""
    D, HD, F = ADAPTER["hidden"], ADAPTER["head_dim"], ADAPTER["mlp"]
    out = {}

    def bf(name, shape, std=0.02, one=False):
        t = randn(seed, name, shape, device, std)
        out[name] = (t + 1 if one else t).to(torch.bfloat16)

    p0 = "llm_adapter."
    bf(p0 + "embed.weight", (vocab, D), 1.0)
    for i in range(n_blocks):
        p = f"{p0}blocks.{i}."
        for a in ("self_attn", "cross_attn"):
            for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                bf(f"{p}{a}.{n}.weight", (D, D))
            bf(f"{p}{a}.q_norm.weight", (HD,), one=True)
            bf(f"{p}{a}.k_norm.weight", (HD,), one=True)
        for n in ("norm_self_attn", "norm_cross_attn", "norm_mlp"):
            bf(f"{p}{n}.weight", (D,), one=True)
        bf(p + "mlp.0.weight", (F, D))
        bf(p + "mlp.0.bias", (F,))
        bf(p + "mlp.2.weight", (D, F))
        bf(p + "mlp.2.bias", (D,))
    bf(p0 + "out_proj.weight", (D, D))
    bf(p0 + "out_proj.bias", (D,))
    bf(p0 + "norm.weight", (D,), one=True)
    return out


# ----------------------------------------------------------------------------- VAE decoder
# The Wan-2.1 decoder as the reference's asset builder stores it (tools/build_assets.py:160-180):
# 3x3 convs OHWI [O, 3, 3, I], 1x1 convs [O, I], RMS_norm gammas 1-D, all bf16. Stage channels
# (384, 384, 384, 192, 96): three residual blocks per stage, a Resample (nearest 2x + conv to half
# the channels) after each of the first three stages, 15 "upsamples" entries in all.
VAE_DIMS = (384, 384, 384, 192, 96)
LATENT_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508, 0.4134, -0.0715, 0.5517, -0.3632,
               -0.1922, -0.9497, 0.2503, -0.2921]
LATENT_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743, 3.2687, 2.1526, 2.8652, 1.5579, 1.6382,
              1.1253, 2.8251, 1.916]


def vae_tensors(seed: int, dims=VAE_DIMS, z_dim: int = 16, device="cpu") -> dict:
    """A synthetic Wan-2.1 VAE decoder file: conv weights N(0, 1 / fan_in) so activations keep their
    scale through the stack, biases N(0, 0.02), gammas 1 + N(0, 0.02)."""
    out = {}

    def conv(name, o, i, k):
        shape = (o, k, k, i) if k == 3 else (o, i)
        out[name + ".weight"] = (randn(seed, name + ".weight", shape, device) / math.sqrt(i * k * k)).to(torch.bfloat16)
        out[name + ".bias"] = randn(seed, name + ".bias", (o,), device, 0.02).to(torch.bfloat16)

    def gamma(name, c):
        out[name + ".gamma"] = (1 + randn(seed, name + ".gamma", (c,), device, 0.02)).to(torch.bfloat16)

    def res(p, i, o):
        gamma(p + ".residual.0", i)
        conv(p + ".residual.2", o, i, 3)
        gamma(p + ".residual.3", o)
        conv(p + ".residual.6", o, o, 3)
        if i != o:
            conv(p + ".shortcut", o, i, 1)

    conv("conv2", z_dim, z_dim, 1)
    c = dims[0]
    conv("decoder.conv1", c, z_dim, 3)
    res("decoder.middle.0", c, c)
    gamma("decoder.middle.1.norm", c)
    conv("decoder.middle.1.to_qkv", 3 * c, c, 1)
    conv("decoder.middle.1.proj", c, c, 1)
    res("decoder.middle.2", c, c)
    idx, cin = 0, dims[0]
    for s, cout in enumerate(dims[1:]):
        for _ in range(3):
            res(f"decoder.upsamples.{idx}", cin, cout)
            cin = cout
            idx += 1
        if s < len(dims) - 2:
            conv(f"decoder.upsamples.{idx}.resample.1", cout // 2, cout, 3)
            cin = cout // 2
            idx += 1
    gamma("decoder.head.0", cin)
    conv("decoder.head.2", 3, cin, 3)
    return out
