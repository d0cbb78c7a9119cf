"""The Wan-2.1 VAE decoder on a B200: its operators (NHWC 3x3 convolution with the fused 2x
upsample and residual, channel RMS norm + SiLU, single-head attention at d = 384) against the numpy
oracle, and the whole decoder against the reference's own vae_decode (tests/golden/vae_64.npz).

Tolerances (relative L2): the fp32 operators 1e-5 (bf16 weights read exactly, fp32 sums in another
order); the decoded image 1e-4."""

import os

import numpy as np
import pytest
import torch

import oracle
from oracle import text_np, vae_np
from tests._util import rel_l2
from tests.conftest import GOLDEN, pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _conv_weights(o, i, seed, k=3):
    g = torch.Generator().manual_seed(seed)
    shape = (o, 3, 3, i) if k == 3 else (o, i)
    return {"c.weight": (torch.randn(shape, generator=g) / (3 * i ** 0.5)).to(torch.bfloat16),
            "c.bias": (0.1 * torch.randn(o, generator=g)).to(torch.bfloat16)}


@pytest.mark.parametrize("h,w,cin,cout,up,acc", [(8, 8, 16, 384, False, False), (13, 7, 96, 3, False, True),
                                                 (6, 5, 384, 192, True, False), (32, 32, 192, 96, False, True)])
def test_conv3x3_matches_oracle(h, w, cin, cout, up, acc):
    ops, W = pkg("ops"), pkg("weights")
    t = _conv_weights(cout, cin, h * 31 + cin)
    lin = W.linear_weights(t, "c.", DEV)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(h * w, cin, generator=g)
    H, Wd = (2 * h, 2 * w) if up else (h, w)
    base = torch.randn(H * Wd, cout, generator=g)
    out = ops.conv3x3(x.to(DEV), lin, h, w, up=up, into=base.clone().to(DEV) if acc else None).cpu().numpy()
    xc = x.numpy().T.reshape(cin, h, w)
    if up:
        xc = xc.repeat(2, 1).repeat(2, 2)
    ref = vae_np.conv(oracle.DequantWeights(oracle.to_numpy(t)), xc, "c").reshape(cout, H * Wd).T
    if acc:
        ref = ref + base.numpy()
    assert rel_l2(out, ref) < 1e-5


@pytest.mark.parametrize("C,silu", [(384, True), (96, False)])
def test_channel_norm_matches_oracle(C, silu):
    ops = pkg("ops")
    g = torch.Generator().manual_seed(C)
    x = torch.randn(300, C, generator=g) * 3
    gamma = 1 + 0.1 * torch.randn(C, generator=g)
    y = ops.channel_norm(x.to(DEV), gamma.to(DEV), C, silu).cpu().numpy()
    W = oracle.DequantWeights({"n.gamma": gamma.numpy()})
    ref = vae_np.norm(W, x.numpy().T.reshape(C, 300, 1), "n").reshape(C, 300).T
    if silu:
        ref = oracle.silu(ref)
    assert rel_l2(y, ref) < 1e-5


def test_single_head_attention_d384():
    ops = pkg("ops")
    L, D = 200, 384
    g = torch.Generator().manual_seed(9)
    qkv = torch.randn(L, 3 * D, generator=g)
    out = ops.attention(qkv.to(DEV), qkv.to(DEV), qkv.to(DEV), Lq=L, Lk=L, H=1, D=D, ldq=3 * D, ldk=3 * D, ldv=3 * D,
                        q_off=0, k_off=D, v_off=2 * D, out_dtype=torch.float32).cpu().numpy()
    q, k, v = (qkv[:, i * D:(i + 1) * D].numpy()[None] for i in range(3))
    assert rel_l2(out, text_np.attention(q, k, v)[0]) < 1e-5


# At least 2^20 scores the single head runs on the tensor cores: S = Q K^T and O = P V as
# two-plane bf16 GEMMs (about 16 significant bits per operand, fp32 sums) around a row softmax.
@pytest.mark.parametrize("Lq,Lk", [(2048, 2048), (1024, 1536)])
def test_single_head_attention_d384_tensor_cores(Lq, Lk):
    ops = pkg("ops")
    D = 384
    g = torch.Generator().manual_seed(Lq + Lk)
    q = torch.randn(Lq, 3 * D, generator=g) * 1.5
    kv = torch.randn(Lk, 3 * D, generator=g)
    out = ops.attention(q.to(DEV), kv.to(DEV), kv.to(DEV), Lq=Lq, Lk=Lk, H=1, D=D, ldq=3 * D, ldk=3 * D, ldv=3 * D,
                        q_off=0, k_off=D, v_off=2 * D, out_dtype=torch.float32).cpu().numpy()
    qn = q[:, :D].numpy()[None]
    kn, vn = kv[:, D:2 * D].numpy()[None], kv[:, 2 * D:].numpy()[None]
    assert rel_l2(out, text_np.attention(qn, kn, vn)[0]) < 3e-5


def test_vae_decoder_matches_reference():
    syn, vae = pkg("synthetic"), pkg("vae")
    g = dict(np.load(os.path.join(GOLDEN, "vae_64.npz")))
    dec = vae.VAEDecoder(syn.vae_tensors(int(g["seed"])), DEV)
    img = dec.decode(torch.from_numpy(g["latent"])).cpu().numpy()
    err = rel_l2(img, g["image"])
    print(f"VAE decoder, 8x8 latent -> 64x64: rel L2 {err:.2e}")
    assert img.shape == (3, 64, 64) and err < 1e-4
