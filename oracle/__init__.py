"""CPU oracle for the Anima DiT denoising path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the math of the reference's PyTorch implementation
(tools/reference.py) and of its weight-format decoders (tools/quant.py). It exists to check the
CUDA path and is never part of it: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import it.

Parity pin: tests/golden/ holds fixtures produced by running the reference's own
tools/reference.py and tools/quant.py on seeded inputs (script: tests/golden/make_golden.py);
tests/test_oracle.py checks this restatement against every one of them.
"""

from .ref_np import *  # noqa: F401,F403


def to_numpy(d: dict) -> dict:
    """torch tensors of a checkpoint dict -> numpy for the oracle (bf16 -> fp32, fp8 -> raw bytes)."""
    import torch

    out = {}
    for k, v in d.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu()
            if v.dtype == torch.float8_e4m3fn:
                v = v.view(torch.uint8)
            elif v.dtype == torch.bfloat16:
                v = v.float()
            v = v.numpy()
        out[k] = v
    return out
