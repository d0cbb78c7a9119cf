"""Shared helpers for the test suite (not a test module)."""

import numpy as np
import torch


def to_np(d):
    """torch tensors -> numpy for the oracle: bf16 -> fp32, fp8 -> raw uint8 bytes."""
    import oracle

    return oracle.to_numpy(d)


def rel_l2(got, ref):
    """||got - ref|| / ||ref||, the reference's comparison metric (tools/check.js:24-37)."""
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
