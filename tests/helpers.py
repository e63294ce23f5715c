"""Shared helpers of the parity tests (tolerances and comparisons)."""

import os

import numpy as np
import torch

from oracle import orthocache_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

# Output tolerances (max abs): 1e-5 for float32 inputs, 2e-3 for float16 / bfloat16.
TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3}
# Scores within this relative distance of the threshold may flip either way.
NEAR_REL = 1e-5


def golden(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def as_np(t):
    if isinstance(t, np.ndarray):
        return t
    return t.detach().float().cpu().numpy()


def cast_np(a, dtype):
    """numpy float32 array rounded through a torch dtype (what the GPU sees)."""
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).float().numpy()


def assert_close(out, ref, dtype, what=""):
    err = float(np.max(np.abs(as_np(out).astype(np.float64) - np.asarray(ref, np.float64)))) if np.size(ref) else 0.0
    tol = TOL[dtype]
    assert err <= tol, f"{what}: max abs error {err:.3g} > {tol:g}"
    return err


def assert_mask(mask, keep_ref, score_ref, thr, what=""):
    """Bit-exact mask except tiles whose score is within NEAR_REL of thr (listed)."""
    m = as_np(mask).astype(bool)
    near = orc.near_threshold(score_ref, thr, NEAR_REL)
    bad = (m != keep_ref) & ~near
    assert not bad.any(), f"{what}: {int(bad.sum())} mask mismatches outside the near-threshold list"
    return np.argwhere(near)


def gpu_forced(mask, score_ref, thr):
    """(where, keep) for the oracle's ``forced`` argument: the GPU's decisions
    on the near-threshold tiles (where either decision is correct), so that
    outputs and counts can be compared exactly in every case."""
    return orc.near_threshold(score_ref, thr, NEAR_REL), as_np(mask).astype(bool)
