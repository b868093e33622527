"""Shared helpers for the parity tests: seeded inputs and the stated tolerances."""
from __future__ import annotations

import numpy as np

# North-star tolerance versus the f32 oracle (stated once, used everywhere).
MAX_ABS = 2e-3
REL_L2 = 1e-3


def randn(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(int(np.prod(shape))).astype(np.float32) * np.float32(scale)
            ).reshape(shape)


def to_dev(x, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def to_np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close(orc, got, want, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    ma = orc.max_abs(got, want)
    rl = orc.rel_l2(got, want)
    assert ma <= max_abs and rl <= rel_l2, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"
    return ma, rl
