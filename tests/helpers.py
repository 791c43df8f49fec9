"""Shared test helpers: seeded inputs, numpy<->torch bf16, the parity check."""

from __future__ import annotations

import numpy as np
import torch

import oracle as O

# Parity bar for float outputs: max|y - ref| / max|ref| <= TOL and, per
# element, |y - ref| <= TOL*|ref| + TOL*rms(ref).
TOL = 1e-2


def to_dev(a: np.ndarray, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == O.BF16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(O.BF16)
    return t.numpy()


def parity(y, ref, tol: float = TOL):
    y = np.asarray(y, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert np.all(np.isfinite(y)), "non-finite output"
    diff = np.abs(y - ref)
    scale = float(np.max(np.abs(ref)))
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    max_rel = float(np.max(diff)) / max(scale, 1e-30)
    bad = diff > tol * np.abs(ref) + tol * rms
    assert max_rel <= tol, f"max rel err {max_rel:.3e} > {tol}"
    assert not bad.any(), f"{int(bad.sum())} elements outside tolerance (worst {float(diff.max()):.3e})"
    return max_rel


def normal(rng, shape, std=1.0, dtype=np.float32):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(dtype)


def moe_weights(rng, D, I, E, std=0.02):
    """Router [D, E], gate/up [E, D, I], down [E, I, D] fp32 ~ N(0, std) (kappa layouts)."""
    router = normal(rng, (D, E), std)
    gate = normal(rng, (E, D, I), std)
    up = normal(rng, (E, D, I), std)
    down = normal(rng, (E, I, D), std)
    return router, gate, up, down
