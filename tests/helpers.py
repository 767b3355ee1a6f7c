"""Shared seeded input generators for the parity tests."""
import numpy as np
import torch


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def rand_i8(g, shape, lo=-128, hi=127):
    return g.integers(lo, hi + 1, size=shape, dtype=np.int64).astype(np.int8)


def rand_i4(g, shape):
    return g.integers(-8, 8, size=shape, dtype=np.int64).astype(np.int8)


def to_dev(a, device, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device)


def assert_equal(got: torch.Tensor, want: np.ndarray, what: str = ""):
    g = got.detach().cpu().numpy()
    assert g.shape == want.shape, (what, g.shape, want.shape)
    if not np.array_equal(g, want):
        bad = np.argwhere(g != want)
        idx = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatches, first at {idx}: got {g[idx]} want {want[idx]}")


def assert_close(got: torch.Tensor, want: np.ndarray, rel=1e-3, what: str = ""):
    """Float parity: |got - want| <= rel * max(|want|, 1e-3 * max|want|)."""
    g = got.detach().float().cpu().numpy()
    w = want.astype(np.float32)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    floor = 1e-3 * max(float(np.abs(w).max()), 1e-30)
    tol = rel * np.maximum(np.abs(w), floor)
    err = np.abs(g - w)
    if not np.all(err <= tol):
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(f"{what}: max violation at {i}: got {g[i]} want {w[i]} tol {tol[i]}")
