"""Test helpers: move raw int16 Q8.8 arrays between host and device."""
import numpy as np


def dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int16)).cuda()


def host(t) -> np.ndarray:
    return t.cpu().numpy()


def empty(n: int, fill: int = -23131):
    """Device buffer poisoned with 0xA5A5 so unwritten words show up."""
    import torch
    return torch.full((max(int(n), 1),), fill, dtype=torch.int16, device="cuda")


def rand16(rng, n, lo=-32768, hi=32768):
    return rng.integers(lo, hi, size=int(n), dtype=np.int64).astype(np.int16)


def assert_same(got: np.ndarray, want: np.ndarray, what: str = ""):
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    bad = np.flatnonzero(got != want)
    if bad.size:
        i = bad[:8]
        raise AssertionError(f"{what}: {bad.size} of {got.size} words differ; first {i.tolist()} "
                             f"got {got[i].tolist()} want {want[i].tolist()}")
