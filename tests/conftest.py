"""Shared test setup: the `gpu` marker, import paths and golden fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def split(flat: np.ndarray, lens: np.ndarray) -> list[np.ndarray]:
    out, o = [], 0
    for n in lens:
        out.append(flat[o:o + int(n)])
        o += int(n)
    return out


def cases(name: str) -> list[dict]:
    """Unflatten a fixture written as {key}_{i} entries plus `count`."""
    z = load_npz(name)
    n = int(z["count"])
    out = [dict() for _ in range(n)]
    for k, v in z.items():
        if k == "count":
            continue
        key, _, idx = k.rpartition("_")
        out[int(idx)][key] = v
    return out


def bits(a) -> np.ndarray:
    return np.asarray(a, np.float32).view(np.uint32)


def same_bits(a, b) -> np.ndarray:
    """Bitwise float equality, any NaN equal to any NaN (the reference's st_same)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return (bits(a) == bits(b)) | (np.isnan(a) & np.isnan(b))


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    oracle.set_expf_mode(0)
    return oracle


def fma32(a, b, c) -> np.float32:
    """Correctly rounded float32 fma(a, b, c) (C's fmaf), computed exactly."""
    from fractions import Fraction
    a, b, c = (np.float32(v) for v in (a, b, c))
    if not (np.isfinite(a) and np.isfinite(b) and np.isfinite(c)):
        return np.float32(np.float64(a) * np.float64(b) + np.float64(c))
    r = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    f = np.float32(float(r))
    best = None
    for cand in (np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))):
        if not np.isfinite(cand):
            continue
        d = abs(Fraction(float(cand)) - r)
        if best is None or d < best[0] or (d == best[0] and int(cand.view(np.uint32)) % 2 == 0):
            best = (d, cand)
    out = best[1]
    if out == 0 and r == 0:
        # exact zero: sign follows IEEE (x + -x = +0 in round-to-nearest)
        out = np.float32(np.float64(a) * np.float64(b) + np.float64(c))
    return np.float32(out)
