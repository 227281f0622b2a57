"""Shared test helpers (tolerances follow the reference harness)."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def assert_close(actual, expected, rtol=1e-5, atol=1e-6):
    """Same contract as the reference's tests/utils.py:244-251."""
    np.testing.assert_allclose(np.asarray(actual), np.asarray(expected), rtol=rtol, atol=atol)


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))


def rms_rel_maxabs(actual, expected) -> float:
    """max |a - e| / rms(e): the bf16-path tolerance metric (<= 2e-2)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    rms = float(np.sqrt(np.mean(e * e)))
    return float(np.max(np.abs(a - e))) / max(rms, 1e-30)
