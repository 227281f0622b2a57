"""Loader of the recorded reference test calls (tests/golden/refcall_*.npz,
written by tests/golden/record_reference_calls.py from the reference's
unchanged component test files)."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def files():
    return sorted(GOLDEN.glob("refcall_*.npz"))


def load(path):
    """-> (test id, function name, args tuple, expected result, rtol, atol)."""
    with np.load(path) as z:
        args = []
        for i in range(int(z["n_args"])):
            a, kind = z[f"arg{i}"], str(z[f"kind{i}"])
            args.append(a if kind == "array" else bool(a) if kind == "bool" else int(a) if kind == "int"
                        else float(a))
        return str(z["test"]), str(z["fn"]), tuple(args), z["result"], float(z["rtol"]), float(z["atol"])
