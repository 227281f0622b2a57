"""The recorded reference test calls (tests/golden/refcall_*.npz) cover the
reference's four component test files, and the CPU restatement in
``oracle/`` reproduces every recorded result within the tolerance the
reference's test body applies."""

import numpy as np

from oracle import moe_oracle as O
from tests import refcalls

ORACLE = {
    "mul_mat_id": O.mul_mat_id_literal,
    "moe_ffn_block": O.moe_ffn_block_literal,
    "swiglu": O.swiglu,
    "rms_norm_linalg": O.rms_norm,
}


def test_recorded_calls_cover_the_reference_tests():
    tests = {refcalls.load(p)[0] for p in refcalls.files()}
    per_file = {}
    for t in tests:
        per_file.setdefault(t.split("::")[0].rsplit("/", 1)[-1], set()).add(t)
    # test_mul_mat_id.py:15-85 (4), test_moe_ffn_block.py:20-196 (4),
    # test_swiglu.py:15-59 (4), test_rms_norm.py (8)
    assert {k: len(v) for k, v in per_file.items()} == {
        "test_mul_mat_id.py": 4, "test_moe_ffn_block.py": 4, "test_swiglu.py": 4, "test_rms_norm.py": 8}


def test_oracle_reproduces_recorded_calls():
    for p in refcalls.files():
        test, fn, args, expected, rtol, atol = refcalls.load(p)
        got = ORACLE[fn](*args)
        np.testing.assert_allclose(got, expected, rtol=rtol, atol=atol, err_msg=test)
