"""mul_mat_id through the reference-shaped module vs the reference's outputs.

Cases and tolerance follow tests/components/test_mul_mat_id.py:15-85 of the
reference (rtol 1e-4, atol 1e-5); expected values are the reference oracle's
own outputs stored in tests/golden/.
"""

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.utils import assert_close, golden_names, load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("mmid_"))
def test_golden_case(mul_mat_id_module, name):
    g = load_golden(name)
    out = mul_mat_id_module.mul_mat_id(g["weights"], g["input"], g["ids"])
    assert out.shape == g["expected"].shape and out.dtype == np.float32
    assert_close(out, g["expected"], rtol=1e-4, atol=1e-5)


def test_single_expert_per_token(mul_mat_id_module):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((4, 3, 8)) * 0.1).astype(np.float32)
    x = (rng.standard_normal((3, 1, 2)) * 0.1).astype(np.float32)
    ids = np.array([[0, 3]], dtype=np.int32)
    assert_close(mul_mat_id_module.mul_mat_id(w, x, ids), O.mul_mat_id_literal(w, x, ids), rtol=1e-4, atol=1e-5)


def test_all_tokens_one_expert_many_tiles(mul_mat_id_module):
    rng = np.random.default_rng(12)
    w = (rng.standard_normal((70, 50, 4)) * 0.1).astype(np.float32)
    x = (rng.standard_normal((50, 1, 300)) * 0.1).astype(np.float32)
    ids = np.full((1, 300), 3, dtype=np.int32)
    assert_close(mul_mat_id_module.mul_mat_id(w, x, ids), O.mul_mat_id_grouped(w, x, ids), rtol=1e-4, atol=1e-5)


def test_out_of_range_ids_raise(mul_mat_id_module):
    from frank_b200._lib import FrankError

    w = np.ones((4, 3, 2), np.float32)
    x = np.ones((3, 1, 2), np.float32)
    with pytest.raises(FrankError):
        mul_mat_id_module.mul_mat_id(w, x, np.array([[0, 2]], dtype=np.int32))
    with pytest.raises(FrankError):
        mul_mat_id_module.mul_mat_id(w, x, np.array([[-1, 0]], dtype=np.int32))


def test_rejects_float64(mul_mat_id_module):
    w = np.ones((4, 3, 2))
    with pytest.raises(ValueError):
        mul_mat_id_module.mul_mat_id(w, np.ones((3, 1, 2), np.float32), np.zeros((1, 2), np.int32))


def test_zero_tokens(mul_mat_id_module):
    w = np.ones((4, 3, 2), np.float32)
    out = mul_mat_id_module.mul_mat_id(w, np.ones((3, 2, 0), np.float32), np.zeros((2, 0), np.int32))
    assert out.shape == (4, 2, 0)
