"""moe_ffn_block through the reference-shaped module (fp32 path) vs the
reference's outputs.  Cases follow tests/components/test_moe_ffn_block.py:
20-196 of the reference (rtol 1e-4, atol 1e-5) plus the fp32 headline
configuration and fine-grained / decode shapes; expected values come from
the reference oracle (tests/golden/)."""

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.utils import assert_close, golden_names, load_golden

pytestmark = pytest.mark.gpu


def _args(g):
    return (g["input"], g["gate_inp_w"], g["up_exps_w"], g["gate_exps_w"], g["down_exps_w"], int(g["n_expert"]),
            int(g["n_expert_used"]), int(g["n_embd"]), int(g["n_ff"]), bool(g["normalize_weights"]))


@pytest.mark.parametrize("name", golden_names("moe_"))
def test_golden_case(moe_ffn_module, name):
    g = load_golden(name)
    y = moe_ffn_module.moe_ffn_block(*_args(g))
    assert y.shape == g["expected"].shape and y.dtype == np.float32
    assert_close(y, g["expected"], rtol=1e-4, atol=1e-5)


def test_c1_meets_fp32_rms_tolerance(moe_ffn_module):
    """fp32 headline configuration: max-abs <= 1e-5 x output RMS."""
    g = load_golden("moe_c1_fp32")
    y = moe_ffn_module.moe_ffn_block(*_args(g))
    e = g["expected"]
    assert np.max(np.abs(y - e)) <= 1e-5 * np.sqrt(np.mean(e * e))


def test_deterministic(moe_ffn_module):
    g = load_golden("moe_mixtral_like")
    a = moe_ffn_module.moe_ffn_block(*_args(g))
    b = moe_ffn_module.moe_ffn_block(*_args(g))
    assert np.array_equal(a, b)


def test_ragged_tokens_against_restatement(moe_ffn_module):
    rng = np.random.default_rng(21)
    T, H, F, E, k = 131, 48, 40, 16, 3
    x = rng.standard_normal((T, H)).astype(np.float32)
    wr = (rng.standard_normal((E, H)) * 0.2).astype(np.float32)
    wu, wg = ((rng.standard_normal((F, H, E)) * 0.05).astype(np.float32) for _ in range(2))
    wd = (rng.standard_normal((H, F, E)) * 0.05).astype(np.float32)
    y = moe_ffn_module.moe_ffn_block(x, wr, wu, wg, wd, E, k, H, F, True)
    assert_close(y, O.moe_ffn_block_grouped(x, wr, wu, wg, wd, E, k, H, F, True), rtol=1e-4, atol=1e-5)


def test_bad_shapes_raise(moe_ffn_module):
    g = load_golden("moe_basic")
    a = list(_args(g))
    a[7] = a[7] + 1  # n_embd mismatch
    with pytest.raises(ValueError):
        moe_ffn_module.moe_ffn_block(*a)
