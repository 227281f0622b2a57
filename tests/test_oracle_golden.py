"""Pin the CPU restatement (oracle/) to the reference's own outputs.

The fixtures in tests/golden/ were produced by running the reference's
oracles/moe.py, oracles/activation.py and oracles/normalization.py, the
sub-layer composed as oracles/transformer_layer.py:107-124 does
(tests/golden/make_golden.py).
"""

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.utils import assert_close, golden_names, load_golden


@pytest.mark.parametrize("name", golden_names("mmid_"))
def test_mul_mat_id_literal_and_grouped_match_reference(name):
    g = load_golden(name)
    lit = O.mul_mat_id_literal(g["weights"], g["input"], g["ids"])
    grp = O.mul_mat_id_grouped(g["weights"], g["input"], g["ids"])
    assert_close(lit, g["expected"], rtol=1e-6, atol=1e-7)
    assert_close(grp, g["expected"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", golden_names("moe_"))
def test_moe_ffn_block_literal_and_grouped_match_reference(name):
    g = load_golden(name)
    args = (g["input"], g["gate_inp_w"], g["up_exps_w"], g["gate_exps_w"], g["down_exps_w"],
            int(g["n_expert"]), int(g["n_expert_used"]), int(g["n_embd"]), int(g["n_ff"]),
            bool(g["normalize_weights"]))
    lit = O.moe_ffn_block_literal(*args)
    grp = O.moe_ffn_block_grouped(*args)
    assert lit.shape == g["expected"].shape
    assert_close(lit, g["expected"], rtol=1e-6, atol=1e-7)
    assert_close(grp, g["expected"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", golden_names("swiglu_"))
def test_swiglu_matches_reference(name):
    g = load_golden(name)
    assert_close(O.swiglu(g["gate"], g["up"]), g["expected"], rtol=0, atol=0)


@pytest.mark.parametrize("name", golden_names("rmsnorm_"))
def test_rms_norm_matches_reference(name):
    g = load_golden(name)
    assert_close(O.rms_norm(g["input"], g["weight"], float(g["eps"])), g["expected"], rtol=0, atol=0)


@pytest.mark.parametrize("name", golden_names("sublayer_"))
def test_moe_ffn_sublayer_matches_reference(name):
    g = load_golden(name)
    args = (g["residual"], g["ffn_norm_w"], float(g["rms_eps"]), g["gate_inp_w"], g["up_exps_w"], g["gate_exps_w"],
            g["down_exps_w"], int(g["n_expert"]), int(g["n_expert_used"]), int(g["n_embd"]), int(g["n_ff"]),
            bool(g["normalize_weights"]))
    lit = O.moe_ffn_sublayer(*args, grouped=False)
    grp = O.moe_ffn_sublayer(*args)
    assert_close(lit, g["expected"], rtol=1e-6, atol=1e-7)
    assert_close(grp, g["expected"], rtol=1e-5, atol=1e-7)


def test_permutation_is_stable_argsort():
    rng = np.random.default_rng(0)
    for E, k, T in ((8, 2, 100), (128, 8, 257), (4, 1, 1), (16, 4, 0)):
        ids = rng.integers(0, E, size=(k, T)).astype(np.int32)
        ss, off, pos = O.permutation(ids, E)
        flat = ids.reshape(-1)
        assert np.array_equal(ss, np.argsort(flat, kind="stable"))
        assert off[0] == 0 and off[-1] == flat.size
        assert np.array_equal(np.diff(off), np.bincount(flat, minlength=E))
        assert np.array_equal(ss[pos], np.arange(flat.size))
        # stable: within an expert block the flat slots ascend
        for e in range(E):
            blk = ss[off[e]:off[e + 1]]
            assert np.all(np.diff(blk) > 0)


def test_topk_ties_go_to_lowest_index():
    probs = np.array([[0.25, 0.1], [0.25, 0.4], [0.25, 0.4], [0.25, 0.1]], dtype=np.float32)
    w, ids = O.topk_stable(probs, 2)
    assert ids[:, 0].tolist() == [0, 1]
    assert ids[:, 1].tolist() == [1, 2]
    assert np.allclose(w[:, 0], 0.25)


def test_renormalised_weights_sum_to_one():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((16, 32)).astype(np.float32)
    wr = rng.standard_normal((8, 32)).astype(np.float32)
    w, ids = O.route(x, wr, 3, True)
    assert np.allclose(w.sum(axis=0), 1.0, atol=1e-6)
    assert np.all(np.diff(w, axis=0) <= 0)  # descending
