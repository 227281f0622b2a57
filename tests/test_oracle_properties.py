"""Properties of the oracle restatement on random inputs (CPU, hypothesis):
the facts the GPU parity tests lean on beyond the fixed golden vectors.

- routing: k distinct ids per token, weights in descending order, ties to
  the lower index, renormalised weights summing to 1 (moe_ffn_block.mlir:72-128);
- grouped restatements equal the literal step-by-step forms
  (oracles/moe.py:9-48, :51-132) on random shapes and ids, including
  repeated and absent experts;
- the block is linear in the down weights and row-independent in the tokens;
- the sub-layer's output minus its residual is the block applied to the
  normalised residual (oracles/transformer_layer.py:107-124).
"""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import moe_oracle as O

shapes = st.tuples(st.integers(1, 9), st.integers(1, 8), st.integers(1, 5), st.integers(2, 12))  # T, E, k, H


def _block_inputs(seed, T, H, F, E):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H))
    wr = rng.standard_normal((E, H)) * 0.3
    wu = rng.standard_normal((F, H, E)) * 0.3
    wg = rng.standard_normal((F, H, E)) * 0.3
    wd = rng.standard_normal((H, F, E)) * 0.3
    return x, wr, wu, wg, wd


@settings(max_examples=60, deadline=None)
@given(shapes, st.integers(0, 10_000), st.booleans())
def test_routing_invariants(shape, seed, normalize):
    T, E, k, H = shape
    k = min(k, E)
    rng = np.random.default_rng(seed)
    # coarse logits make exact ties frequent
    logits = rng.integers(-3, 4, size=(E, T)).astype(np.float64)
    w, ids = O.route_from_logits(logits, k, normalize)
    probs = O.softmax_experts(logits)
    for t in range(T):
        assert len(set(ids[:, t].tolist())) == k
        assert np.all(np.diff(w[:, t]) <= 0)  # renormalising divides by a positive sum: order kept
        chosen = probs[ids[:, t], t]
        # descending by probability, equal probabilities in ascending id order
        for j in range(k - 1):
            assert chosen[j] > chosen[j + 1] or (chosen[j] == chosen[j + 1] and ids[j, t] < ids[j + 1, t])
        # nothing left out beats the last chosen one
        rest = np.setdiff1d(np.arange(E), ids[:, t])
        if rest.size:
            assert np.all((probs[rest, t] < chosen[-1]) | ((probs[rest, t] == chosen[-1]) & (rest > ids[-1, t])))
        if normalize:
            assert abs(w[:, t].sum() - 1.0) < 1e-12


@settings(max_examples=40, deadline=None)
@given(shapes, st.integers(1, 10), st.integers(0, 10_000))
def test_mul_mat_id_grouped_equals_literal(shape, O_, seed):
    T, E, k, I = shape
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((O_, I, E))
    inp = rng.standard_normal((I, k, T))
    ids = rng.integers(0, E, size=(k, T)).astype(np.int32)  # repeats and absent experts
    np.testing.assert_allclose(O.mul_mat_id_grouped(w, inp, ids), O.mul_mat_id_literal(w, inp, ids),
                               rtol=1e-12, atol=1e-12)


@settings(max_examples=30, deadline=None)
@given(shapes, st.integers(1, 6), st.integers(0, 10_000), st.booleans())
def test_block_grouped_equals_literal(shape, F, seed, normalize):
    T, E, k, H = shape
    k = min(k, E)
    x, wr, wu, wg, wd = _block_inputs(seed, T, H, F, E)
    args = (x, wr, wu, wg, wd, E, k, H, F, normalize)
    np.testing.assert_allclose(O.moe_ffn_block_grouped(*args), O.moe_ffn_block_literal(*args),
                               rtol=1e-10, atol=1e-12)


@settings(max_examples=30, deadline=None)
@given(shapes, st.integers(1, 6), st.integers(0, 10_000), st.floats(-3, 3))
def test_block_linear_in_down_weights_and_row_independent(shape, F, seed, alpha):
    T, E, k, H = shape
    k = min(k, E)
    x, wr, wu, wg, wd = _block_inputs(seed, T, H, F, E)
    y = O.moe_ffn_block_grouped(x, wr, wu, wg, wd, E, k, H, F, False)
    ya = O.moe_ffn_block_grouped(x, wr, wu, wg, alpha * wd, E, k, H, F, False)
    np.testing.assert_allclose(ya, alpha * y, rtol=1e-10, atol=1e-12)
    # each token's output depends on that token alone
    for t in range(T):
        yt = O.moe_ffn_block_grouped(x[t:t + 1], wr, wu, wg, wd, E, k, H, F, False)
        np.testing.assert_allclose(yt[0], y[t], rtol=1e-12, atol=1e-12)


@settings(max_examples=30, deadline=None)
@given(shapes, st.integers(1, 6), st.integers(0, 10_000), st.floats(1e-8, 1e-2))
def test_sublayer_is_residual_plus_block_of_norm(shape, F, seed, eps):
    T, E, k, H = shape
    k = min(k, E)
    x, wr, wu, wg, wd = _block_inputs(seed, T, H, F, E)
    nw = np.random.default_rng(seed + 1).standard_normal(H)
    out = O.moe_ffn_sublayer(x, nw, eps, wr, wu, wg, wd, E, k, H, F, False)
    xn = O.rms_norm(x, nw, eps)
    np.testing.assert_allclose(out - x, O.moe_ffn_block_grouped(xn, wr, wu, wg, wd, E, k, H, F, False),
                               rtol=1e-9, atol=1e-11)
    # with unit weights and eps = 0 every normalised row has root mean square 1
    ones = O.rms_norm(x, np.ones(H), 0.0)
    np.testing.assert_allclose(np.sqrt(np.mean(ones * ones, axis=-1)), 1.0, rtol=1e-12)
