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


# fp32 unit roundoff
U32 = 2.0 ** -24


def strict_routing(logits64, err_scale, gpu_w, gpu_ids, k, normalize, probs64=None):
    """The strict routing tier: the GPU's expert ids must equal the oracle's
    top-k on float64 logits for every token whose k-th/(k+1)-th logit gap is
    above twice the worst-case fp32 accumulation error of a length-H dot
    product on each side of the gap (gamma_H * sum_i |w_i x_i|, Higham's
    bound), doubled again for the tensor core's truncating accumulation.

    ``logits64`` [E,T] float64 logits of the inputs the GPU saw,
    ``err_scale`` [E,T] the per-logit error bound of :func:`router_error_scale`.  Returns ``(w, ids, n_near, n_diff)``:
    the routing the oracle should run with (the oracle's own ids and float64
    weights, except on near-tied tokens where the GPU chose differently: there
    the GPU's ids with the oracle's float64 weights at those ids), the number
    of near-tied tokens and the number of tokens whose ids differ.  Raises
    AssertionError if a token outside the near-tie set differs."""
    from oracle import moe_oracle as O

    E, T = logits64.shape
    ow, oids = O.route_from_logits(logits64, k, normalize)
    gpu_ids = np.asarray(gpu_ids)
    if k < E:
        order = np.argsort(-logits64, axis=0, kind="stable")
        srt = np.take_along_axis(logits64, order, axis=0)
        gap = srt[k - 1] - srt[k]
    else:
        gap = np.full(T, np.inf)
    # the two logits compared each carry at most max_e err_scale[e, t];
    # doubled once more for the tensor core's truncating accumulation
    near = gap <= 4.0 * err_scale.max(axis=0)
    diff = np.any(gpu_ids != oids, axis=0)
    bad = diff & ~near
    assert not bad.any(), (f"{int(bad.sum())} tokens route differently with a logit gap above the fp32 bound "
                           f"(first: {np.flatnonzero(bad)[:5]})")
    ids = oids.copy()
    w = np.asarray(ow, dtype=np.float64).copy()
    if diff.any():
        p = O.softmax_experts(logits64[:, diff]) if probs64 is None else probs64[:, diff]
        gi = gpu_ids[:, diff].astype(np.int64)
        wd = np.take_along_axis(p, gi, axis=0)
        if normalize:
            wd = wd / wd.sum(axis=0, keepdims=True)
        ids[:, diff] = gi
        w[:, diff] = wd
    # weights of agreeing tokens: the GPU's fp32 weights within fp32 rounding of the oracle's
    ok = ~diff
    np.testing.assert_allclose(np.asarray(gpu_w, dtype=np.float64)[:, ok], w[:, ok], rtol=1e-4, atol=1e-6)
    return w, ids.astype(np.int32), int(near.sum()), int(diff.sum())


def router_error_scale(wr32, x_bf16_f64):
    """gamma_H * |Wr| @ |x|.T: the worst-case fp32 error of each router logit
    (H products summed in fp32, gamma_H = H*u / (1 - H*u))."""
    H = wr32.shape[1]
    gamma = H * U32 / (1.0 - H * U32)
    return gamma * (np.abs(wr32.astype(np.float64)) @ np.abs(x_bf16_f64).T)


class ExpertSlices:
    """A [O, I, E]-indexable float64 view of packed [E, O, I] expert weights
    that converts one expert at a time (``w[:, :, e]``), so the grouped oracle
    can run on multi-GB weight sets without a float64 copy of all of them."""

    dtype = np.dtype(np.float64)

    def __init__(self, packed):
        self.packed = packed  # torch [E, O, I] (any device, bf16 or fp32)
        E, O_, I = packed.shape
        self.shape = (O_, I, E)

    def __getitem__(self, key):
        a, b, e = key
        assert a == slice(None) and b == slice(None) and isinstance(e, (int, np.integer))
        return self.packed[int(e)].float().cpu().numpy().astype(np.float64)


def strict_route(x64, wr32, gpu_w, gpu_ids, k, normalize):
    """:func:`strict_routing` from the inputs: float64 logits of ``x64``
    [T,H] (the values the GPU read) under the fp32 router ``wr32`` [E,H]."""
    wr32 = np.asarray(wr32, dtype=np.float32)
    logits = wr32.astype(np.float64) @ x64.T
    return strict_routing(logits, router_error_scale(wr32, x64), gpu_w, gpu_ids, k, normalize)
