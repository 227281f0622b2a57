"""NumPy restatement of the reference MoE FFN path (test infrastructure only).

Every function cites the reference file:line it follows (paths relative to
the frank-models project root).  Two forms are provided:

* ``*_literal`` follow the reference step by step, including the
  materialised gather of whole expert matrices (``oracles/moe.py:33-48``).
  They are only feasible at small sizes.
* ``*_grouped`` are algebraically identical restatements that sort the
  (slot, token) pairs by expert and run one dense GEMM per expert.  They are
  what the CPU baseline times at the large configurations.

The one deliberate deviation from the reference is the top-k tie rule: the
reference uses ``np.argsort(-probs, axis=0)`` (``oracles/moe.py:95``), whose
default sort is not stable, so the expert chosen among exactly equal
probabilities is unspecified.  Here ties go to the LOWEST expert index
(``kind="stable"``), the same rule the CUDA router kernel implements.
"""

from __future__ import annotations

import numpy as np


# --------------------------------------------------------------------------
# activation  (oracles/activation.py:6-21, components/activation/swiglu.mlir:37-47)
# --------------------------------------------------------------------------

def silu(x: np.ndarray) -> np.ndarray:
    """u / (1 + exp(-u))  -- oracles/activation.py:6-8."""
    return x / (1 + np.exp(-x))


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """gate * silu(up): SiLU is applied to ``up``, not ``gate``
    (oracles/activation.py:11-21, components/activation/swiglu.mlir:37-46)."""
    return gate * silu(up)


# --------------------------------------------------------------------------
# routing  (components/moe/moe_ffn_block.mlir:54-128, oracles/moe.py:86-105)
# --------------------------------------------------------------------------

def router_logits(x: np.ndarray, wr: np.ndarray) -> np.ndarray:
    """logits[E, T] = Wr[E, H] @ x[T, H].T  -- oracles/moe.py:87."""
    return wr @ x.T


def softmax_experts(logits: np.ndarray) -> np.ndarray:
    """Max-subtracted softmax over the expert axis 0 -- oracles/moe.py:90-91,
    moe_ffn_block.mlir:72-75."""
    e = np.exp(logits - logits.max(axis=0, keepdims=True))
    return e / e.sum(axis=0, keepdims=True)


def topk_stable(probs: np.ndarray, k: int):
    """Descending top-k over axis 0, ties to the lowest expert index.

    Follows oracles/moe.py:95-100 (argsort of -probs, take_along_axis) and
    the ``ogt`` comparator of moe_ffn_block.mlir:77-89, with the tie rule
    pinned to stable order.  Returns (weights [k, T] float, ids [k, T] int32).
    """
    idx = np.argsort(-probs, axis=0, kind="stable")[:k]
    w = np.take_along_axis(probs, idx, axis=0)
    return w, idx.astype(np.int32)


def renormalize(w: np.ndarray) -> np.ndarray:
    """w / sum_k w  -- oracles/moe.py:103-105, moe_ffn_block.mlir:91-128."""
    return w / w.sum(axis=0, keepdims=True)


def route(x, wr, k, normalize):
    """Router -> softmax -> top-k -> optional renorm.  Returns (w [k,T], ids [k,T])."""
    probs = softmax_experts(router_logits(x, wr))
    w, ids = topk_stable(probs, k)
    if normalize:
        w = renormalize(w)
    return w, ids


def route_from_logits(logits, k, normalize):
    """Same as :func:`route` but starting from precomputed logits [E, T]."""
    w, ids = topk_stable(softmax_experts(logits), k)
    if normalize:
        w = renormalize(w)
    return w, ids


# --------------------------------------------------------------------------
# permutation  (canonical order defined by mul_mat_id.mlir:51-53)
# --------------------------------------------------------------------------

def permutation(ids: np.ndarray, n_expert: int):
    """Expert-sorted order of the flattened (slot, token) pairs.

    ``mul_mat_id.mlir:51-53`` flattens ids[k, T] slot-major, so flat slot
    s = j*T + t.  The grouped path processes slots sorted by expert, stable
    in s.  Returns:
      sorted_slots[k*T]  -- flat slot s at each sorted row
      offsets[E+1]       -- exclusive prefix of per-expert counts
      slot_pos[k*T]      -- sorted row of each flat slot (inverse permutation)
    """
    flat = ids.reshape(-1).astype(np.int64)
    sorted_slots = np.argsort(flat, kind="stable").astype(np.int32)
    counts = np.bincount(flat, minlength=n_expert)
    offsets = np.zeros(n_expert + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    slot_pos = np.empty_like(sorted_slots)
    slot_pos[sorted_slots] = np.arange(sorted_slots.size, dtype=np.int32)
    return sorted_slots, offsets, slot_pos


# --------------------------------------------------------------------------
# mul_mat_id  (oracles/moe.py:9-48, components/moe/mul_mat_id.mlir:22-120)
# --------------------------------------------------------------------------

def mul_mat_id_literal(weights, inp, ids):
    """out[:, j, t] = weights[:, :, ids[j, t]] @ inp[:, j, t].

    Step by step as oracles/moe.py:30-48: transpose weights to [E, O, I]
    (mul_mat_id.mlir:38-48), gather whole matrices per (slot, token)
    (:58-61), matrix-vector per pair (:86-94), transpose to [O, k, T]
    (:96-117).
    """
    wt = weights.transpose(2, 0, 1)                # [E, O, I]
    g = wt[ids]                                    # [k, T, O, I]
    xin = inp.transpose(1, 2, 0)                   # [k, T, I]
    out = np.einsum("etoi,eti->eto", g, xin)       # [k, T, O]
    return out.transpose(2, 0, 1)


def mul_mat_id_grouped(weights, inp, ids):
    """Grouped restatement of :func:`mul_mat_id_literal`: one GEMM per expert
    over the slots routed to it.  Identical algebra, O(k*T*O*I) work."""
    n_out, n_in, n_expert = weights.shape
    k, T = ids.shape
    flat_in = inp.reshape(n_in, k * T)             # column s = j*T + t
    sorted_slots, offsets, _ = permutation(ids, n_expert)
    out = np.empty((n_out, k * T), dtype=np.result_type(weights, inp))
    for e in range(n_expert):
        sl = sorted_slots[offsets[e]:offsets[e + 1]]
        if sl.size == 0:
            continue
        out[:, sl] = weights[:, :, e] @ flat_in[:, sl]
    return out.reshape(n_out, k, T)


# --------------------------------------------------------------------------
# moe_ffn_block  (oracles/moe.py:51-132, components/moe/moe_ffn_block.mlir:34-209)
# --------------------------------------------------------------------------

def moe_ffn_block_literal(x, wr, w_up, w_gate, w_down, n_expert, k, n_embd, n_ff,
                          normalize):
    """Follows oracles/moe.py:84-132 step for step (replicate, three
    mul_mat_id calls, swiglu(gate, up), weight, sum over k, transpose)."""
    T = x.shape[0]
    w, ids = route(x, wr, k, normalize)
    xr = np.broadcast_to(x.T[:, None, :], (n_embd, k, T)).copy()   # moe.py:109-111
    up = mul_mat_id_literal(w_up, xr, ids)                         # moe.py:114
    gate = mul_mat_id_literal(w_gate, xr, ids)                     # moe.py:117
    act = swiglu(gate, up)                                         # moe.py:120
    down = mul_mat_id_literal(w_down, act, ids)                    # moe.py:123
    return (down * w[None, :, :]).sum(axis=1).T                    # moe.py:126-132


def moe_ffn_block_grouped(x, wr, w_up, w_gate, w_down, n_expert, k, n_embd, n_ff,
                          normalize, routing=None):
    """Grouped restatement of :func:`moe_ffn_block_literal`.

    Per expert e with routed slots S_e: h = swiglu(X_S @ Wg_e.T, X_S @ Wu_e.T),
    d = h @ Wd_e.T, scaled by the gate weight of each slot, then summed over
    the k slots of each token in slot order j = 0..k-1 (moe.py:126-129).
    ``routing`` may pass precomputed (w, ids) to skip the router.
    """
    T = x.shape[0]
    if routing is None:
        w, ids = route(x, wr, k, normalize)
    else:
        w, ids = routing
    sorted_slots, offsets, _ = permutation(ids, n_expert)
    dt = np.result_type(x, w_up)
    d_slots = np.zeros((k * T, n_embd), dtype=dt)
    tok = sorted_slots % T
    wflat = w.reshape(-1)
    for e in range(n_expert):
        lo, hi = offsets[e], offsets[e + 1]
        if lo == hi:
            continue
        sl = sorted_slots[lo:hi]
        xe = x[tok[lo:hi]]
        g = xe @ w_gate[:, :, e].T
        u = xe @ w_up[:, :, e].T
        h = swiglu(g, u)
        d_slots[sl] = (h @ w_down[:, :, e].T) * wflat[sl][:, None]
    return d_slots.reshape(k, T, n_embd).sum(axis=0)


# --------------------------------------------------------------------------
# MoE FFN sub-layer  (oracles/transformer_layer.py:107-124,
# architectures/llm/transformer_layer_moe_prefill.mlir:211-245)
# --------------------------------------------------------------------------

def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """(x / sqrt(sum(x^2, -1) / H + eps)) * weight, step for step as
    oracles/normalization.py:10-43 (components/normalization/rms_norm.mlir:18-80)."""
    ss = np.sum(x * x, axis=-1, keepdims=True)
    rms = np.sqrt(ss / x.shape[-1] + eps)
    return (x / rms) * weight


def moe_ffn_sublayer(residual, ffn_norm_w, eps, wr, w_up, w_gate, w_down, n_expert, k, n_embd, n_ff, normalize,
                     routing=None, grouped=True):
    """residual + moe_ffn_block(rms_norm(residual, ffn_norm_w, eps)) --
    oracles/transformer_layer.py:107-124 (rms_norm at :110, block :112-123,
    residual add :124).  ``routing`` as in :func:`moe_ffn_block_grouped`."""
    xn = rms_norm(residual, ffn_norm_w, eps)
    if grouped:
        moe = moe_ffn_block_grouped(xn, wr, w_up, w_gate, w_down, n_expert, k, n_embd, n_ff, normalize,
                                    routing=routing)
    else:
        moe = moe_ffn_block_literal(xn, wr, w_up, w_gate, w_down, n_expert, k, n_embd, n_ff, normalize)
    return residual + moe
