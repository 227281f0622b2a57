"""GGUF-style parameter binding (frank_b200.params): name and shape checks on
the host, and on the GPU a toy parameter dict (the reference's layout,
tests/models/test_toy_llm.py:111-124 of the reference) run through the layer
against the oracle."""

import numpy as np
import pytest
import torch

from frank_b200 import params as P
from oracle import moe_oracle as O
from tests.utils import assert_close


def _toy_params(n_layers=2, E=4, k=2, H=32, F=48, seed=0):
    rng = np.random.default_rng(seed)
    p = {}
    for i in range(n_layers):
        b = f"blk.{i}."
        p[b + "ffn_norm.weight"] = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        p[b + "ffn_gate_inp.weight"] = (rng.standard_normal((E, H)) * 0.1).astype(np.float32)
        p[b + "ffn_up_exps.weight"] = (rng.standard_normal((F, H, E)) * 0.1).astype(np.float32)
        p[b + "ffn_gate_exps.weight"] = (rng.standard_normal((F, H, E)) * 0.1).astype(np.float32)
        p[b + "ffn_down_exps.weight"] = (rng.standard_normal((H, F, E)) * 0.1).astype(np.float32)
        p[b + "attn_q.weight"] = np.zeros((H, H), np.float32)  # other tensors of the layer are ignored
    return p


def test_names_follow_the_reference():
    n = P.param_names(3)
    assert n == {"norm": "blk.3.ffn_norm.weight", "router": "blk.3.ffn_gate_inp.weight",
                 "up": "blk.3.ffn_up_exps.weight", "gate": "blk.3.ffn_gate_exps.weight",
                 "down": "blk.3.ffn_down_exps.weight"}


def test_shapes_inferred_and_checked():
    p = _toy_params()
    s = P.moe_param_shapes(p, 1)
    assert (s.n_expert, s.n_embd, s.n_ff, s.has_norm) == (4, 32, 48, True)
    q = dict(p)
    del q["blk.0.ffn_norm.weight"]
    assert not P.moe_param_shapes(q, 0).has_norm
    q = dict(p)
    del q["blk.0.ffn_down_exps.weight"]
    with pytest.raises(KeyError, match="ffn_down_exps"):
        P.moe_param_shapes(q, 0)
    q = dict(p)
    q["blk.0.ffn_gate_exps.weight"] = np.zeros((48, 32, 5), np.float32)
    with pytest.raises(ValueError, match="ffn_gate_exps"):
        P.moe_param_shapes(q, 0)
    q = dict(p)
    q["blk.0.ffn_down_exps.weight"] = np.zeros((48, 32, 4), np.float32)  # [F, H, E] instead of [H, F, E]
    with pytest.raises(ValueError, match="ffn_down_exps"):
        P.moe_param_shapes(q, 0)
    q = dict(p)
    q["blk.0.ffn_norm.weight"] = np.zeros(31, np.float32)
    with pytest.raises(ValueError, match="ffn_norm"):
        P.moe_param_shapes(q, 0)


@pytest.mark.gpu
def test_layers_from_params_match_oracle():
    p = _toy_params()
    layers = P.moe_layers_from_params(p, 2, n_expert_used=2, dtype=torch.float32)
    rng = np.random.default_rng(9)
    for i, layer in enumerate(layers):
        b = f"blk.{i}."
        resid = (rng.standard_normal((10, 32)) * 2).astype(np.float32)
        y = layer.sublayer(torch.from_numpy(resid).cuda(), 1e-5).cpu().numpy()
        ref = O.moe_ffn_sublayer(resid, p[b + "ffn_norm.weight"], 1e-5, p[b + "ffn_gate_inp.weight"],
                                 p[b + "ffn_up_exps.weight"], p[b + "ffn_gate_exps.weight"],
                                 p[b + "ffn_down_exps.weight"], 4, 2, 32, 48, False)
        assert_close(y, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_chunked_packing_equals_one_shot():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((70, 24, 3)).astype(np.float32)
    from frank_b200 import ops
    whole = ops.prepack_experts(torch.from_numpy(w).cuda(), torch.bfloat16)
    chunked = P.pack_reference_experts(w, torch.bfloat16, "cuda", chunk_bytes=24 * 3 * 4 * 9).packed
    assert torch.equal(whole, chunked)
