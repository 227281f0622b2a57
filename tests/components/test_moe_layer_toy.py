"""Whole MoE transformer layers of the reference's toy model, with the MoE
FFN sub-layer on the B200.

The fixtures (tests/golden/layer_toy_*.npz, written by make_golden.py from
the reference's own oracles) hold, for layers 0 and 1 of the toy model
(n_embd 64, n_ff 128, 4 experts, top-2; tests/models/test_toy_llm.py:29-124)
on the token batches of its prefill tests (:677-801): the layer input, the
attention half's residual ``input + attention(rms_norm(input))``
(oracles/transformer_layer.py:74-104, evaluated by the reference's attention
oracle, which is outside this library's scope) and the output of the
reference's whole ``transformer_layer_moe`` (:14-124).  The GPU test runs
the MoE FFN sub-layer ``residual1 + moe_ffn_block(rms_norm(residual1))``
through ``B200Module.moe_ffn_sublayer`` (fp32 path) on that residual and
must reproduce the whole layer's output within the toy model test's
tolerance, rtol 1e-3 / atol 1e-4 (test_toy_llm.py:730-736).
"""

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.utils import golden_names, load_golden

CASES = golden_names("layer_toy_")


def _sublayer_args(g):
    r = g["residual1"].reshape(-1, int(g["n_embd"]))
    return (r, g["ffn_norm_w"], float(g["rms_eps"]), g["gate_inp_w"], g["up_exps_w"], g["gate_exps_w"],
            g["down_exps_w"], int(g["n_expert"]), int(g["n_expert_used"]), int(g["n_embd"]), int(g["n_ff"]),
            bool(g["normalize_weights"]))


def test_cases_present():
    assert len(CASES) == 6


@pytest.mark.parametrize("name", CASES)
def test_oracle_composes_the_layer(name):
    """The restatement's sub-layer on the attention residual reproduces the
    reference's whole layer (pins the composition on the CPU)."""
    g = load_golden(name)
    got = O.moe_ffn_sublayer(*_sublayer_args(g), grouped=False)
    np.testing.assert_allclose(got.reshape(g["expected"].shape), g["expected"], rtol=1e-3, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_layer_with_b200_moe_sublayer(name, moe_ffn_module):
    g = load_golden(name)
    got = moe_ffn_module.moe_ffn_sublayer(*_sublayer_args(g))
    np.testing.assert_allclose(got.reshape(g["expected"].shape), g["expected"], rtol=1e-3, atol=1e-4)
