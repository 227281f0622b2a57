"""swiglu vs the reference's outputs (tests/components/test_swiglu.py:15-59:
default tolerance rtol 1e-5 / atol 1e-6, large values rtol 1e-4 / atol 1e-5)."""

import numpy as np
import pytest
import torch

from tests.utils import assert_close, golden_names, load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("swiglu_"))
def test_golden_case(swiglu_module, name):
    g = load_golden(name)
    out = swiglu_module.swiglu(g["gate"], g["up"])
    if name == "swiglu_large":
        assert_close(out, g["expected"], rtol=1e-4, atol=1e-5)
    else:
        assert_close(out, g["expected"])


def test_bf16_tensor_path(swiglu_module):
    g = torch.randn(3, 5, 64, device="cuda").bfloat16()
    u = torch.randn(3, 5, 64, device="cuda").bfloat16()
    out = swiglu_module.swiglu(g, u)
    ref = g.float() * (u.float() / (1 + torch.exp(-u.float())))
    assert out.dtype == torch.bfloat16
    assert torch.allclose(out.float(), ref, rtol=1e-2, atol=1e-2)


def test_silu_applies_to_up_not_gate(swiglu_module):
    gate = np.full((1, 1, 4), 2.0, np.float32)
    up = np.array([[[0.0, 1.0, -1.0, 3.0]]], np.float32)
    expected = 2.0 * up / (1 + np.exp(-up))
    assert_close(swiglu_module.swiglu(gate, up), expected)
