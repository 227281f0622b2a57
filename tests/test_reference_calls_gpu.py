"""The reference's own component tests, replayed on the B200 module.

tests/golden/record_reference_calls.py runs the reference's test files
(tests/components/test_{mul_mat_id,moe_ffn_block,swiglu,rms_norm}.py)
unchanged and records every module call their bodies make -- arguments,
the reference oracle's result and the tolerance the body passes to
``assert_close``.  Here each call goes through ``frank_b200.B200Module``
(numpy in, numpy out, as the reference harness calls its IREE module) and
the result must meet that same tolerance: rtol 1e-4 / atol 1e-5 for the
MoE functions, the reference's default 1e-5 / 1e-6 for swiglu and rms_norm.
"""

import numpy as np
import pytest

from tests import refcalls

pytestmark = pytest.mark.gpu

FILES = refcalls.files()


@pytest.mark.parametrize("path", FILES, ids=[p.stem.replace("refcall_", "") for p in FILES])
def test_reference_call(b200_module, path):
    test, fn, args, expected, rtol, atol = refcalls.load(path)
    got = getattr(b200_module, fn)(*args)
    np.testing.assert_allclose(np.asarray(got), expected, rtol=rtol, atol=atol, err_msg=test)
