"""Run the reference's component test files UNCHANGED and record every call
they make on the compiled module, for replay against the B200 module.

    python tests/golden/record_reference_calls.py --reference <frank-models checkout>

The reference's tests (tests/components/test_{mul_mat_id,moe_ffn_block,
swiglu,rms_norm}.py) import ``compile_component`` / ``link_and_compile`` /
``assert_close`` from their ``tests/utils.py``, which needs the IREE compiler
and runtime (tests/utils.py:14-31) -- not installable offline.  This script
runs those test files as they are, under pytest, with a stand-in
``tests.utils`` whose module objects compute each call with the reference's
own oracles (oracles/moe.py, oracles/activation.py, oracles/normalization.py)
and record it: the method name, every argument, the result and the
tolerance the test body then passes to ``assert_close``.  The reference's
assertions run too (and pass trivially, since the stand-in returns the
oracle's result).  One ``refcall_*.npz`` per call lands in this directory;
tests/test_reference_calls_gpu.py replays each call through
``frank_b200.B200Module`` on a B200 and applies the recorded tolerance.

The reference's sources stay where they are: only the recorded inputs and
outputs are written here, and nothing at test time needs the reference tree.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
TEST_FILES = ["test_mul_mat_id.py", "test_moe_ffn_block.py", "test_swiglu.py", "test_rms_norm.py"]


class _State:
    calls: list = []      # dicts, in call order
    pending: list = []    # calls of the running test not yet matched to an assert_close


def _current_test() -> str:
    cur = os.environ.get("PYTEST_CURRENT_TEST", "?")
    return cur.split(" ")[0]


class IREEConfig:
    """Stand-in for tests/utils.py:IREEConfig (no runtime is created)."""

    def __init__(self, backend="llvm-cpu", iree_tools_dir=None, save_linked_ir=None, **_):
        self.backend = backend


class RecordingModule:
    """Stand-in for the compiled module: ``module.<fn>(*args)`` evaluates the
    reference's oracle for that function and records the call."""

    def __init__(self, oracles):
        self._oracles = oracles

    def __getattr__(self, name):
        fn = self._oracles[name]

        def call(*args):
            result = np.asarray(fn(*args))
            rec = {"test": _current_test(), "fn": name, "args": args, "result": result}
            _State.calls.append(rec)
            _State.pending.append(rec)
            return result

        return call


def make_utils(oracles):
    mod = types.ModuleType("tests.utils")
    mod.IREEConfig = IREEConfig

    def compile_component(component_path, iree_cfg, *a, **k):
        return RecordingModule(oracles)

    def link_and_compile(main_path=None, library_paths=None, iree_cfg=None, *a, **k):
        return RecordingModule(oracles)

    def assert_close(actual, expected, rtol=1e-5, atol=1e-6):
        # same contract as the reference's tests/utils.py:244-251; the
        # tolerance is attached to the calls made since the previous assert
        for rec in _State.pending:
            rec["rtol"], rec["atol"] = rtol, atol
        _State.pending.clear()
        np.testing.assert_allclose(np.asarray(actual), np.asarray(expected), rtol=rtol, atol=atol)

    mod.compile_component = compile_component
    mod.link_and_compile = link_and_compile
    mod.assert_close = assert_close
    return mod


def _save(calls, out_dir: Path):
    for old in out_dir.glob("refcall_*.npz"):
        old.unlink()
    seen = {}
    for rec in calls:
        test = rec["test"].split("::")
        base = f"refcall_{Path(test[0]).stem.replace('test_', '')}__{test[-1]}"
        n = seen.get(base, 0)
        seen[base] = n + 1
        arrays = {"fn": np.array(rec["fn"]), "test": np.array(rec["test"]), "result": rec["result"],
                  "rtol": np.array(rec["rtol"]), "atol": np.array(rec["atol"]), "n_args": np.array(len(rec["args"]))}
        for i, a in enumerate(rec["args"]):
            if isinstance(a, np.ndarray):
                arrays[f"arg{i}"] = a
                arrays[f"kind{i}"] = np.array("array")
            else:
                kind = "bool" if isinstance(a, (bool, np.bool_)) else "int" if isinstance(a, (int, np.integer)) \
                    else "float"
                arrays[f"arg{i}"] = np.array(a)
                arrays[f"kind{i}"] = np.array(kind)
        np.savez_compressed(out_dir / f"{base}__{n}.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a frank-models checkout")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    ref = Path(args.reference).resolve()
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref))
    import oracles.activation as act
    import oracles.moe as moe
    import oracles.normalization as norm
    import pytest

    oracles = {"mul_mat_id": moe.mul_mat_id, "moe_ffn_block": moe.moe_ffn_block, "swiglu": act.swiglu,
               "rms_norm_linalg": norm.rms_norm}
    import tests as ref_tests  # the reference's own tests package (its __init__ only)

    assert Path(ref_tests.__file__).resolve().parent == ref / "tests", ref_tests.__file__
    sys.modules["tests.utils"] = make_utils(oracles)
    files = [str(ref / "tests" / "components" / f) for f in TEST_FILES]
    rc = pytest.main(["-q", "-p", "no:cacheprovider", "--rootdir", str(ref), *files])
    if rc != 0:
        raise SystemExit(f"the reference's tests failed under the recording module (pytest exit {rc})")
    missing = [r["test"] for r in _State.calls if "rtol" not in r]
    if missing:
        raise SystemExit(f"calls without a following assert_close: {missing}")
    _save(_State.calls, Path(args.out))
    print(f"recorded {len(_State.calls)} calls from {len({r['test'] for r in _State.calls})} tests")


if __name__ == "__main__":
    main()
