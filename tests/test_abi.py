"""CPU checks of the C-ABI library: it exists, loads without a GPU, and
exports every function include/*.h declares; the Python binding covers the
same set."""

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(frank_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__  # noqa: F401  (ensures sys.path)
    from frank_b200 import _lib

    if not _lib.LIB_PATH.exists():
        import importlib.util

        spec = importlib.util.spec_from_file_location("fb_build", REPO / "frank-models_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return ctypes.CDLL(str(_lib.LIB_PATH))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "frank_moe_ffn_block" in names and "frank_mul_mat_id" in names and "frank_swiglu" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(lib, name):
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_covers_header():
    from frank_b200 import _lib

    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_calls_without_device_work(lib):
    from frank_b200 import _lib

    L = _lib.load()
    assert L.frank_abi_version() == 102
    # size queries are pure host arithmetic
    assert L.frank_moe_ffn_block_workspace_size(1, 16384, 4096, 14336, 8, 2) > 16384 * 2 * 4096 * 2
    assert L.frank_permute_workspace_size(0, 8) > 0
    # argument validation fails before touching a device
    st = L.frank_softmax_topk(None, 4, 0, 1, 0, None, None, None)
    assert st == _lib.EINVAL and b"E=" in L.frank_last_error()
    st = L.frank_swiglu(7, None, None, None, 4, None)
    assert st == _lib.EINVAL
    st = L.frank_moe_ffn_block(1, None, 0, None, None, None, None, 4, 8, 9, 64, 64, 0, 0, None, None, None, None,
                               0, None)
    assert st == _lib.EINVAL and b"n_expert_used" in L.frank_last_error()
