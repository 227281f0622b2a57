"""ctypes binding of ``libfrankmoe.so`` (the C ABI in include/frank_moe.h).

The library is built in-tree by ``frank-models_b200/build.py``.  There is no
fallback: if the shared object is missing or fails to load, every call
raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfrankmoe.so"

F32 = 0
BF16 = 1
ROUTER_PACKED = 16  # wr_dtype of a router pack (frank_router_pack)

OK = 0
EINVAL = -1
EIDS = -2
ECUDA = -3
ENOSPC = -4
ETIMEOUT = -5
ENCCL = -6

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/frank_moe.h one to one.
SIGNATURES = {
    "frank_last_error": (ctypes.c_char_p, []),
    "frank_abi_version": (_c_int, []),
    "frank_num_sms": (_c_int, []),
    "frank_swiglu": (_c_int, [_c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_vp]),
    "frank_softmax_topk": (_c_int, [_c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp]),
    "frank_router_scratch_bytes": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64]),
    "frank_router_pack_size": (_c_size, [_c_i64, _c_i64]),
    "frank_router_pack_offset": (_c_size, [_c_i64, _c_i64]),
    "frank_router_pack": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp]),
    "frank_router_topk": (_c_int, [_c_int, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int,
                                   _c_vp, _c_vp, _c_vp, _c_vp]),
    "frank_permute_workspace_size": (_c_size, [_c_i64, _c_i64]),
    "frank_permute": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_size, _c_vp]),
    "frank_permute_noalloc": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),
    "frank_prepack_experts": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp]),
    "frank_mul_mat_id_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "frank_mul_mat_id": (_c_int, [_c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp,
                                  _c_vp, _c_vp, _c_size, _c_vp]),
    "frank_moe_ffn_block_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "frank_moe_ffn_block": (_c_int, [_c_int, _c_vp, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64,
                                     _c_i64, _c_i64, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_size, _c_vp]),
    "frank_rms_norm": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float, _c_int, _c_vp, _c_vp]),
    "frank_moe_ffn_sublayer_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "frank_moe_ffn_sublayer": (_c_int, [_c_int, _c_vp, _c_vp, ctypes.c_float, _c_int, _c_vp, _c_vp, _c_vp, _c_vp,
                                        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_vp,
                                        _c_size, _c_vp]),
    "frank_gather_rows": (_c_int, [_c_int, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp]),
    "frank_gather_weights": (_c_int, [_c_vp, _c_vp, _c_i64, _c_vp, _c_vp]),
    "frank_expert_ffn_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64]),
    "frank_expert_ffn": (_c_int, [_c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp,
                                  _c_vp, _c_vp, _c_size, _c_vp]),
    "frank_combine": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp]),
    "frank_copy_row_segments": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp]),
    "frank_ep_plan": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp]),
    "frank_ep_dispatch": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp,
                                   _c_vp, _c_int, _c_i64, _c_vp, _c_vp]),
    "frank_expert_ffn_scatter": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp,
                                          _c_vp, _c_vp, _c_vp, _c_int, _c_i64, _c_vp, _c_size, _c_vp]),
    "frank_read_device_error": (_c_int, [_c_vp, _c_vp]),
    "frank_launch_count": (ctypes.c_uint64, []),
    "frank_selftest_bounded_wait": (_c_int, [_c_i64, _c_vp, _c_vp]),
    "frank_profile_stages": (_c_int, [_c_int]),
    "frank_profile_read": (_c_int, [_c_vp, _c_int, _c_vp]),
}

_lib = None


class FrankError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"frank status {code}: {msg}")
        self.code = code


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise FrankError(-3, f"{p} is missing: build it with `python frank-models_b200/build.py`")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    """Raise FrankError with frank_last_error() when status != 0."""
    if status != OK:
        msg = load().frank_last_error()
        raise FrankError(status, msg.decode() if msg else "")
