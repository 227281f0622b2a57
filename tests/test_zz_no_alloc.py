"""frank_permute_noalloc: the permutation for callers that cannot allocate
device memory (their host framework owns the memory pool, or their FFI
binding cannot keep a workspace alive).  It uses a fixed 1 MiB library-owned
device array as scratch instead of a caller workspace.

Checked through the C ABI against the existing workspace-taking entry point
(frank_permute): integer outputs must be identical, on two calls in a row
(the second call sees the first call's leftovers in the shared array).
Kept in its own file, collected last.
"""


import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from frank_b200 import _lib

    return _lib, _lib.load()


def _outs(n, E):
    dev = torch.device("cuda")
    return (torch.full((n,), -7, dtype=torch.int32, device=dev),
            torch.full((E + 1,), -7, dtype=torch.int32, device=dev),
            torch.full((n,), -7, dtype=torch.int32, device=dev),
            torch.zeros(1, dtype=torch.int32, device=dev))


def _with_workspace(ids, E):
    L, lib = _lib()
    n = ids.numel()
    ss, off, pos, err = _outs(n, E)
    ws_bytes = lib.frank_permute_workspace_size(n, E)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=ids.device)
    st = torch.cuda.current_stream().cuda_stream
    L.check(lib.frank_permute(ids.data_ptr(), n, E, ss.data_ptr(), off.data_ptr(), pos.data_ptr(), err.data_ptr(),
                              ws.data_ptr(), ws_bytes, st))
    return ss, off, pos, err


def _no_alloc(ids, E):
    L, lib = _lib()
    n = ids.numel()
    ss, off, pos, err = _outs(n, E)
    st = torch.cuda.current_stream().cuda_stream
    L.check(lib.frank_permute_noalloc(ids.data_ptr(), n, E, ss.data_ptr(), off.data_ptr(), pos.data_ptr(),
                                      err.data_ptr(), st))
    return ss, off, pos, err


def test_no_alloc_matches_workspace_entry_point_twice():
    rng = np.random.default_rng(1234)
    cases = [(128, 8, 4000), (8, 2, 16384)]  # (E, k, T); the second is larger and reuses the array
    for E, k, T in cases:
        ids = torch.from_numpy(rng.integers(0, E, size=(k, T)).astype(np.int32)).cuda()
        a = _with_workspace(ids, E)
        b = _no_alloc(ids, E)
        torch.cuda.synchronize()
        for x, y in zip(a, b):
            assert torch.equal(x, y)
        assert int(b[1][-1].item()) == k * T


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    L, lib = _lib()
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    big_n = 1 << 22  # needs ~16 MiB of scratch
    st = lib.frank_permute_noalloc(ids.data_ptr(), big_n, 8, None, None, None, None,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == L.EINVAL
    assert b"scratch" in lib.frank_last_error()
