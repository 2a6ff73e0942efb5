"""ocrvl_op_argmax_noalloc: the allocation-free argmax for callers that must
not allocate device memory (a server whose GPU memory is already reserved by
its own pools, or a loop that cannot take cudaMalloc's possible device
synchronisation).  It must give the same ids as ocrvl_op_argmax, call after
call, although its keys live in one static device array that every call
reuses.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rapidocrvl_b200 import _lib, gguf  # noqa: E402


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("typ", [gguf.Q4_ROW, gguf.Q8_ROW])
def test_noalloc_argmax_matches_allocating_entry_point(typ):
    torch = _torch()
    L = _lib.load()
    rows, cols, m = 8192, 1024, 3
    rng = np.random.default_rng(17)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    sc, packed = gguf.quantize_rows(typ, w)
    wd = torch.from_numpy(packed).cuda()
    sd = torch.from_numpy(sc).cuda()
    rs = torch.zeros(rows, dtype=torch.int32, device="cuda")
    _lib.check(L.ocrvl_op_rowsum(typ, rows, cols, _p(wd), _p(rs), None))
    # two calls in a row with different inputs: the second must not see the
    # first call's keys left in the shared static array
    for call, seed in enumerate((1, 2)):
        x = torch.from_numpy(np.random.default_rng(seed).standard_normal((m, cols)).astype(np.float32)).cuda()
        want = torch.full((m,), -1, dtype=torch.int32, device="cuda")
        got = torch.full((m,), -1, dtype=torch.int32, device="cuda")
        _lib.check(L.ocrvl_op_argmax(typ, rows, cols, _p(wd), _p(sd), _p(rs), m, _p(x), _p(want), None))
        _lib.check(L.ocrvl_op_argmax_noalloc(typ, rows, cols, _p(wd), _p(sd), _p(rs), m, _p(x), _p(got), None))
        torch.cuda.synchronize()
        assert got.cpu().tolist() == want.cpu().tolist(), f"call {call}"
        assert all(0 <= i < rows for i in got.cpu().tolist())


def test_noalloc_argmax_rejects_more_vectors_than_its_scratch():
    _torch()
    L = _lib.load()
    rc = L.ocrvl_op_argmax_noalloc(gguf.Q4_ROW, 256, 1024, None, None, None, 9, None, None, None)
    assert rc == _lib.E_INVALID
    assert "exceeds the 8 vectors" in _lib.last_error()
