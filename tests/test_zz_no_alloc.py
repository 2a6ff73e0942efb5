"""ocrvl_op_argmax_noalloc: the allocation-free argmax for callers that must
not allocate device memory (a server whose GPU memory is already reserved by
its own pools, or a loop that cannot take cudaMalloc's possible device
synchronisation).  It must give the same ids as ocrvl_op_argmax, call after
call, although its keys live in one static device array that every call
reuses.  This file is collected last on purpose."""
import ctypes as C
import os
import subprocess
import sys

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


@pytest.mark.parametrize("m", [1, 3, 8])  # 1: the single-vector GEMV; 8: the whole static array
@pytest.mark.parametrize("typ", [gguf.Q4_ROW, gguf.Q8_ROW])
def test_noalloc_argmax_matches_allocating_entry_point(typ, m):
    torch = _torch()
    L = _lib.load()
    rows, cols = 8192, 1024
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


_FRESH = r"""
import ctypes as C, sys
import numpy as np, torch
from rapidocrvl_b200 import _lib, gguf
L = _lib.load()
rows, cols, m = 4096, 1024, 8
typ = gguf.Q4_ROW
w = (np.random.default_rng(3).standard_normal((rows, cols)) * 0.02).astype(np.float32)
sc, packed = gguf.quantize_rows(typ, w)
p = lambda t: C.c_void_p(t.data_ptr())
wd, sd = torch.from_numpy(packed).cuda(), torch.from_numpy(sc).cuda()
rs = torch.zeros(rows, dtype=torch.int32, device="cuda")
x = torch.randn(m, cols, device="cuda")
ids = torch.zeros(m, dtype=torch.int32, device="cuda")
_lib.check(L.ocrvl_op_rowsum(typ, rows, cols, p(wd), p(rs), None))
# first call: module load and the static array's address lookup
_lib.check(L.ocrvl_op_argmax_noalloc(typ, rows, cols, p(wd), p(sd), p(rs), m, p(x), p(ids), None))
torch.cuda.synchronize()
before = torch.cuda.mem_get_info()[0]
for _ in range(20):
    _lib.check(L.ocrvl_op_argmax_noalloc(typ, rows, cols, p(wd), p(sd), p(rs), m, p(x), p(ids), None))
torch.cuda.synchronize()
after = torch.cuda.mem_get_info()[0]
print(before, after)
"""


def test_noalloc_argmax_leaves_free_device_memory_unchanged():
    """In a fresh process that never calls the allocating entry point: once
    the first call has loaded the module, further calls leave the device's
    free memory exactly as it was (any allocation takes at least a page)."""
    _torch()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", _FRESH], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    before, after = map(int, r.stdout.split()[-2:])
    assert before == after, (before, after)
