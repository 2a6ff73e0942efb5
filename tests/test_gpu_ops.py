"""Kernel-level parity: CUDA ops (through the C ABI) against the CPU oracle.

Integer work (dequantisation, int8-activation dots) and every float step whose
order the kernels restate are compared bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rapidocrvl_b200 import _lib, gguf  # noqa: E402

TYPES = [gguf.Q8_ROW, gguf.Q4_ROW, gguf.Q6_ROW]


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


def _quant(typ, rows, cols, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    sc, packed = gguf.quantize_rows(typ, w)
    return sc, packed


def _orc_matvec(L, typ, sc, packed, x):
    import pyoracle

    rows, cols = packed.shape[0], x.shape[-1]
    out = np.zeros(rows, np.float32)
    L.orc_matvec(typ, rows, cols, pyoracle.ptr(sc), pyoracle.ptr(packed), pyoracle.ptr(np.ascontiguousarray(x)),
                 pyoracle.ptr(out))
    return out


def _mat_on_dev(torch, L, typ, sc, packed):
    rows, pb = packed.shape
    cols = {gguf.Q8_ROW: pb, gguf.Q4_ROW: pb * 2, gguf.Q6_ROW: pb * 4 // 3}[typ]
    w = _dev(torch, packed)
    s = _dev(torch, sc)
    rs = torch.zeros(rows, dtype=torch.int32, device="cuda")
    _lib.check(L.ocrvl_op_rowsum(typ, rows, cols, _p(w), _p(rs), None))
    return w, s, rs, cols


@pytest.mark.parametrize("typ", TYPES)
@pytest.mark.parametrize("rows,cols,m", [(256, 1024, 1), (300, 2048, 3), (1024, 3072, 8), (64, 128, 2)])
def test_matvec_bit_exact(oracle_lib, typ, rows, cols, m):
    torch = _torch()
    L = _lib.load()
    sc, packed = _quant(typ, rows, cols, seed=rows + cols + m)
    w, s, rs, _ = _mat_on_dev(torch, L, typ, sc, packed)
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((m, cols)) * 0.5).astype(np.float32)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    xd = _dev(torch, x)
    _lib.check(L.ocrvl_op_matvec(typ, rows, cols, _p(w), _p(s), _p(rs), m, _p(xd), None, 0.0, _p(out), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in range(m):
        want = _orc_matvec(oracle_lib, typ, sc, packed, x[i])
        assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32)), f"seq {i}: max diff {np.abs(got[i]-want).max()}"


@pytest.mark.parametrize("typ", TYPES)
def test_matvec_rmsnorm_prologue_bit_exact(oracle_lib, typ):
    import pyoracle

    torch = _torch()
    L = _lib.load()
    rows, cols, m = 512, 1024, 2
    sc, packed = _quant(typ, rows, cols, seed=11)
    w, s, rs, _ = _mat_on_dev(torch, L, typ, sc, packed)
    rng = np.random.default_rng(3)
    h = rng.standard_normal((m, cols)).astype(np.float32)
    nw = (rng.standard_normal(cols) * 0.02).astype(np.float32)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    hd, nwd = _dev(torch, h), _dev(torch, nw)  # keep device inputs alive until the kernel has run
    _lib.check(L.ocrvl_op_matvec(typ, rows, cols, _p(w), _p(s), _p(rs), m, _p(hd), _p(nwd), 1e-5, _p(out), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in range(m):
        xn = np.zeros(cols, np.float32)
        oracle_lib.orc_rmsnorm(pyoracle.ptr(h[i]), pyoracle.ptr(nw), cols, C.c_float(1e-5), pyoracle.ptr(xn))
        want = _orc_matvec(oracle_lib, typ, sc, packed, xn)
        assert np.array_equal(got[i], want)


@pytest.mark.parametrize("typ", TYPES)
@pytest.mark.parametrize("in_place", [0, 1])
def test_matvec_add_rmsnorm_bit_exact(oracle_lib, typ, in_place):
    import pyoracle

    torch = _torch()
    L = _lib.load()
    rows, cols, m = 1024, 2048, 2
    sc, packed = _quant(typ, rows, cols, seed=5)
    w, s, rs, _ = _mat_on_dev(torch, L, typ, sc, packed)
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((m, cols)) * 0.3).astype(np.float32)
    res = rng.standard_normal((m, rows)).astype(np.float32)
    nw = (rng.standard_normal(rows) * 0.02).astype(np.float32)
    resd = _dev(torch, res.copy())
    vout = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    nout = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    xd, nwd = _dev(torch, x), _dev(torch, nw)
    _lib.check(L.ocrvl_op_matvec_add_rmsnorm(typ, rows, cols, _p(w), _p(s), _p(rs), m, _p(xd), _p(resd),
                                             in_place, _p(nwd), 1e-5, _p(vout), _p(nout), None))
    torch.cuda.synchronize()
    for i in range(m):
        r = res[i].copy()
        want = np.zeros(rows, np.float32)
        oracle_lib.orc_matvec_add_rmsnorm(typ, rows, cols, pyoracle.ptr(sc), pyoracle.ptr(packed), pyoracle.ptr(x[i]),
                                          pyoracle.ptr(r), pyoracle.ptr(nw), C.c_float(1e-5), in_place,
                                          pyoracle.ptr(want))
        assert np.array_equal(nout[i].cpu().numpy(), want)
        assert np.array_equal(resd[i].cpu().numpy(), r)


@pytest.mark.parametrize("typ", TYPES)
def test_swiglu_bit_exact(oracle_lib, typ):
    import pyoracle

    torch = _torch()
    L = _lib.load()
    rows, cols, m = 3072, 1024, 1
    sg, pg = _quant(typ, rows, cols, seed=21)
    su, pu = _quant(typ, rows, cols, seed=22)
    wg, sgd, rsg, _ = _mat_on_dev(torch, L, typ, sg, pg)
    wu, sud, rsu, _ = _mat_on_dev(torch, L, typ, su, pu)
    x = (np.random.default_rng(1).standard_normal((m, cols)) * 2).astype(np.float32)
    out = torch.zeros((m, rows), dtype=torch.float32, device="cuda")
    xd = _dev(torch, x)
    _lib.check(L.ocrvl_op_swiglu(typ, rows, cols, _p(wg), _p(sgd), _p(rsg), _p(wu), _p(sud), _p(rsu), m,
                                 _p(xd), _p(out), None))
    torch.cuda.synchronize()
    want = np.zeros(rows, np.float32)
    oracle_lib.orc_swiglu(typ, rows, cols, pyoracle.ptr(sg), pyoracle.ptr(pg), pyoracle.ptr(su), pyoracle.ptr(pu),
                          pyoracle.ptr(x[0]), pyoracle.ptr(want))
    assert np.array_equal(out[0].cpu().numpy(), want)


@pytest.mark.parametrize("typ", TYPES)
def test_argmax_matches_oracle(oracle_lib, typ):
    import pyoracle

    torch = _torch()
    L = _lib.load()
    rows, cols, m = 103424, 1024, 2
    sc, packed = _quant(typ, rows, cols, seed=99)
    w, s, rs, _ = _mat_on_dev(torch, L, typ, sc, packed)
    x = np.random.default_rng(4).standard_normal((m, cols)).astype(np.float32)
    ids = torch.zeros(m, dtype=torch.int32, device="cuda")
    xd = _dev(torch, x)
    _lib.check(L.ocrvl_op_argmax(typ, rows, cols, _p(w), _p(s), _p(rs), m, _p(xd), _p(ids), None))
    torch.cuda.synchronize()
    for i in range(m):
        want = oracle_lib.orc_argmax_matvec(typ, rows, cols, pyoracle.ptr(sc), pyoracle.ptr(packed),
                                            pyoracle.ptr(x[i]), None)
        assert int(ids[i]) == want


def test_argmax_ties_pick_lowest_row(oracle_lib):
    torch = _torch()
    L = _lib.load()
    rows, cols = 4096, 128
    packed = np.zeros((rows, cols), np.uint8)
    packed[[17, 900, 4000], 0] = 5  # three equal maxima
    sc = np.ones(rows, np.float32)
    w, s, rs, _ = _mat_on_dev(torch, L, gguf.Q8_ROW, sc, packed)
    x = np.ones((1, cols), np.float32)
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    xd = _dev(torch, x)
    _lib.check(L.ocrvl_op_argmax(gguf.Q8_ROW, rows, cols, _p(w), _p(s), _p(rs), 1, _p(xd), _p(ids), None))
    torch.cuda.synchronize()
    assert int(ids[0]) == 17


def test_rmsnorm_bit_exact(oracle_lib):
    import pyoracle

    torch = _torch()
    L = _lib.load()
    n, m = 1024, 3
    rng = np.random.default_rng(8)
    x = rng.standard_normal((m, n)).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    xd, wd = _dev(torch, x), _dev(torch, w)
    _lib.check(L.ocrvl_op_rmsnorm(n, m, _p(xd), _p(wd), 1e-5, _p(out), None))
    torch.cuda.synchronize()
    for i in range(m):
        want = np.zeros(n, np.float32)
        oracle_lib.orc_rmsnorm(pyoracle.ptr(x[i]), pyoracle.ptr(w), n, C.c_float(1e-5), pyoracle.ptr(want))
        assert np.array_equal(out[i].cpu().numpy(), want)


def test_op_rejects_bad_shapes():
    L = _lib.load()
    rc = L.ocrvl_op_matvec(gguf.Q4_ROW, 10, 100, None, None, None, 1, None, None, 0.0, None, None)
    assert rc == _lib.E_INVALID
    assert "128" in _lib.last_error()
