"""The C-ABI library: it builds for sm_100a, loads without a GPU, exports
exactly the functions include/ocrvl_cuda.h declares, and rejects bad
arguments on the host before any CUDA call.  No compute entry point runs."""
import ctypes as C
import os
import re
import subprocess

import pytest

from rapidocrvl_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ocrvl_cuda.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = re.sub(r"#[^\n]*", "", src)
    return set(re.findall(r"\b(ocrvl_[a-z0-9_]+)\s*\(", src))


def exported_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_matches_binding_table():
    names = header_functions()
    assert len(names) >= 25
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_library_exports_every_header_symbol():
    L = _lib.load()
    syms = exported_symbols(_lib.lib_path())
    missing = header_functions() - syms
    assert not missing, missing
    for name in header_functions():
        assert getattr(L, name) is not None
    # no stray C-ABI exports beyond the header
    extra = {s for s in syms if s.startswith("ocrvl_")} - header_functions()
    assert not extra, extra


def _desc(**kw):
    d = _lib.ModelDesc()
    base = dict(vocab_size=1000, hidden_size=256, intermediate_size=384, num_layers=2, num_heads=4, num_kv_heads=2,
                head_dim=128, rms_norm_eps=1e-5, rope_theta=5e5)
    base.update(kw)
    for k, v in base.items():
        setattr(d, k, v)
    for i, s in enumerate((16, 24, 24)):
        d.mrope_section[i] = s
    return d


@pytest.mark.parametrize("kw,msg", [
    (dict(head_dim=64), "head_dim must be 128"),
    (dict(num_layers=0), "dimensions must be positive"),
    (dict(num_heads=3), "num_heads must be"),
    (dict(hidden_size=200), "multiples of 128"),
    (dict(num_heads=32, num_kv_heads=2), "num_heads must be"),
])
def test_init_rejects_bad_shapes_on_host(kw, msg):
    L = _lib.load()
    h = C.c_void_p()
    rc = L.ocrvl_init(0, C.byref(_desc(**kw)), C.byref(h))
    assert rc == _lib.E_INVALID
    assert msg in _lib.last_error()
    assert not h.value


def test_null_handles_are_rejected():
    L = _lib.load()
    assert L.ocrvl_init(0, None, None) == _lib.E_INVALID
    assert L.ocrvl_quant_type(None) == _lib.E_INVALID
    assert L.ocrvl_seq_len(None) == _lib.E_INVALID
    assert L.ocrvl_model_stream(None) is None
    assert L.ocrvl_step(None, None, 1, None, None, None, 1, None, None) == _lib.E_INVALID
    h2d, d2h = C.c_int64(), C.c_int64()
    assert L.ocrvl_step_io_bytes(None, 1, C.byref(h2d), C.byref(d2h)) == _lib.E_INVALID
    assert L.ocrvl_decode_greedy_device(None, None, 1, None, 1, None) == _lib.E_INVALID
    L.ocrvl_free(None)
    L.ocrvl_seq_free(None)


def test_device_count_reports_or_fails_cleanly():
    n = _lib.load().ocrvl_device_count()
    assert n >= 0 or n == _lib.E_CUDA
    if n < 0:
        assert "cudaGetDeviceCount" in _lib.last_error()
