"""The CPU oracle reproduces every committed golden fixture bit for bit
(tests/golden/make_golden.py wrote them), and the seeded tiny decoders the
GPU suite runs on are byte-identical to the ones the fixtures came from."""
import ctypes as C
import json
import os
import sys

import numpy as np
import pytest

from rapidocrvl_b200 import config, synth

import pyoracle
from pyoracle import ptr

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
QT = {"q8": 1000, "q4": 1001, "q6": 1002}


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("q", ["q8", "q4", "q6"])
def test_ops_fixture(oracle_lib, q):
    L = oracle_lib
    f = _load(f"ops_{q}.npz")
    typ = QT[q]
    rows = f["mv_packed"].shape[0]
    cols = f["mv_x"].size
    out = np.zeros(rows, np.float32)
    L.orc_matvec(typ, rows, cols, ptr(f["mv_scale"]), ptr(f["mv_packed"]), ptr(f["mv_x"]), ptr(out))
    assert np.array_equal(_bits(out), _bits(f["mv_out"]))

    rows, cols = f["add_packed"].shape[0], f["add_x"].size
    for ip in (0, 1):
        r = f["add_resid"].copy()
        no = np.zeros(rows, np.float32)
        L.orc_matvec_add_rmsnorm(typ, rows, cols, ptr(f["add_scale"]), ptr(f["add_packed"]), ptr(f["add_x"]), ptr(r),
                                 ptr(f["add_norm_w"]), np.float32(1e-5), ip, ptr(no))
        assert np.array_equal(_bits(r), _bits(f[f"add_resid_out{ip}"]))
        assert np.array_equal(_bits(no), _bits(f[f"add_norm_out{ip}"]))

    rows, cols = f["swi_gpacked"].shape[0], f["swi_x"].size
    out = np.zeros(rows, np.float32)
    L.orc_swiglu(typ, rows, cols, ptr(f["swi_gscale"]), ptr(f["swi_gpacked"]), ptr(f["swi_uscale"]),
                 ptr(f["swi_upacked"]), ptr(f["swi_x"]), ptr(out))
    assert np.array_equal(_bits(out), _bits(f["swi_out"]))

    rows, cols = f["lm_packed"].shape[0], f["lm_x"].shape[1]
    for i in range(f["lm_x"].shape[0]):
        best = C.c_float(0)
        idx = L.orc_argmax_matvec(typ, rows, cols, ptr(f["lm_scale"]), ptr(f["lm_packed"]),
                                  ptr(np.ascontiguousarray(f["lm_x"][i])), C.byref(best))
        assert idx == f["lm_ids"][i]


def test_misc_fixture(oracle_lib):
    L = oracle_lib
    f = _load("misc.npz")
    for n in f["softmax_lens"]:
        y = f[f"softmax_in_{n}"].copy()
        L.orc_softmax(ptr(y), int(n))
        assert np.array_equal(_bits(y), _bits(f[f"softmax_out_{n}"])), n
    cfg = config.Config(**synth.TINY_CONFIG)
    oc = pyoracle.make_config(cfg)
    cs = np.zeros(64, np.float32)
    sn = np.zeros(64, np.float32)
    L.orc_rope_table(C.byref(oc), 7, 3, 11, ptr(cs), ptr(sn))
    assert np.array_equal(_bits(cs), _bits(f["rope_cos"])) and np.array_equal(_bits(sn), _bits(f["rope_sin"]))
    y = f["rope_in"].copy()
    L.orc_rope(ptr(y), 4, 128, ptr(cs), ptr(sn))
    assert np.array_equal(_bits(y), _bits(f["rope_out"]))
    for n in (5, 40):
        o = np.zeros(16 * 128, np.float32)
        L.orc_attention(ptr(f[f"attn_q_{n}"]), ptr(f[f"attn_k_{n}"]), ptr(f[f"attn_v_{n}"]), n, 16, 2, 128, ptr(o))
        assert np.array_equal(_bits(o), _bits(f[f"attn_out_{n}"]))
    for i in range(f["rms_x"].shape[0]):
        o = np.zeros(1024, np.float32)
        L.orc_rmsnorm(ptr(np.ascontiguousarray(f["rms_x"][i])), ptr(f["rms_w"]), 1024, np.float32(1e-5), ptr(o))
        assert np.array_equal(_bits(o), _bits(f["rms_out"][i]))


def test_tiny_greedy_fixture(tiny_models):
    sys.path.insert(0, GOLDEN)
    from make_golden import file_sha256

    with open(os.path.join(GOLDEN, "tiny_greedy.json")) as fh:
        g = json.load(fh)
    cfg = config.Config(**synth.TINY_CONFIG)
    assert synth.random_prompt(g["prompt_len"], cfg.vocab_size, g["prompt_seed"]) == g["prompt"]
    for q, d in tiny_models.items():
        path = os.path.join(d, f"model-{q}.gguf")
        assert file_sha256(path) == g["models"][q]["gguf_sha256"], f"seeded tiny {q} model changed"
        om = pyoracle.OracleModel(path, config.load(d))
        ids = om.generate(g["prompt"], g["max_new"], eos=[])
        om.close()
        assert ids == g["models"][q]["ids"]


def test_sampling_fixture():
    f = _load("sampling.npz")
    for V in (2048, 4160):
        x, seeds = f[f"logits_{V}"], f[f"seeds_{V}"]
        for c, (t, k) in enumerate(f["cases"]):
            for r in range(x.shape[0]):
                st = pyoracle.RNG(int(seeds[r]))
                assert pyoracle.sample_token(x[r], float(t), int(k), st) == f[f"ids_{V}"][c, r], (V, t, k, r)
                assert st.state == int(f[f"states_{V}"][c, r])
