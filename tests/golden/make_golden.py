"""Regenerates the golden fixtures in tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

The Go reference cannot run on this image (no Go toolchain), so the fixtures
are the oracle's outputs on seeded inputs; the oracle itself is pinned to the
reference's own known-answer tests by tests/test_oracle_kats.py.  The CPU
suite checks that the oracle still reproduces every fixture bit for bit, and
the GPU suite checks the CUDA engine against the same files, so a change on
either side shows up as a fixture mismatch.

Files
  ops_{q8,q4,q6}.npz  quantized matrices (as stored in GGUF) with inputs and
                      oracle outputs of matvec, matvec+residual+RMSNorm (in
                      place and out only), SwiGLU and lm_head argmax
  misc.npz            softmax for every length rule (1..40, 64, 100), RoPE
                      table + rotation, decode attention at 5 and 40 cached
                      positions, RMSNorm
  tiny_greedy.json    greedy ids of the seeded tiny decoders (q8/q6/q4) and
                      the sha256 of each GGUF file the ids came from
  sampling.npz        logits rows with, per (temperature, top_k), the sampled
                      id and the advanced fastRNG state of each row's seed
                      (top-k candidates, full vocabulary in one and in four
                      cumulative-sum blocks, argmax)
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import pyoracle  # noqa: E402
from pyoracle import ptr  # noqa: E402

from rapidocrvl_b200 import config, gguf, synth  # noqa: E402

QTYPES = {"q8": gguf.Q8_ROW, "q4": gguf.Q4_ROW, "q6": gguf.Q6_ROW}
# (rows, cols) of the fixture matrices: tiny-decoder-like qkv / o / gate / lm_head shapes
MV_SHAPE = (160, 256)
ADD_SHAPE = (256, 256)
SWI_SHAPE = (192, 256)
LM_SHAPE = (512, 256)
EPS = np.float32(1e-5)
GREEDY_PROMPT = (6, 0)  # (length, seed) of synth.random_prompt
GREEDY_NEW = 24


def _f32(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


def ops_fixture(q: str) -> dict:
    L = pyoracle.lib()
    typ = QTYPES[q]
    rng = np.random.default_rng({"q8": 11, "q4": 12, "q6": 13}[q])
    f = {}

    rows, cols = MV_SHAPE
    sc, pk = gguf.quantize_rows(typ, _f32(rng, (rows, cols), 0.02))
    x = _f32(rng, cols)
    out = np.zeros(rows, np.float32)
    L.orc_matvec(typ, rows, cols, ptr(sc), ptr(pk), ptr(x), ptr(out))
    f.update(mv_scale=sc, mv_packed=pk, mv_x=x, mv_out=out)

    rows, cols = ADD_SHAPE
    sc, pk = gguf.quantize_rows(typ, _f32(rng, (rows, cols), 0.02))
    x = _f32(rng, cols)
    res = _f32(rng, rows)
    nw = _f32(rng, rows, 0.02)
    f.update(add_scale=sc, add_packed=pk, add_x=x, add_resid=res, add_norm_w=nw)
    for in_place in (0, 1):
        r = res.copy()
        no = np.zeros(rows, np.float32)
        L.orc_matvec_add_rmsnorm(typ, rows, cols, ptr(sc), ptr(pk), ptr(x), ptr(r), ptr(nw), EPS, in_place, ptr(no))
        f[f"add_resid_out{in_place}"] = r
        f[f"add_norm_out{in_place}"] = no

    rows, cols = SWI_SHAPE
    gs, gp = gguf.quantize_rows(typ, _f32(rng, (rows, cols), 0.02))
    us, up = gguf.quantize_rows(typ, _f32(rng, (rows, cols), 0.02))
    x = _f32(rng, cols)
    out = np.zeros(rows, np.float32)
    L.orc_swiglu(typ, rows, cols, ptr(gs), ptr(gp), ptr(us), ptr(up), ptr(x), ptr(out))
    f.update(swi_gscale=gs, swi_gpacked=gp, swi_uscale=us, swi_upacked=up, swi_x=x, swi_out=out)

    rows, cols = LM_SHAPE
    sc, pk = gguf.quantize_rows(typ, _f32(rng, (rows, cols), 0.02))
    xs = _f32(rng, (4, cols))
    ids = np.zeros(4, np.int32)
    for i in range(4):
        best = C.c_float(0)
        ids[i] = L.orc_argmax_matvec(typ, rows, cols, ptr(sc), ptr(pk), ptr(np.ascontiguousarray(xs[i])),
                                     C.byref(best))
    f.update(lm_scale=sc, lm_packed=pk, lm_x=xs, lm_ids=ids)
    return f


def misc_fixture() -> dict:
    L = pyoracle.lib()
    rng = np.random.default_rng(21)
    f = {}
    lens = list(range(1, 41)) + [64, 100]
    f["softmax_lens"] = np.array(lens, np.int32)
    for n in lens:
        x = _f32(rng, n, 3.0)
        y = x.copy()
        L.orc_softmax(ptr(y), n)
        f[f"softmax_in_{n}"] = x
        f[f"softmax_out_{n}"] = y

    cfg = config.Config(**synth.TINY_CONFIG)
    oc = pyoracle.make_config(cfg)
    half = cfg.head_dim // 2
    cs = np.zeros(half, np.float32)
    sn = np.zeros(half, np.float32)
    L.orc_rope_table(C.byref(oc), 7, 3, 11, ptr(cs), ptr(sn))
    x = _f32(rng, 4 * cfg.head_dim)
    y = x.copy()
    L.orc_rope(ptr(y), 4, cfg.head_dim, ptr(cs), ptr(sn))
    f.update(rope_cos=cs, rope_sin=sn, rope_in=x, rope_out=y)

    heads, kvh, dim = 16, 2, 128
    for n in (5, 40):
        q = _f32(rng, heads * dim)
        k = _f32(rng, (n, kvh * dim))
        v = _f32(rng, (n, kvh * dim))
        o = np.zeros(heads * dim, np.float32)
        L.orc_attention(ptr(q), ptr(k), ptr(v), n, heads, kvh, dim, ptr(o))
        f.update({f"attn_q_{n}": q, f"attn_k_{n}": k, f"attn_v_{n}": v, f"attn_out_{n}": o})

    x = _f32(rng, (3, 1024))
    w = _f32(rng, 1024, 0.02)
    out = np.zeros((3, 1024), np.float32)
    for i in range(3):
        L.orc_rmsnorm(ptr(np.ascontiguousarray(x[i])), ptr(w), 1024, EPS, ptr(out[i]))
    f.update(rms_x=x, rms_w=w, rms_out=out)
    return f


# (temperature, top_k) cases of the sampling fixture; top_k 0 = full vocabulary
SAMPLE_CASES = [(0.0, 0), (0.8, 1), (1.0, 2), (0.7, 3), (1.0, 4), (1.3, 5), (1.0, 40), (0.6, 200), (1.0, 0), (0.5, 0),
                (1.7, 0)]


def sampling_fixture() -> dict:
    rng = np.random.default_rng(33)
    f = {"cases": np.array(SAMPLE_CASES, np.float64)}
    for V in (2048, 4160):
        x = _f32(rng, (6, V), 2.0)
        x[1] = np.round(x[1] * 2) / 2  # ties
        x[2, : V // 2] = -30.0
        seeds = rng.integers(-(1 << 62), 1 << 62, 6, dtype=np.int64)
        f[f"logits_{V}"] = x
        f[f"seeds_{V}"] = seeds
        ids = np.zeros((len(SAMPLE_CASES), 6), np.int32)
        states = np.zeros((len(SAMPLE_CASES), 6), np.uint64)
        for c, (t, k) in enumerate(SAMPLE_CASES):
            for r in range(6):
                st = pyoracle.RNG(int(seeds[r]))
                ids[c, r] = pyoracle.sample_token(x[r], t, k, st)
                states[c, r] = st.state
        f[f"ids_{V}"] = ids
        f[f"states_{V}"] = states
    return f


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for blk in iter(lambda: fh.read(1 << 20), b""):
            h.update(blk)
    return h.hexdigest()


def greedy_fixture() -> dict:
    out = {"prompt_len": GREEDY_PROMPT[0], "prompt_seed": GREEDY_PROMPT[1], "max_new": GREEDY_NEW, "models": {}}
    cfg = config.Config(**synth.TINY_CONFIG)
    prompt = synth.random_prompt(GREEDY_PROMPT[0], cfg.vocab_size, GREEDY_PROMPT[1])
    out["prompt"] = prompt
    for q in ("q8", "q6", "q4"):
        d = synth.ensure("tiny", q)
        path = os.path.join(d, f"model-{q}.gguf")
        om = pyoracle.OracleModel(path, config.load(d))
        ids = om.generate(prompt, GREEDY_NEW, eos=[])
        om.close()
        out["models"][q] = {"gguf_sha256": file_sha256(path), "ids": ids}
    return out


def main():
    pyoracle.build()
    for q in QTYPES:
        np.savez_compressed(os.path.join(HERE, f"ops_{q}.npz"), **ops_fixture(q))
    np.savez_compressed(os.path.join(HERE, "misc.npz"), **misc_fixture())
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), **sampling_fixture())
    with open(os.path.join(HERE, "tiny_greedy.json"), "w") as fh:
        json.dump(greedy_fixture(), fh)
        fh.write("\n")


if __name__ == "__main__":
    main()
