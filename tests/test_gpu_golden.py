"""The CUDA engine (through the C ABI) against the committed golden fixtures
(tests/golden/make_golden.py): op outputs bit for bit, greedy ids of the
seeded tiny decoders equal, and the image-prompt generation path (embedding
rows at placeholder positions, M-RoPE positions, rope delta) against the
oracle run the same way."""
import ctypes as C
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rapidocrvl_b200 import GenerateOptions, LoadOptions, Runtime, _lib, config, synth  # noqa: E402
from rapidocrvl_b200.runtime import expand_single_image_placeholder, multimodal_positions  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
QT = {"q8": 1000, "q4": 1001, "q6": 1002}


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return C.c_void_p(t.data_ptr())


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


class _Dev:
    """Device copies of fixture arrays, kept alive for the whole test."""

    def __init__(self, torch):
        self.torch = torch
        self.keep = []

    def __call__(self, a):
        t = self.torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.keep.append(t)
        return t

    def mat(self, L, typ, scale, packed, cols):
        w, s = self(packed), self(scale)
        rs = self.torch.zeros(packed.shape[0], dtype=self.torch.int32, device="cuda")
        self.keep.append(rs)
        _lib.check(L.ocrvl_op_rowsum(typ, packed.shape[0], cols, _p(w), _p(rs), None))
        return w, s, rs


@pytest.mark.parametrize("q", ["q8", "q4", "q6"])
def test_ops_match_golden(q):
    torch = _torch()
    L = _lib.load()
    f = np.load(os.path.join(GOLDEN, f"ops_{q}.npz"))
    typ = QT[q]
    d = _Dev(torch)

    rows, cols = f["mv_packed"].shape[0], f["mv_x"].size
    w, s, rs = d.mat(L, typ, f["mv_scale"], f["mv_packed"], cols)
    out = d(np.zeros(rows, np.float32))
    _lib.check(L.ocrvl_op_matvec(typ, rows, cols, _p(w), _p(s), _p(rs), 1, _p(d(f["mv_x"])), None, 0.0, _p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(f["mv_out"]))

    rows, cols = f["add_packed"].shape[0], f["add_x"].size
    w, s, rs = d.mat(L, typ, f["add_scale"], f["add_packed"], cols)
    for ip in (0, 1):
        res = d(f["add_resid"].copy())
        vout = d(np.zeros(rows, np.float32))
        nout = d(np.zeros(rows, np.float32))
        _lib.check(L.ocrvl_op_matvec_add_rmsnorm(typ, rows, cols, _p(w), _p(s), _p(rs), 1, _p(d(f["add_x"])), _p(res),
                                                 ip, _p(d(f["add_norm_w"])), 1e-5, _p(vout), _p(nout), None))
        torch.cuda.synchronize()
        assert np.array_equal(_bits(nout.cpu().numpy()), _bits(f[f"add_norm_out{ip}"]))
        assert np.array_equal(_bits(res.cpu().numpy()), _bits(f[f"add_resid_out{ip}"]))

    rows, cols = f["swi_gpacked"].shape[0], f["swi_x"].size
    wg, sg, rsg = d.mat(L, typ, f["swi_gscale"], f["swi_gpacked"], cols)
    wu, su, rsu = d.mat(L, typ, f["swi_uscale"], f["swi_upacked"], cols)
    out = d(np.zeros(rows, np.float32))
    _lib.check(L.ocrvl_op_swiglu(typ, rows, cols, _p(wg), _p(sg), _p(rsg), _p(wu), _p(su), _p(rsu), 1,
                                 _p(d(f["swi_x"])), _p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(f["swi_out"]))

    rows, cols = f["lm_packed"].shape[0], f["lm_x"].shape[1]
    w, s, rs = d.mat(L, typ, f["lm_scale"], f["lm_packed"], cols)
    m = f["lm_x"].shape[0]
    ids = torch.zeros(m, dtype=torch.int32, device="cuda")
    _lib.check(L.ocrvl_op_argmax(typ, rows, cols, _p(w), _p(s), _p(rs), m, _p(d(f["lm_x"])), _p(ids), None))
    torch.cuda.synchronize()
    assert ids.cpu().numpy().tolist() == f["lm_ids"].tolist()


def test_rmsnorm_matches_golden():
    torch = _torch()
    L = _lib.load()
    f = np.load(os.path.join(GOLDEN, "misc.npz"))
    d = _Dev(torch)
    m, n = f["rms_x"].shape
    out = d(np.zeros((m, n), np.float32))
    _lib.check(L.ocrvl_op_rmsnorm(n, m, _p(d(f["rms_x"])), _p(d(f["rms_w"])), 1e-5, _p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(f["rms_out"]))


@pytest.mark.parametrize("q", ["q8", "q6", "q4"])
def test_tiny_greedy_matches_golden(tiny_models, q):
    _torch()
    with open(os.path.join(GOLDEN, "tiny_greedy.json")) as fh:
        g = json.load(fh)
    rt = Runtime.load(tiny_models[q], LoadOptions(quantization=q, max_position=4096, kv_pool_bytes=1 << 28))
    got = rt.generate_with_options(g["prompt"], GenerateOptions(max_new_tokens=g["max_new"], eos_token_ids=[]))
    rt.close()
    assert got.tokens == g["models"][q]["ids"]


def _oracle_image_generate(orc, cfg, ids, emb, grid, max_new):
    inp = expand_single_image_placeholder(ids, len(emb), cfg.image_token_id)
    pos, delta = multimodal_positions(inp, grid, cfg.image_token_id, cfg.spatial_merge_size)
    seq = orc.new_seq(len(inp) + max_new)
    cur = 0
    tok = -1
    for i, t in enumerate(inp):
        e = emb[cur] if t == cfg.image_token_id else orc.embed(t)
        cur += t == cfg.image_token_id
        tok, _, _ = seq.forward(e, pos[i], need_logits=i == len(inp) - 1)
    out = list(inp)
    for i in range(max_new):
        out.append(tok)
        if i + 1 >= max_new:
            break
        p = len(out) - 1 + delta
        tok, _, _ = seq.forward(orc.embed(tok), (p, p, p), need_logits=True)
    return out


@pytest.mark.parametrize("q", ["q4", "q8"])
def test_image_embeds_generation_matches_oracle(tiny_models, q):
    """GenerateWithImageEmbeds (internal/model/model.go:1582-1707): one image
    placeholder expanded to a 1x4x4 grid (2x2 merge -> 4 embedding rows)."""
    _torch()
    import pyoracle

    d = tiny_models[q]
    cfg = config.load(d)
    cfg.image_token_id = 999
    cfg.spatial_merge_size = 2
    rt = Runtime.load(d, LoadOptions(quantization=q, max_position=4096, kv_pool_bytes=1 << 28))
    rt.cfg.image_token_id = 999
    rt.cfg.spatial_merge_size = 2
    orc = pyoracle.OracleModel(os.path.join(d, f"model-{q}.gguf"), cfg)
    emb = (np.random.default_rng(4).standard_normal((4, cfg.hidden_size)) * 0.05).astype(np.float32)
    ids = [5, 17, 999, 23, 42]
    got = rt.generate_with_image_embeds(ids, emb, [1, 4, 4], GenerateOptions(max_new_tokens=16, eos_token_ids=[]))
    want = _oracle_image_generate(orc, cfg, ids, emb, [1, 4, 4], 16)
    assert got.prompt_tokens == 8
    assert got.tokens == want
    with pytest.raises(ValueError, match="not enough image placeholder"):
        rt.generate_with_image_embeds([5, 999, 999, 6], emb[:3], [1, 4, 4], GenerateOptions(max_new_tokens=2))
    orc.close()
    rt.close()


def test_sampling_fixture_on_device():
    """ocrvl_op_sample on the fixture's logits rows: the oracle's ids and RNG
    states for every (temperature, top_k) case."""
    torch = _torch()
    L = _lib.load()
    f = np.load(os.path.join(GOLDEN, "sampling.npz"))
    for V in (2048, 4160):
        x = torch.from_numpy(np.ascontiguousarray(f[f"logits_{V}"])).cuda()
        m = x.shape[0]
        work = torch.zeros((m, V), dtype=torch.float32, device="cuda")
        for c, (t, k) in enumerate(f["cases"]):
            st = torch.from_numpy(f[f"seeds_{V}"].copy()).cuda()
            out = torch.full((m,), -1, dtype=torch.int32, device="cuda")
            full = t > 0 and k != 1 and not (1 < k < V)
            _lib.check(L.ocrvl_op_sample(m, V, _p(x), float(t), int(k), _p(st), _p(out), None, None,
                                         _p(work) if full else None, None))
            torch.cuda.synchronize()
            assert out.cpu().numpy().tolist() == f[f"ids_{V}"][c].tolist(), (V, t, k)
            assert st.cpu().numpy().view(np.uint64).tolist() == f[f"states_{V}"][c].tolist(), (V, t, k)
