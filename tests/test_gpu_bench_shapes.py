"""Parity of the CUDA engine against the CPU oracle on the benchmark-size
decoder (hidden 1024, 18 layers, 16 q heads over 2 kv heads = GQA group 8,
SwiGLU 3072, vocab 103424): the shapes and kernel paths the BASELINE
configurations run, which the tiny decoders (group 2, 16-row GEMM tiles) do
not reach.

  * 64 sequences in one step (Q4/Q6: the tcgen05 batched kernel with its
    32-row QKV / gate-up tiles, 48-row split-K o / down tiles over 6 K groups
    and 256-row lm_head tiles; Q8: groups of 8), caches from 33 to 4,095
    positions restored from seeded K/V, three steps: logits within the spec
    tolerance of the oracle's and ids equal;
  * a Q6 image prompt of configs[2]'s shape (1,225 embedding rows on a
    1x70x70 grid with a 2x2 merge, then 16 text ids, sectioned M-RoPE
    prefill) followed by 32 greedy ids;
  * single sequences at 4,096 and 8,448 cached positions (configs[3]'s and
    configs[4]'s longest contexts).

The reference behaviour matched is Runtime.forwardEmbeddingForSampling
(internal/model/model.go:3475-3643) through its CPU branches, restated by
oracle/oracle.cpp.
"""
import os

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

from rapidocrvl_b200 import GenerateOptions, LoadOptions, Runtime, config, synth  # noqa: E402
from rapidocrvl_b200.runtime import expand_single_image_placeholder, multimodal_positions  # noqa: E402

LOGIT_ATOL = 2e-2
LOGIT_RTOL = 1e-2
KV_BYTES_PER_POSITION = 18 * 2 * 2 * 128 * 4


def _need_gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _kv_pool(cfg, pool_len, seed):
    """Seeded K/V rows [layers][pool_len][kv_heads*head_dim] that sequences
    take windows of (K scaled by 0.5, V unit normal)."""
    rng = np.random.default_rng(seed)
    kvd = cfg.num_key_value_heads * cfg.head_dim
    shape = (cfg.num_hidden_layers, pool_len, kvd)
    k = (0.5 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
    v = rng.standard_normal(shape, dtype=np.float32)
    return k, v


def _window(pool, n, off):
    idx = (np.arange(n) + off) % pool.shape[1]
    return np.ascontiguousarray(pool[:, idx])


def _check_logits(got, want, what):
    """The spec's tolerance, then bit equality: every kernel of the step
    restates the reference's arithmetic in its order (int8 dots, the fp32
    FMA slot orders, the norms, RoPE, the softmax forms and the sequential
    value sums), so the logits are the oracle's bit for bit."""
    err = np.abs(got - want)
    bad = err > LOGIT_ATOL + LOGIT_RTOL * np.abs(want)
    assert not bad.any(), f"{what}: {int(bad.sum())} logits outside tolerance, max err {float(err.max()):.3g}"
    nd = int(np.count_nonzero(got != want))
    assert nd == 0, f"{what}: {nd} logits differ from the oracle's bits (max |diff| {float(err.max()):.3g})"


def _check_id(got_id, want_id, got, want, what):
    """Equal argmax, with the evidence printed when they differ: both ids'
    logits on each side and the largest logit difference."""
    if got_id == want_id:
        return
    err = float(np.abs(got - want).max())
    top = np.argsort(want)[-3:][::-1]
    raise AssertionError(
        f"{what}: argmax {got_id} vs oracle {want_id}; oracle logits [{want_id}]={want[want_id]:.9g} "
        f"[{got_id}]={want[got_id]:.9g} (gap {want[want_id] - want[got_id]:.3g}); engine [{want_id}]={got[want_id]:.9g} "
        f"[{got_id}]={got[got_id]:.9g}; max |logit diff| {err:.3g}; oracle top-3 {top.tolist()} "
        f"{[float(want[i]) for i in top]}")


def _open(q, max_position, pool_bytes):
    import pyoracle

    d = synth.ensure("bench", q)
    cfg = config.load(d)
    rt = Runtime.load(d, LoadOptions(quantization=q, max_position=max_position, kv_pool_bytes=pool_bytes))
    orc = pyoracle.OracleModel(os.path.join(d, f"model-{q}.gguf"), cfg)
    return cfg, rt, orc


@pytest.mark.parametrize("q", ["q4", "q6", "q8"])
def test_64_sequences_bench_model_vs_oracle(q):
    """configs[3]-shaped step on the benchmark decoder: 64 sequences whose
    caches span the attention paths (33 positions: first long cache; 1,024 /
    1,025: the 64-page segment rule; 4,095; lengths with and without a
    16-position tail), stepped together three times; every sequence's logits
    within tolerance of the oracle's and its argmax equal."""
    _need_gpu()
    rng = np.random.default_rng(2)
    n = 64
    lens = rng.integers(256, 1100, size=n).tolist()
    lens[:8] = [4095, 2050, 1024, 1025, 33, 47, 512, 767]
    pool_bytes = (sum(lens) + 16 * n + 64 * 16) * KV_BYTES_PER_POSITION + (64 << 20)
    cfg, rt, orc = _open(q, 4608, pool_bytes)
    if q != "q8":
        # one launch of the batched tensor-core kernel for all 64 sequences
        assert rt.step_io_bytes(n)[1] == 4 * n + 4
    kp, vp = _kv_pool(cfg, max(lens), 7)
    seqs, oseqs = [], []
    for j, L in enumerate(lens):
        k, v = _window(kp, L, 131 * j), _window(vp, L, 131 * j)
        s = rt.new_sequence(L + 8)
        s.import_kv(k, v)
        o = orc.new_seq(L + 8)
        o.import_kv(k, v)
        seqs.append(s)
        oseqs.append(o)
    del kp, vp
    toks = [int(t) for t in rng.integers(0, cfg.vocab_size, size=n)]
    for step in range(3):
        ids, logits = rt.step(seqs, ids=toks, return_logits=True)
        for j in range(n):
            otok, olog, _ = oseqs[j].forward(orc.embed(toks[j]), lens[j] + step, need_logits=True, want_logits=True)
            what = f"{q} step {step} seq {j} (context {lens[j] + step})"
            _check_logits(logits[j], olog, what)
            _check_id(int(ids[j]), otok, logits[j], olog, what)
        toks = [int(i) for i in ids]
    rt.close()
    orc.close()


@pytest.mark.parametrize("q,n0", [("q4", 4096), ("q8", 8448)])
def test_long_context_bench_model_vs_oracle(q, n0):
    """One sequence at 4,096 (configs[3]'s longest) and 8,448 (configs[4]'s
    longest: an 8,192-token prompt plus 256 new) cached positions, restored
    from seeded K/V: four steps, logits within tolerance and argmax equal."""
    _need_gpu()
    cfg, rt, orc = _open(q, n0 + 64, (n0 + 64) * KV_BYTES_PER_POSITION + (64 << 20))
    kp, vp = _kv_pool(cfg, n0, 11)
    s = rt.new_sequence(n0 + 8)
    s.import_kv(kp, vp)
    o = orc.new_seq(n0 + 8)
    o.import_kv(kp, vp)
    del kp, vp
    tok = 4242
    for step in range(4):
        ids, logits = rt.step([s], ids=[tok], return_logits=True)
        otok, olog, _ = o.forward(orc.embed(tok), n0 + step, need_logits=True, want_logits=True)
        _check_logits(logits[0], olog, f"{q} context {n0 + step}")
        _check_id(int(ids[0]), otok, logits[0], olog, f"{q} context {n0 + step}")
        tok = otok
    rt.close()
    orc.close()


def test_q6_image_prompt_configs2_shape():
    """configs[2]'s decode shape on the Q6 benchmark decoder: one image
    placeholder expanded to 1,225 embedding rows (a 1x70x70 patch grid with
    a 2x2 merge, as a 980x980 page gives), 16 text ids, the sectioned M-RoPE
    positions of multimodalPositionsInto (model.go:1717-1783) for the
    prefill and len - 1 + delta for generated tokens; 32 greedy ids equal to
    the oracle's."""
    _need_gpu()
    cfg, rt, orc = _open("q6", 4096, 2 << 30)
    image_token = 100295
    for c in (cfg, rt.cfg):
        c.image_token_id = image_token
        c.spatial_merge_size = 2
    grid = [1, 70, 70]
    rng = np.random.default_rng(1)
    emb = (0.05 * rng.standard_normal((1225, cfg.hidden_size))).astype(np.float32)
    text = synth.random_prompt(16, cfg.vocab_size, 1)
    ids = text[:4] + [image_token] + text[4:]
    got = rt.generate_with_image_embeds(ids, emb, grid, GenerateOptions(max_new_tokens=32, eos_token_ids=[]))
    inp = expand_single_image_placeholder(ids, len(emb), image_token)
    pos, delta = multimodal_positions(inp, grid, image_token, 2)
    assert len(inp) == 1241 and got.prompt_tokens == 1241
    assert len({p for p in pos[4:1229]}) == 1225 and delta != 0  # distinct (t, h, w) per patch
    seq = orc.new_seq(len(inp) + 32)
    cur = 0
    tok = -1
    for i, t in enumerate(inp):
        e = emb[cur] if t == image_token else orc.embed(t)
        cur += t == image_token
        tok, _, _ = seq.forward(e, pos[i], need_logits=i == len(inp) - 1)
    want = list(inp)
    for i in range(32):
        want.append(tok)
        if i + 1 >= 32:
            break
        p = len(want) - 1 + delta
        tok, _, _ = seq.forward(orc.embed(tok), (p, p, p), need_logits=True)
    assert got.tokens == want
    rt.close()
    orc.close()
