"""Device sampling (ocrvl_op_sample, ocrvl_step_sample, ocrvl_generate)
against the CPU oracle's restatement of the reference's generation-loop
sampler: the same logits and fastRNG seeds give the same ids, candidates and
advanced RNG states, bit for bit."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import pyoracle  # noqa: E402
from rapidocrvl_b200 import GenerateOptions, LoadOptions, Runtime, _lib, config, synth  # noqa: E402

MASK64 = 0xFFFFFFFFFFFFFFFF


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return C.c_void_p(t.data_ptr())


def _device_sample(logits, temp, k, seeds, cands=False):
    torch = _torch()
    m, V = logits.shape
    x = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    st = torch.from_numpy(np.array([s & MASK64 for s in seeds], np.uint64).view(np.int64)).cuda()
    out = torch.full((m,), -7, dtype=torch.int32, device="cuda")
    kk = k if 1 < k < V else 0
    ci = torch.zeros((m, max(kk, 1)), dtype=torch.int32, device="cuda") if cands and kk else None
    cs = torch.zeros((m, max(kk, 1)), dtype=torch.float32, device="cuda") if cands and kk else None
    full = temp > 0 and k != 1 and not (1 < k < V)
    work = torch.zeros((m, V), dtype=torch.float32, device="cuda") if full else None
    _lib.check(_lib.load().ocrvl_op_sample(m, V, _p(x), float(temp), int(k), _p(st), _p(out),
                                           None if ci is None else _p(ci), None if cs is None else _p(cs),
                                           None if work is None else _p(work), None))
    torch.cuda.synchronize()
    states = st.cpu().numpy().view(np.uint64)
    return (out.cpu().numpy(), states, None if ci is None else ci.cpu().numpy(),
            None if cs is None else cs.cpu().numpy())


def _oracle_row(row, temp, k, seed):
    r = pyoracle.RNG(seed)
    tok = pyoracle.sample_token(row, temp, k, r)
    return tok, r.state


def _check(logits, temp, k, seeds, cands=True):
    ids, states, ci, cs = _device_sample(logits, temp, k, seeds, cands)
    for i, row in enumerate(logits):
        tok, st = _oracle_row(row, temp, k, seeds[i])
        assert int(ids[i]) == tok, (i, temp, k, int(ids[i]), tok)
        assert int(states[i]) == st, (i, temp, k)
        if ci is not None:
            want_ids, want_sc = pyoracle.topk_select(row, k)
            assert np.array_equal(ci[i], want_ids), (i, k)
            assert np.array_equal(cs[i].view(np.uint32), want_sc.view(np.uint32)), (i, k)


@pytest.mark.parametrize("V", [1000, 103424])
@pytest.mark.parametrize("k", [2, 3, 4, 5, 8, 9, 64, 999])
@pytest.mark.parametrize("temp", [0.7, 1.0, 1.3])
def test_topk_matches_oracle(V, k, temp):
    rng = np.random.default_rng(V + k)
    m = 8
    logits = (rng.standard_normal((m, V)) * 2.5).astype(np.float32)
    seeds = [int(s) for s in rng.integers(-(1 << 63), (1 << 63) - 1, m, dtype=np.int64)]
    _check(logits, temp, k, seeds)


def test_topk_largest_k():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((2, 103424)).astype(np.float32)
    _check(logits, 0.9, 4096, [11, 12])


@pytest.mark.parametrize("k", [3, 17, 300])
def test_topk_ties_go_to_the_lower_id(k):
    rng = np.random.default_rng(k)
    m, V = 6, 5000
    logits = (np.round(rng.standard_normal((m, V)) * 2) / 2).astype(np.float32)  # few distinct values
    logits[0, ::7] = 0.0
    logits[0, 3::7] = -0.0  # -0 ties with +0
    logits[1, :] = 1.0  # every logit equal
    _check(logits, 1.0, k, list(range(100, 100 + m)))
    _check(logits, 0.8, k, list(range(200, 200 + m)))


@pytest.mark.parametrize("V", [16, 1024, 4096, 4112, 103424])
@pytest.mark.parametrize("temp", [0.5, 1.0, 1.7])
def test_full_vocabulary_matches_oracle(V, temp):
    rng = np.random.default_rng(V)
    m = 8
    logits = (rng.standard_normal((m, V)) * 2).astype(np.float32)
    logits[1] = -50.0  # flat row
    logits[2, V // 3] = 40.0  # one dominant token
    logits[3] = np.linspace(0.0, -300.0, V, dtype=np.float32)  # exp scales past 2^-127: weights the
    # reference's vector exp wraps to negative values, so the binary search meets a non-monotone sum
    seeds = [int(s) for s in rng.integers(0, 1 << 62, m)]
    _check(logits, temp, 0, seeds, cands=False)
    _check(logits, temp, V, seeds, cands=False)  # top_k >= vocab is the full path too


def test_argmax_takes_the_first_maximum_and_no_draw():
    logits = np.zeros((3, 300), np.float32)
    logits[0, [7, 90]] = 5.0
    logits[1, 299] = 1.0
    logits[2, :] = -1.0
    for temp, k in ((0.0, 40), (0.7, 1)):
        ids, states, _, _ = _device_sample(logits, temp, k, [1, 2, 3])
        assert ids.tolist() == [7, 299, 0] and states.tolist() == [1, 2, 3]


def _pair(kind, q):
    d = synth.ensure(kind, q)
    cfg = config.load(d)
    rt = Runtime.load(d, LoadOptions(quantization=q, max_position=4096, kv_pool_bytes=1 << 28))
    orc = pyoracle.OracleModel(os.path.join(d, f"model-{q}.gguf"), cfg)
    return cfg, rt, orc


@pytest.mark.parametrize("kind,q,temp,k,seed", [
    ("tiny", "q8", 0.8, 20, 7),
    ("tiny", "q4", 1.0, 5, -3),
    ("tiny", "q6", 1.2, 3, 99),
    ("tiny-v1024", "q8", 0.9, 0, 3),
    ("tiny-v1024", "q4", 1.0, 0, 12345),
])
def test_generate_sampled_matches_oracle(kind, q, temp, k, seed):
    _torch()
    cfg, rt, orc = _pair(kind, q)
    ids = synth.random_prompt(9, cfg.vocab_size, seed & 0xFFFF)
    opts = GenerateOptions(max_new_tokens=40, temperature=temp, top_k=k, seed=seed, eos_token_ids=[])
    got = rt.generate_with_options(ids, opts)
    want = orc.generate_sampled(ids, 40, temp, k, seed, eos=[])
    assert got.tokens == want
    assert got.tokens != orc.generate(ids, 40, eos=[]) or k == 1  # it did sample


def test_full_vocabulary_generation_needs_whole_blocks():
    _torch()
    cfg, rt, _ = _pair("tiny", "q8")  # vocab 1000
    with pytest.raises(_lib.OcrvlError, match="multiple of 16"):
        rt.generate_with_options([5, 6], GenerateOptions(max_new_tokens=3, temperature=1.0, top_k=0))


@pytest.mark.parametrize("q,n", [("q8", 3), ("q4", 10), ("q8", 10)])
def test_step_sample_batch_matches_oracle(q, n):
    """n sequences, each with its own RNG; n > 8 is one batched launch for
    Q4 and two launches (8 + 2, each drawing with its own RNG states) for Q8."""
    _torch()
    cfg, rt, orc = _pair("tiny", q)
    seqs = [rt.new_sequence(64) for _ in range(n)]
    oseqs = [orc.new_seq(64) for _ in range(n)]
    seeds = [1000 + 17 * i for i in range(n)]
    states = np.array(seeds, np.uint64)
    orngs = [pyoracle.RNG(s) for s in seeds]
    toks = [int(t) for t in synth.random_prompt(n, cfg.vocab_size, 4)]
    for p in range(12):
        got = rt.step_sample(seqs, ids=toks, temperature=0.9, top_k=7, rng_states=states)
        want = []
        for i in range(n):
            _, logits, _ = oseqs[i].forward(orc.embed(toks[i]), p, need_logits=True, want_logits=True)
            want.append(pyoracle.sample_token(logits, 0.9, 7, orngs[i]))
        assert got.tolist() == want, p
        assert [int(s) for s in states] == [r.state for r in orngs]
        toks = want
