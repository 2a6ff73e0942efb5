"""The sampler of the generation loop on the CPU oracle (the checker of the
device sampler): the reference's own sampling tests
(internal/model/sampling_test.go) as known answers, the fastRNG stream,
sampling distributions, and the host-side choice of sampler
(model.go:1846-1868)."""
import ctypes as C

import numpy as np
import pytest

import pyoracle
from rapidocrvl_b200 import _lib
from rapidocrvl_b200.runtime import (GenerateOptions, generation_needs_sampling, generation_uses_argmax,
                                     sampling_rng_state)

MASK64 = 0xFFFFFFFFFFFFFFFF


def splitmix64(state):
    """fastRNG.Float64 (model.go:1833-1840) in Python integers: (u, state)."""
    state = (state + 0x9E3779B97F4A7C15) & MASK64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    z ^= z >> 31
    return (z >> 11) * 2.0 ** -53, state


def test_rng_first_output_is_splitmix64():
    # splitmix64 from state 0 first returns 0xe220a8397b1dcdaf (its published
    # first output); Float64 keeps the top 53 bits
    r = pyoracle.RNG(0)
    assert r.float64() == (0xE220A8397B1DCDAF >> 11) * 2.0 ** -53
    assert r.state == 0x9E3779B97F4A7C15


@pytest.mark.parametrize("seed", [0, 1, 42, -1, -(1 << 63), (1 << 63) - 1])
def test_rng_stream_matches_python_restatement(seed):
    r = pyoracle.RNG(seed)
    st = seed & MASK64
    for _ in range(64):
        u, st = splitmix64(st)
        assert r.float64() == u and r.state == st
        assert 0.0 <= u < 1.0


def test_topk_candidates_sorted():
    # TestTopKCandidatesSorted / TestTopKCandidatesUnsortedContainsTopK
    ids, sc = pyoracle.topk_select([0.5, 9, -1, 7, 3, 8, 2], 3)
    assert ids.tolist() == [1, 5, 3] and sc.tolist() == [9, 8, 7]


def test_topk_sorts_all_and_breaks_ties_by_id():
    # TestSortTokenScoresDescSmall, TestRankedCandidatesTopKZeroSortsAll
    assert pyoracle.topk_select([0.5, 3, -1, 2], 4)[0].tolist() == [1, 3, 0, 2]
    assert pyoracle.topk_select([2, 5, 1], 3)[0].tolist() == [1, 0, 2]
    # topKSelectWithWork: equal scores go to the lower id; -0 equals +0
    ids, _ = pyoracle.topk_select(np.array([1, 3, 3, 0.0, -0.0, 3, 0.0], np.float32), 6)
    assert ids.tolist() == [1, 2, 5, 0, 3, 4]


def test_pick_cumulative_float32():
    # TestPickCumulativeFloat32
    cdf = [0.25, 0.75, 1.0]
    for pick, want in ((0.01, 0), (0.25, 0), (0.26, 1), (0.75, 1), (0.90, 2)):
        assert pyoracle.pick_cumulative(cdf, pick) == want
    assert pyoracle.pick_cumulative(cdf, 1.1) == -1


def test_top_k_one_and_zero_temperature_use_argmax():
    # TestSampleTopKOneUsesArgmax
    r = pyoracle.RNG(1)
    assert pyoracle.sample_token([-1, 3, 2], 1.0, 1, r) == 1
    assert pyoracle.sample_token([-1, 3, 3, 2], 0.0, 5, r) == 1  # first maximum
    assert r.state == 1  # no draw


def test_sampled_ids_are_valid_and_draw_once():
    # TestSampleFullLogitsReturnsValidID / ...TemperatureScaleReturnsValidID
    # (full-vocabulary rows of 16: whole 16-float blocks)
    logits = np.full(16, -100.0, np.float32)
    logits[2] = 0
    for temp in (0.5, 0.8, 1.0, 1.5):
        for seed in range(8):
            r = pyoracle.RNG(seed)
            got = pyoracle.sample_token(logits, temp, 0, r)
            assert 0 <= got < 16
            assert r.state == (seed + 0x9E3779B97F4A7C15) & MASK64
    x = np.array([0.5, 9, -1, 7, 3, 8, 2], np.float32)
    for k in (2, 3, 4, 5, 6):
        r = pyoracle.RNG(3)
        got = pyoracle.sample_token(x, 0.8, k, r)
        assert got in pyoracle.topk_select(x, k)[0].tolist()
        assert r.state == (3 + 0x9E3779B97F4A7C15) & MASK64


def test_full_vocabulary_needs_whole_16_float_blocks():
    r = pyoracle.RNG(0)
    assert pyoracle.sample_token(np.zeros(1000, np.float32), 1.0, 0, r) == -2
    assert pyoracle.sample_token(np.zeros(1024, np.float32), 1.0, 0, r) in range(1024)


def _softmax(x, t):
    z = np.asarray(x, np.float64) / t
    z = np.exp(z - z.max())
    return z / z.sum()


@pytest.mark.parametrize("temp,k", [(1.0, 3), (0.7, 4), (1.0, 6), (1.3, 8), (0.5, 12)])
def test_topk_draws_follow_the_softmax(temp, k):
    rng = np.random.default_rng(k)
    logits = rng.standard_normal(200).astype(np.float32)
    ids, sc = pyoracle.topk_select(logits, k)
    p = _softmax(sc, temp)
    n = 20000
    r = pyoracle.RNG(12345)
    counts = {int(i): 0 for i in ids}
    for _ in range(n):
        counts[pyoracle.sample_candidates(ids, sc, temp, r)] += 1
    freq = np.array([counts[int(i)] for i in ids]) / n
    assert np.all(np.abs(freq - p) <= 4 * np.sqrt(p * (1 - p) / n) + 1e-3), (freq, p)


@pytest.mark.parametrize("temp", [0.6, 1.0, 1.4])
def test_full_vocabulary_draws_follow_the_softmax(temp):
    rng = np.random.default_rng(7)
    for n_vocab in (64, 4160):  # one cumulative chain; four blocks
        logits = rng.standard_normal(n_vocab).astype(np.float32)
        logits[:8] += 3.0
        p = _softmax(logits, temp)
        n = 8000
        r = pyoracle.RNG(99)
        counts = np.zeros(n_vocab)
        for _ in range(n):
            counts[pyoracle.sample_full(logits, temp, r)] += 1
        top = np.argsort(-p)[:8]
        freq = counts[top] / n
        assert np.all(np.abs(freq - p[top]) <= 4 * np.sqrt(p[top] * (1 - p[top]) / n) + 2e-3), (freq, p[top])


def test_sampling_rng_only_when_needed():
    # TestSamplingRNGOnlyWhenNeeded
    assert not generation_needs_sampling(GenerateOptions(max_new_tokens=1, temperature=0))
    assert not generation_needs_sampling(GenerateOptions(max_new_tokens=1, temperature=1, top_k=1))
    assert not generation_needs_sampling(GenerateOptions(max_new_tokens=0, temperature=1))
    assert generation_needs_sampling(GenerateOptions(max_new_tokens=1, temperature=1))
    assert generation_uses_argmax(GenerateOptions(temperature=0.0, top_k=40))
    assert generation_uses_argmax(GenerateOptions(temperature=0.9, top_k=1))
    assert sampling_rng_state(GenerateOptions(max_new_tokens=1, temperature=1, seed=-1)) == MASK64
    assert sampling_rng_state(GenerateOptions(max_new_tokens=1, temperature=0, seed=5)) is None


def test_abi_sampler_rejects_bad_arguments():
    """Argument checks that run before any device work."""
    L = _lib.load()
    st = (C.c_uint64 * 1)(0)
    out = (C.c_int32 * 1)(0)
    dummy = C.c_void_p(16)  # never dereferenced: each call fails validation first
    E = _lib.E_INVALID
    assert L.ocrvl_op_sample(0, 100, dummy, 1.0, 5, st, out, None, None, None, None) == E
    assert L.ocrvl_op_sample(1, 1, dummy, 1.0, 5, st, out, None, None, None, None) == E
    assert L.ocrvl_op_sample(1, 100, None, 1.0, 5, st, out, None, None, None, None) == E
    assert L.ocrvl_op_sample(1, 100, dummy, float("nan"), 5, st, out, None, None, None, None) == E
    assert L.ocrvl_op_sample(1, 100, dummy, 1.0, -1, st, out, None, None, None, None) == E
    assert L.ocrvl_op_sample(1, 10000, dummy, 1.0, 4097, st, out, None, None, None, None) == E  # top_k cap
    assert L.ocrvl_op_sample(1, 1000, dummy, 1.0, 0, st, out, None, None, dummy, None) == E  # 1000 % 16
    assert L.ocrvl_op_sample(1, 1024, dummy, 1.0, 0, st, out, None, None, None, None) == E  # no work
    assert L.ocrvl_op_sample(1, 1024, dummy, 1.0, 5, None, out, None, None, None, None) == E  # no rng
    assert L.ocrvl_op_sample(1, 1024, dummy, 1.0, 0, st, out, dummy, None, dummy, None) == E  # candidates
    assert "multiple of 16" in _lib.last_error() or "candidates" in _lib.last_error()
    assert L.ocrvl_step_sample(None, None, 1, None, None, None, 1.0, 5, st, out) == E
    n = C.c_int(0)
    assert L.ocrvl_generate(None, None, 0, 1, None, 0, 1.0, 5, 0, out, 1, C.byref(n)) == E
