"""Decode-step parity of the CUDA engine against the CPU oracle on seeded
synthetic decoders (tolerance from the spec: logits within 2e-2 absolute or
1e-2 relative; greedy ids equal; KV append bit-exact)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rapidocrvl_b200 import GenerateOptions, LoadOptions, Runtime, config, synth  # noqa: E402

LOGIT_ATOL = 2e-2
LOGIT_RTOL = 1e-2


def _need_gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _pair(model_dir, q):
    import pyoracle

    cfg = config.load(model_dir)
    rt = Runtime.load(model_dir, LoadOptions(quantization=q, max_position=4096, kv_pool_bytes=1 << 28))
    orc = pyoracle.OracleModel(os.path.join(model_dir, f"model-{q}.gguf"), cfg)
    return cfg, rt, orc


@pytest.mark.parametrize("q", ["q8", "q6", "q4"])
def test_greedy_ids_match_oracle(tiny_models, q):
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models[q], q)
    ids = synth.random_prompt(12, cfg.vocab_size, 0)
    got = rt.generate_with_options(ids, GenerateOptions(max_new_tokens=70, eos_token_ids=[]))
    want = orc.generate(ids, 70, eos=[])
    assert got.prompt_tokens == 12
    assert got.tokens == want


@pytest.mark.parametrize("q", ["q8", "q4"])
def test_stepwise_logits_and_kv(tiny_models, q):
    """Token-by-token: logits within tolerance, argmax equal, KV compared."""
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models[q], q)
    seq = rt.new_sequence(128)
    oseq = orc.new_seq(128)
    tok = 5
    worst = 0.0
    for p in range(80):  # crosses n = 6/7, 16 (softmax tail rule), 64 (two value chunks) and page edges
        ids, logits = rt.step([seq], ids=[tok], need_logits=True, return_logits=True)
        otok, ologits, _ = oseq.forward(orc.embed(tok), p, need_logits=True, want_logits=True)
        err = np.abs(logits[0] - ologits)
        worst = max(worst, float(err.max()))
        assert np.all(err <= LOGIT_ATOL + LOGIT_RTOL * np.abs(ologits)), f"pos {p}: max err {err.max()}"
        assert int(ids[0]) == otok, f"pos {p}: argmax {ids[0]} vs {otok}"
        if p == 0:
            for layer in range(cfg.num_hidden_layers):
                k, v = seq.read_kv(layer)
                ok, ov = oseq.kv(layer)
                assert np.array_equal(k, ok) and np.array_equal(v, ov), "first append must be bit-exact"
        tok = int(ids[0])
    assert len(seq) == 80
    for layer in range(cfg.num_hidden_layers):
        k, v = seq.read_kv(layer)
        ok, ov = oseq.kv(layer)
        assert k.shape == ok.shape
        np.testing.assert_allclose(k, ok, rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(v, ov, rtol=1e-3, atol=1e-4)


def test_prompt_steps_without_logits(tiny_models):
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models["q4"], "q4")
    seq = rt.new_sequence(64)
    oseq = orc.new_seq(64)
    prompt = synth.random_prompt(20, cfg.vocab_size, 3)
    for p, t in enumerate(prompt):
        last = p == len(prompt) - 1
        ids, _ = rt.step([seq], ids=[t], need_logits=last)
        otok, _, _ = oseq.forward(orc.embed(t), p, need_logits=last)
        if not last:
            assert int(ids[0]) == -1
    assert int(ids[0]) == otok


def test_batched_step_equals_single(tiny_models):
    """Sequences stepped together give the same bits as stepped alone."""
    _need_gpu()
    cfg, rt, _ = _pair(tiny_models["q8"], "q8")
    prompts = [synth.random_prompt(n, cfg.vocab_size, n) for n in (3, 9, 21)]

    def run(batched):
        seqs = [rt.new_sequence(64) for _ in prompts]
        outs = [[] for _ in prompts]
        steps = max(len(p) for p in prompts) + 10
        toks = [p[0] for p in prompts]
        for i in range(steps):
            live = [j for j in range(len(prompts))]
            if batched:
                ids, logits = rt.step([seqs[j] for j in live], ids=[toks[j] for j in live], return_logits=True)
            else:
                res = [rt.step([seqs[j]], ids=[toks[j]], return_logits=True) for j in live]
                ids = np.array([r[0][0] for r in res])
                logits = np.stack([r[1][0] for r in res])
            for j in live:
                outs[j].append(logits[j])
                nxt = i + 1
                toks[j] = prompts[j][nxt] if nxt < len(prompts[j]) else int(ids[j])
        return outs

    a, b = run(True), run(False)
    for j in range(len(prompts)):
        for x, y in zip(a[j], b[j]):
            assert np.array_equal(x, y)


@pytest.mark.parametrize("q", ["q4", "q8"])
def test_many_sequences_step_equals_single(tiny_models, q):
    """A step over more sequences than one launch takes (20 here, 64 at most)
    gives each sequence the same ids and logits, bit for bit, as stepping it
    alone; the device-fed loop over 12 sequences matches too."""
    _need_gpu()
    cfg, rt, _ = _pair(tiny_models[q], q)
    n = 20
    prompts = [synth.random_prompt(4 + (j % 5), cfg.vocab_size, 100 + j) for j in range(n)]
    seq_a = [rt.new_sequence(48) for _ in range(n)]
    seq_b = [rt.new_sequence(48) for _ in range(n)]
    # prefill each sequence alone (different lengths), then one joint step
    last = []
    for j in range(n):
        for t in prompts[j][:-1]:
            rt.step([seq_a[j]], ids=[t], need_logits=False)
            rt.step([seq_b[j]], ids=[t], need_logits=False)
        last.append(prompts[j][-1])
    ids_joint, logits_joint = rt.step(seq_a, ids=last, return_logits=True)
    for j in range(n):
        ids1, logits1 = rt.step([seq_b[j]], ids=[last[j]], return_logits=True)
        assert int(ids1[0]) == int(ids_joint[j])
        assert np.array_equal(logits1[0], logits_joint[j])
    # device-fed loop, 12 sequences at once vs one at a time
    first = [int(i) for i in ids_joint[:12]]
    dev_joint = rt.decode_device(seq_a[:12], first, 5)
    for j in range(12):
        dev1 = rt.decode_device([seq_b[j]], [first[j]], 5)
        assert dev1[:, 0].tolist() == dev_joint[:, j].tolist()
    with pytest.raises(Exception):
        rt.step([rt.new_sequence(4) for _ in range(65)], ids=[1] * 65)


@pytest.mark.parametrize("q", ["q4", "q6"])
def test_batched_64_sequences_tensor_core_step(tiny_models, q):
    """64 sequences with caches past one chunk (the batched kernel: int8
    tensor-core GEMMs) give the same ids and logits, bit for bit, as each
    sequence stepped alone, for three steps in a row."""
    _need_gpu()
    cfg, rt, _ = _pair(tiny_models[q], q)
    n = 64
    # one launch for all 64 (ids of 64 sequences + one status word come back)
    assert rt.step_io_bytes(n)[1] == 4 * n + 4
    lens = [33 + (j * 7) % 20 for j in range(n)]
    prompts = [synth.random_prompt(lens[j], cfg.vocab_size, 500 + j) for j in range(n)]
    seq_a = [rt.new_sequence(80) for _ in range(n)]
    seq_b = [rt.new_sequence(80) for _ in range(n)]
    toks = []
    for j in range(n):
        # prefill through the batched path too: all prompts of one length step together
        for t in prompts[j][:-1]:
            rt.step([seq_b[j]], ids=[t], need_logits=False)
        toks.append(prompts[j][-1])
    for p in range(max(lens) - 1):
        live = [j for j in range(n) if p < lens[j] - 1]
        rt.step([seq_a[j] for j in live], ids=[prompts[j][p] for j in live], need_logits=False)
    for step in range(3):
        ids_joint, logits_joint = rt.step(seq_a, ids=toks, return_logits=True)
        for j in range(n):
            ids1, logits1 = rt.step([seq_b[j]], ids=[toks[j]], return_logits=True)
            assert int(ids1[0]) == int(ids_joint[j]), (step, j)
            assert np.array_equal(logits1[0], logits_joint[j]), (step, j)
        toks = [int(i) for i in ids_joint]


@pytest.mark.parametrize("q", ["q4", "q8"])
def test_long_caches_more_items_than_blocks(tiny_models, q):
    """8 sequences whose chunked attention has more items than the grid has
    blocks (each block then takes several items, with K/V copies started
    before the phase), through prompt steps (append only in the last layer)
    and full steps: ids and logits equal to each sequence stepped alone."""
    _need_gpu()
    cfg, rt, _ = _pair(tiny_models[q], q)
    n = 8
    lens = [150 + 9 * j for j in range(n)]
    prompts = [synth.random_prompt(L, cfg.vocab_size, 900 + j) for j, L in enumerate(lens)]
    seq_a = [rt.new_sequence(L + 8) for L in lens]
    seq_b = [rt.new_sequence(L + 8) for L in lens]
    for p in range(max(lens) - 1):
        live = [j for j in range(n) if p < lens[j] - 1]
        rt.step([seq_a[j] for j in live], ids=[prompts[j][p] for j in live], need_logits=False)
    for j in range(n):
        for t in prompts[j][:-1]:
            rt.step([seq_b[j]], ids=[t], need_logits=False)
    for j in range(n):
        ka, va = seq_a[j].read_kv(1)
        kb, vb = seq_b[j].read_kv(1)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    toks = [pr[-1] for pr in prompts]
    for step in range(3):
        ids_joint, logits_joint = rt.step(seq_a, ids=toks, return_logits=True)
        for j in range(n):
            ids1, logits1 = rt.step([seq_b[j]], ids=[toks[j]], return_logits=True)
            assert int(ids1[0]) == int(ids_joint[j]) and np.array_equal(logits1[0], logits_joint[j]), (step, j)
        toks = [int(i) for i in ids_joint]


def test_embeds_and_mrope_positions(tiny_models):
    """Embedding input and distinct (T,H,W) positions (image-token prefill)."""
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models["q6"], "q6")
    seq = rt.new_sequence(32)
    oseq = orc.new_seq(32)
    rng = np.random.default_rng(0)
    for p in range(10):
        emb = (rng.standard_normal(cfg.hidden_size) * 0.02).astype(np.float32)
        pos = (p, 3 + p // 3, 5 + p % 3) if p < 8 else (p, p, p)
        ids, logits = rt.step([seq], embeds=emb[None], positions=[pos], return_logits=True)
        otok, ologits, _ = oseq.forward(emb, pos, need_logits=True, want_logits=True)
        assert np.all(np.abs(logits[0] - ologits) <= LOGIT_ATOL + LOGIT_RTOL * np.abs(ologits))
        assert int(ids[0]) == otok


def test_eos_and_edge_lengths(tiny_models):
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models["q4"], "q4")
    ids = synth.random_prompt(4, cfg.vocab_size, 11)
    full = orc.generate(ids, 12, eos=[])
    eos = full[4 + 5]
    got = rt.generate_with_options(ids, GenerateOptions(max_new_tokens=12, eos_token_ids=[eos]))
    assert got.tokens == orc.generate(ids, 12, eos=[eos])
    assert rt.generate(ids, 0) == ids
    assert rt.generate(ids[:1], 1) == orc.generate(ids[:1], 1, eos=[])
    with pytest.raises(ValueError):
        rt.generate([], 3)
    with pytest.raises(ValueError):
        rt.generate([cfg.vocab_size], 3)


def test_step_errors_leave_state_unchanged(tiny_models):
    _need_gpu()
    from rapidocrvl_b200 import _lib

    cfg, rt, _ = _pair(tiny_models["q8"], "q8")
    seq = rt.new_sequence(2)
    rt.step([seq], ids=[1])
    rt.step([seq], ids=[2])
    with pytest.raises(_lib.OcrvlError):
        rt.step([seq], ids=[3])  # full
    assert len(seq) == 2
    seq2 = rt.new_sequence(4)
    with pytest.raises(_lib.OcrvlError):
        rt.step([seq2], ids=[cfg.vocab_size + 5])
    assert len(seq2) == 0


@pytest.mark.slow
@pytest.mark.parametrize("q", ["q4", "q8"])
def test_bench_model_greedy_32(q):
    """Benchmark-size decoder: 32 greedy ids after a 512-token prompt match."""
    _need_gpu()
    d = synth.ensure("bench", q)
    cfg, rt, orc = _pair(d, q)
    ids = synth.random_prompt(512, cfg.vocab_size, 0)
    got = rt.generate_with_options(ids, GenerateOptions(max_new_tokens=32, eos_token_ids=[]))
    want = orc.generate(ids, 32, eos=[])
    assert got.tokens == want


def test_import_kv_restores_a_cache(tiny_models):
    """ocrvl_seq_import_kv: the cache of a prefilled sequence, read back and
    imported into a fresh sequence, reads back unchanged and gives the same
    next step (ids and logits bit for bit); a length beyond the sequence's
    capacity is rejected and leaves it unchanged."""
    _need_gpu()
    from rapidocrvl_b200 import _lib

    cfg, rt, _ = _pair(tiny_models["q4"], "q4")
    prompt = synth.random_prompt(41, cfg.vocab_size, 7)  # 40 cached positions: 3 pages, a long cache
    a = rt.new_sequence(64)
    b = rt.new_sequence(64)
    for t in prompt[:-1]:
        rt.step([a], ids=[t], need_logits=False)
    L = cfg.num_hidden_layers
    kv = [a.read_kv(layer) for layer in range(L)]
    k = np.stack([x[0] for x in kv])
    v = np.stack([x[1] for x in kv])
    b.import_kv(k, v)
    assert len(b) == len(a) == 40
    for layer in range(L):
        kb, vb = b.read_kv(layer)
        assert np.array_equal(kb, k[layer]) and np.array_equal(vb, v[layer])
    ida, la = rt.step([a], ids=[prompt[-1]], return_logits=True)
    idb, lb = rt.step([b], ids=[prompt[-1]], return_logits=True)
    assert int(ida[0]) == int(idb[0])
    assert np.array_equal(la, lb)
    too_long = np.zeros((L, 65, k.shape[2]), np.float32)
    with pytest.raises(_lib.OcrvlError):
        b.import_kv(too_long, too_long)
    assert len(b) == 41  # rejected before any change


def test_caches_over_1024_positions(tiny_models):
    """Caches of more than 64 pages (1,024 positions), which the long-cache
    attention splits into half as many, longer segments: one sequence
    prefilled to 1,100 positions token by token matches the oracle's logits
    and argmax at its next step; 12 sequences of 900-2,100 cached positions
    (seeded K/V imported) stepped together in one batched step get the ids
    and logits of stepping each alone, bit for bit."""
    _need_gpu()
    import pyoracle

    q = "q4"
    cfg = config.load(tiny_models[q])
    rt = Runtime.load(tiny_models[q], LoadOptions(quantization=q, max_position=4096, kv_pool_bytes=1 << 30))
    orc = pyoracle.OracleModel(os.path.join(tiny_models[q], f"model-{q}.gguf"), cfg)
    n0 = 1100
    prompt = synth.random_prompt(n0 + 1, cfg.vocab_size, 31)
    seq = rt.new_sequence(n0 + 8)
    oseq = orc.new_seq(n0 + 8)
    for p, t in enumerate(prompt[:-1]):
        rt.step([seq], ids=[t], need_logits=False)
        oseq.forward(orc.embed(t), p, need_logits=False)
    ids, logits = rt.step([seq], ids=[prompt[-1]], return_logits=True)
    otok, ologits, _ = oseq.forward(orc.embed(prompt[-1]), n0, need_logits=True, want_logits=True)
    err = np.abs(logits[0] - ologits)
    assert np.all(err <= LOGIT_ATOL + LOGIT_RTOL * np.abs(ologits)), f"max err {err.max()}"
    assert int(ids[0]) == otok

    rng = np.random.default_rng(5)
    n = 12
    lens = [900 + 109 * j for j in range(n)]
    kvd = cfg.num_key_value_heads * cfg.head_dim
    L = cfg.num_hidden_layers
    seq_a = [rt.new_sequence(x + 8) for x in lens]
    seq_b = [rt.new_sequence(x + 8) for x in lens]
    for j, x in enumerate(lens):
        k = (0.5 * rng.standard_normal((L, x, kvd))).astype(np.float32)
        v = rng.standard_normal((L, x, kvd)).astype(np.float32)
        seq_a[j].import_kv(k, v)
        seq_b[j].import_kv(k, v)
    toks = [int(t) for t in rng.integers(0, cfg.vocab_size, n)]
    for step in range(2):
        ids_joint, logits_joint = rt.step(seq_a, ids=toks, return_logits=True)
        for j in range(n):
            ids1, logits1 = rt.step([seq_b[j]], ids=[toks[j]], return_logits=True)
            assert int(ids1[0]) == int(ids_joint[j]) and np.array_equal(logits1[0], logits_joint[j]), (step, j)
        toks = [int(i) for i in ids_joint]


def test_fill_synthetic_cache_steps_like_the_oracle(tiny_models):
    """ocrvl_seq_fill_synthetic: seeded device-generated K/V (the same seed
    gives the same cache, values in K [-0.5, 0.5) / V [-1, 1)); the cache read
    back and imported into the oracle gives the engine's next-step logits bit
    for bit, and a refill with another length replaces it."""
    _need_gpu()
    cfg, rt, orc = _pair(tiny_models["q4"], "q4")
    a, b = rt.new_sequence(720), rt.new_sequence(720)
    a.fill_synthetic(700, 99)
    b.fill_synthetic(700, 99)
    L = cfg.num_hidden_layers
    kv = [a.read_kv(layer) for layer in range(L)]
    for layer in range(L):
        kb, vb = b.read_kv(layer)
        assert np.array_equal(kb, kv[layer][0]) and np.array_equal(vb, kv[layer][1])
    k = np.stack([x[0] for x in kv])
    v = np.stack([x[1] for x in kv])
    assert k.shape == (L, 700, cfg.num_key_value_heads * cfg.head_dim)
    assert np.all(np.abs(k) <= 0.5) and np.all(np.abs(v) <= 1.0) and np.std(v) > 0.3
    o = orc.new_seq(720)
    o.import_kv(k, v)
    ids, logits = rt.step([a], ids=[17], return_logits=True)
    otok, olog, _ = o.forward(orc.embed(17), 700, need_logits=True, want_logits=True)
    assert int(ids[0]) == otok and np.array_equal(logits[0], olog)
    a.fill_synthetic(40, 1)
    assert len(a) == 40
