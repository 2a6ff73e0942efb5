"""Failure detection of the step kernel, exercised without faulting the GPU.

Every device-side wait of the persistent step kernels is bounded (grid
barrier polls, mbarrier polls and elapsed time); a wait that runs out sets an
error word, every block leaves after draining its copies in flight, the step
returns OCRVL_E_TIMEOUT, the host resets the barrier state and the sequences
keep their length.  The reference's counterpart is the disable-op-and-report
path of its GPU ops (internal/model/model.go:7235-7285).  Here a test-only
poll limit (ocrvl_set_wait_limit) makes the grid-barrier wait run out; with
the default restored the following steps match the oracle bit for bit."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rapidocrvl_b200 import LoadOptions, Runtime, _lib, config, synth  # noqa: E402

OCRVL_E_TIMEOUT = -4


def _need_gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _limit(rt, polls):
    _lib.check(rt._L.ocrvl_set_wait_limit(rt._h, int(polls)))


@pytest.mark.parametrize("n", [1, 12])
def test_barrier_timeout_reported_and_recovered(tiny_models, n):
    """n = 1: the single-sequence kernel; n = 12: the tcgen05 batched kernel
    (its TMEM is released on the early exit)."""
    _need_gpu()
    import pyoracle

    q = "q4"
    cfg = config.load(tiny_models[q])
    rt = Runtime.load(tiny_models[q], LoadOptions(quantization=q, max_position=1024, kv_pool_bytes=1 << 28))
    orc = pyoracle.OracleModel(os.path.join(tiny_models[q], f"model-{q}.gguf"), cfg)
    seqs = [rt.new_sequence(80) for _ in range(n)]
    oseqs = [orc.new_seq(80) for _ in range(n)]
    prompts = [synth.random_prompt(45, cfg.vocab_size, 40 + j) for j in range(n)]
    for p in range(40):
        rt.step(seqs, ids=[pr[p] for pr in prompts], need_logits=False)
        for j in range(n):
            oseqs[j].forward(orc.embed(prompts[j][p]), p, need_logits=False)
    _limit(rt, 1)
    with pytest.raises(_lib.OcrvlError) as e:
        rt.step(seqs, ids=[pr[40] for pr in prompts])
    assert e.value.code == OCRVL_E_TIMEOUT
    assert all(len(s) == 40 for s in seqs)
    with pytest.raises(_lib.OcrvlError) as e:
        rt.decode_device(seqs, [pr[40] for pr in prompts], 3)
    assert e.value.code == OCRVL_E_TIMEOUT
    assert all(len(s) == 40 for s in seqs)
    _limit(rt, 0)
    for p in range(40, 45):
        ids, logits = rt.step(seqs, ids=[pr[p] for pr in prompts], return_logits=True)
        for j in range(n):
            otok, olog, _ = oseqs[j].forward(orc.embed(prompts[j][p]), p, need_logits=True, want_logits=True)
            assert int(ids[j]) == otok and np.array_equal(logits[j], olog), (p, j)
    with pytest.raises(_lib.OcrvlError):
        _limit(rt, -1)
    rt.close()
    orc.close()
