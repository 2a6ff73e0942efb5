"""Continuous batching host logic (rapidocrvl_b200.scheduler) against a fake
runtime on CPU: every request gets its tokens, no more than max_live
sequences step together, a finished request's slot is refilled before the
next step, and each sequence is fed its own previous token."""
import pytest

from rapidocrvl_b200 import scheduler


class _Seq:
    def __init__(self, rt, cap):
        self.rt, self.cap, self.n, self.closed = rt, cap, 0, False

    def __len__(self):
        return self.n

    def close(self):
        self.closed = True
        self.rt.open -= 1


class _Rt:
    def __init__(self):
        self.open = 0
        self.batches = []
        self.fed = {}

    def new_sequence(self, cap):
        self.open += 1
        return _Seq(self, cap)

    def step(self, seqs, ids):
        assert len(seqs) == len(ids) and len(set(map(id, seqs))) == len(seqs)
        self.batches.append(len(seqs))
        out = []
        for s, t in zip(seqs, ids):
            assert not s.closed and s.n < s.cap
            self.fed.setdefault(id(s), []).append(t)
            s.n += 1
            out.append((t * 31 + s.n) % 1000)
        return out, None


@pytest.mark.parametrize("max_live", [1, 3, 64])
def test_continuous_batch(max_live):
    rt = _Rt()
    reqs = [scheduler.Request(i, prompt_tokens=5 + i, max_new_tokens=2 + (i * 7) % 5, first_token=i) for i in range(20)]
    filled, done = [], {}

    def prefill(seq, r):
        seq.n = r.prompt_tokens
        filled.append(r.index)

    st = scheduler.run(rt, reqs, prefill, max_live=max_live, on_finish=lambda r, out: done.setdefault(r.index, out))
    assert sorted(done) == list(range(20)) and filled == list(range(20))
    assert all(len(done[r.index]) == r.max_new_tokens for r in reqs)
    assert st.tokens == sum(r.max_new_tokens for r in reqs) and st.steps == len(rt.batches)
    assert max(rt.batches) <= max_live and rt.open == 0
    # the batch stays full while requests wait
    waiting_full = sum(rt.batches) == st.tokens
    assert waiting_full
    if max_live == 3:
        assert rt.batches[0] == 3
    with pytest.raises(ValueError):
        scheduler.run(rt, reqs, prefill, max_live=65)
