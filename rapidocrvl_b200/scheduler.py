"""Continuous batching of independent requests on one GPU.

The reference serves concurrent requests by running each one's own
``Generate`` on a bounded number of inference slots (runSlots,
cmd/paddleocrvl-server/main.go:397, 493-498; its batcher coalesces requests
but still runs them one by one, 507-531).  Here the live requests of a GPU
step together: every decode step runs all of them in one ``ocrvl_step`` call
(up to 64 sequences, the batched tensor-core kernel for Q4/Q6), a finished
request leaves at once and a waiting one takes its place (its prefill runs
before the step it joins).  Greedy decoding with a fixed number of new
tokens per request (no EOS stop), as the throughput benchmark asks.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional


@dataclass
class Request:
    index: int           # caller's request id
    prompt_tokens: int   # positions the prefill leaves in the cache
    max_new_tokens: int
    first_token: int     # input id of the first decode step (the prompt's last token)


@dataclass
class _Live:
    req: Request
    seq: object
    tok: int
    out: List[int] = field(default_factory=list)


@dataclass
class BatchStats:
    steps: int = 0
    tokens: int = 0
    step_ms: float = 0.0          # summed device time of the decode steps (CUDA events)
    kv_positions_read: int = 0    # sum over steps and live sequences of the attended positions
    batch_sizes: List[int] = field(default_factory=list)


def run(rt, requests: List[Request], prefill: Callable[[object, Request], None], max_live: int = 64,
        stream=None, on_finish: Optional[Callable[[Request, List[int]], None]] = None) -> BatchStats:
    """Decodes every request with at most ``max_live`` live sequences.
    ``prefill(seq, req)`` fills a fresh sequence's cache with the request's
    prompt (untimed); each decode step is timed with CUDA events on
    ``stream`` (the engine's stream) when given.  Returns the step statistics;
    ``on_finish`` receives each request's generated ids."""
    import torch

    if not 1 <= max_live <= 64:
        raise ValueError("max_live must be 1..64")
    waiting = list(requests)
    live: List[_Live] = []
    stats = BatchStats()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    while waiting or live:
        while waiting and len(live) < max_live:
            r = waiting.pop(0)
            s = rt.new_sequence(r.prompt_tokens + r.max_new_tokens + 1)
            prefill(s, r)
            live.append(_Live(r, s, r.first_token))
        seqs = [x.seq for x in live]
        ctx = sum(len(s) + 1 for s in seqs)
        if stream is not None:
            ev0.record(stream)
        ids, _ = rt.step(seqs, ids=[x.tok for x in live])
        if stream is not None:
            ev1.record(stream)
            ev1.synchronize()
            stats.step_ms += ev0.elapsed_time(ev1)
        stats.steps += 1
        stats.tokens += len(live)
        stats.kv_positions_read += ctx
        stats.batch_sizes.append(len(live))
        still: List[_Live] = []
        for x, t in zip(live, ids):
            x.out.append(int(t))
            x.tok = int(t)
            if len(x.out) >= x.req.max_new_tokens:
                if on_finish:
                    on_finish(x.req, x.out)
                x.seq.close()
            else:
                still.append(x)
        live = still
    return stats


def summarize(stats: BatchStats) -> Dict[str, float]:
    n = max(1, len(stats.batch_sizes))
    return {"steps": stats.steps, "tokens": stats.tokens, "mean_batch": stats.tokens / n,
            "step_ms_total": stats.step_ms}
