"""Decode-step benchmark of the B200 engine against BASELINE.json's metric
("decode tokens/s (bs=1 and bs=64, Q4/Q8) and quant-GEMV HBM GB/s").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

One JSON line.  Its headline (``value``, ``e2e``, ``roofline``,
``cpu_baseline``) is configs[1]: the Q4 decoder, batch 1, a 512-token prompt
and K greedy decode tokens (a step is one token).  ``value`` is device-timed
(CUDA events on the engine's stream around K steps of the device-fed decode
loop, inputs resident in HBM); ``e2e`` times the same K tokens through the
reference-facing C ABI (ocrvl_step with host buffers: token in, token out,
one call per token).  Under torchrun each rank decodes its own configs[1]
request on its own GPU (request-parallel replicas, no collective on the data
path); the reported time is the max over ranks.

Further keys of the same line carry the metric's other configurations, each
with its own ms_per_step, roofline and e2e:
  configs0  Q8, batch 1, 32-token prompt, 64 new tokens (1 GPU runs only);
  configs3  Q4, 64 sequences with contexts U[256, 4096] (seed 2), 128 steps
            of one token per sequence (1 GPU runs only);
  configs4  Q8, 512 requests with prompts U[1024, 8192] (seed 3) and 256 new
            tokens each, partitioned over the N GPUs (no collective), each GPU
            running a continuous batch of up to 64 live sequences; value =
            all requests' tokens / max over ranks of the summed step times;
  gemv      quant-GEMV HBM GB/s: the op-level matvec kernel (k_gemv) on
            lm_head-sized matrices (103,424 x 1,024, one input vector) for
            Q4/Q6/Q8 and the row-sum kernel (k_rowsum), each call on another
            of several weight copies (together over twice the L2), CUDA events
            around 20 calls (1 GPU runs only).
Prompt caches of configs3 and configs4 are seeded synthetic K/V written on the
device (the decode time does not depend on the cached values; the reference
prefills token by token, untimed here).

``--impl reference`` times the CPU restatement of the reference's decode path
(oracle/, all host threads) on configs[1] instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (bs=1 and bs=64, Q4/Q8) and quant-GEMV HBM GB/s vs 8 TB/s"
UNIT = "tokens/s"
PROMPT = 512


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--quant", default="q4", choices=["q4", "q6", "q8"])
    ap.add_argument("--prompt", type=int, default=PROMPT)
    ap.add_argument("--workload", default="all", choices=["all", "configs1", "configs0", "configs3", "configs4", "gemv", "sample"],
                    help="all: configs1 headline plus the other configurations' keys; otherwise one of them alone")
    ap.add_argument("--ctx-hi", type=int, default=4096, help="configs3: contexts U[256, ctx_hi] (profiling: smaller)")
    ap.add_argument("--requests", type=int, default=512, help="configs4: requests over all GPUs")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def model_desc(cfg):
    return (f"hidden {cfg.hidden_size}, {cfg.num_hidden_layers} layers, {cfg.num_attention_heads}q/"
            f"{cfg.num_key_value_heads}kv heads, head_dim {cfg.head_dim}, SwiGLU {cfg.intermediate_size}, "
            f"vocab {cfg.vocab_size}")


def workload_config(args, cfg):
    return {
        "workload": f"configs[1]: {args.quant.upper()} decoder ({model_desc(cfg)}), batch 1 per GPU, {args.prompt}-token "
                    f"prompt, {args.warmup}+{args.steps} greedy decode tokens",
        "quant": args.quant,
        "batch_per_gpu": 1,
        "prompt_tokens": args.prompt,
        "context": [args.prompt + args.warmup, args.prompt + args.warmup + args.steps],
        "parallelism": "request-parallel replicas (one sequence per GPU, no collective)",
        "l2": "no flush: per-step working set (all weights + KV) > 126 MB L2",
    }


def algorithmic_bytes(model_dir, quant, cfg):
    """Bytes one decode token streams: rows * (packed row + f32 scale) of every
    quantized matrix incl. lm_head, the 2L+1 f32 norm vectors and one f32
    embedding row; plus K and V (f32, every layer) per attended position."""
    from rapidocrvl_b200 import gguf

    g = gguf.GGUFFile(os.path.join(model_dir, f"model-{quant}.gguf"))
    w = 0
    for name, m in g.tensors.items():
        if m.type in (gguf.Q8_ROW, gguf.Q4_ROW, gguf.Q6_ROW):
            w += int(m.shape[0]) * (gguf.packed_row_bytes(m.type, int(m.shape[1])) + 4)
        elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            w += int(m.shape[0]) * 4
    w += cfg.hidden_size * 4  # embedding row
    kv_tok = cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * cfg.head_dim * 4
    return w, kv_tok


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback"


def roofline(bytes_per_step, ms_per_step, kernel):
    peak, src = hbm_peak()
    achieved = bytes_per_step / (ms_per_step / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": src, "kernel": kernel, "algorithmic_bytes_per_step": bytes_per_step, "traffic": None}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids):
        self.bus = {b.lower()[-12:] for b in bus_ids}
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi's start-up (driver/NVML init) must not fall inside the timed region
            t0 = time.time()
            while self.proc.poll() is None and not self.rows and time.time() - t0 < 20:
                time.sleep(0.05)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10 and parts[1].lower()[-12:] in self.bus:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[6 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def visible_bus_ids(local):
    try:
        r = subprocess.run(["nvidia-smi", "--query-gpu=pci.bus_id", "--format=csv,noheader"], capture_output=True,
                           text=True, timeout=20)
        allb = [x.strip() for x in r.stdout.splitlines() if x.strip()]
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = [int(v) for v in vis.split(",")] if vis else list(range(len(allb)))
        return [allb[idx[local]]] if local < len(idx) and idx[local] < len(allb) else allb[:1]
    except Exception:
        return []


# ---- CPU baseline (the oracle: C++ restatement of the reference CPU path) ---
def cpu_reference_decode(model_dir, quant, cfg, prompt, steps, warmup, budget_s=None):
    """Times the CPU restatement of the reference decode path (oracle/) on all
    host threads (set explicitly: torchrun sets OMP_NUM_THREADS=1 for its
    workers).  Returns (steps, seconds, prefill seconds, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle

    threads = pyoracle.set_threads(host_threads())
    om = pyoracle.OracleModel(os.path.join(model_dir, f"model-{quant}.gguf"), cfg)
    seq = om.new_seq(len(prompt) + warmup + steps + 8)
    t_pre = time.time()
    for p, t in enumerate(prompt):
        tok, _, _ = seq.forward(om.embed(t), p, need_logits=p == len(prompt) - 1)
    t_pre = time.time() - t_pre
    pos = len(prompt)
    tok = seq.decode_steps(tok, pos, warmup) if warmup else tok
    pos += warmup
    if budget_s is not None:
        t0 = time.time()
        tok1 = seq.decode_steps(tok, pos, 1)
        one = time.time() - t0
        pos += 1
        tok = tok1
        steps = max(3, min(steps, int(budget_s / max(one, 1e-4))))
    t0 = time.time()
    seq.decode_steps(tok, pos, steps)
    dt = time.time() - t0
    om.close()
    return steps, dt, t_pre, threads


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from rapidocrvl_b200 import config, synth

    d = synth.ensure("bench", args.quant)
    cfg = config.load(d)
    prompt = synth.random_prompt(args.prompt, cfg.vocab_size, 0)
    steps, dt, t_pre, threads = cpu_reference_decode(d, args.quant, cfg, prompt, args.steps, args.warmup)
    v = steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8/f32",
        "data": "synthetic (seeded N(0,0.02) BF16 weights -> GGUF; uniform prompt ids)",
        "config": workload_config(args, cfg),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{steps} greedy decode steps at context {args.prompt + args.warmup}+ after a "
                                   f"{args.prompt}-token CPU prefill ({t_pre:.1f} s, untimed); C++ restatement of the "
                                   f"reference Go CPU path (no Go toolchain on this image), {threads} OpenMP threads"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU workloads -----------------------------------------------------------
def events():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def bs1_workload(quant, prompt_len, steps, warmup, rank, device, label, clocks_for=None):
    """Batch-1 greedy decode: device-fed loop (value) and one C-ABI call per
    token with host buffers (e2e)."""
    import torch

    from rapidocrvl_b200 import LoadOptions, Runtime, config, synth

    d = synth.ensure("bench", quant)
    cfg = config.load(d)
    total = prompt_len + warmup + 2 * steps + 8
    rt = Runtime.load(d, LoadOptions(quantization=quant, device=device, max_position=max(4096, total),
                                     kv_pool_bytes=2 << 30))
    prompt = synth.random_prompt(prompt_len, cfg.vocab_size, rank)

    def prefill():
        s = rt.new_sequence(total)
        tok = -1
        for p, t in enumerate(prompt):
            ids, _ = rt.step([s], ids=[t], need_logits=p == len(prompt) - 1)
            tok = int(ids[0])
        return s, tok

    seq_dev, tok_dev = prefill()
    seq_e2e, tok_e2e = prefill()
    stream = torch.cuda.ExternalStream(rt.stream_handle)
    out = rt.decode_device([seq_dev], [tok_dev], warmup)
    tok_dev = int(out[-1, 0])
    for _ in range(warmup):
        ids, _ = rt.step([seq_e2e], ids=[tok_e2e])
        tok_e2e = int(ids[0])
    torch.cuda.synchronize()
    res = {}
    ev0, ev1 = events()
    sampler = ClockSampler(clocks_for) if clocks_for is not None else None
    if sampler:
        sampler.__enter__()
    try:
        ev0.record(stream)
        rt.decode_device([seq_dev], [tok_dev], steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        e0, e1 = events()
        e0.record(stream)
        for _ in range(steps):
            ids, _ = rt.step([seq_e2e], ids=[tok_e2e])
            tok_e2e = int(ids[0])
        e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1)
    finally:
        if sampler:
            sampler.__exit__()
    w_bytes, kv_tok = algorithmic_bytes(d, quant, cfg)
    ctx0 = prompt_len + warmup
    kv = sum((ctx0 + i + 1) * kv_tok for i in range(steps)) + steps * kv_tok  # read + append
    res["bytes_per_step"] = w_bytes + kv / steps
    res["ms"], res["ms_e2e"] = ms, ms_e2e
    res["io"] = rt.step_io_bytes(1)
    res["clocks"] = sampler.summary() if sampler else None
    res["cfg"] = cfg
    res["dir"] = d
    res["prompt"] = prompt
    rt.close()
    return res


def batched_workload(quant, n, ctx_hi, steps, warmup, rank, device):
    """configs3: n sequences with contexts U[256, ctx_hi] (seed 2), seeded
    synthetic caches, one token per sequence per step; value through the
    device-fed loop, e2e through ocrvl_step with host buffers."""
    import numpy as np
    import torch

    from rapidocrvl_b200 import LoadOptions, Runtime, config, synth

    d = synth.ensure("bench", quant)
    cfg = config.load(d)
    rng = np.random.default_rng(2 + rank)
    lens = rng.integers(256, ctx_hi + 1, size=n).tolist()
    total_new = warmup + 2 * steps + 2
    _, kv_tok = algorithmic_bytes(d, quant, cfg)
    rt = Runtime.load(d, LoadOptions(quantization=quant, device=device, max_position=ctx_hi + total_new + 64,
                                     kv_pool_bytes=int(sum(lens) + n * (total_new + 32)) * kv_tok + (256 << 20)))
    seqs = [rt.new_sequence(L + total_new + 8) for L in lens]
    t0 = time.time()
    for j, L in enumerate(lens):
        seqs[j].fill_synthetic(L, 1000 * rank + j)
    t_setup = time.time() - t0
    first = [int(t) for t in rng.integers(0, cfg.vocab_size, size=n)]
    out = rt.decode_device(seqs, first, warmup)
    toks = [int(i) for i in out[-1]]
    stream = torch.cuda.ExternalStream(rt.stream_handle)
    torch.cuda.synchronize()
    ev0, ev1 = events()
    ev0.record(stream)
    out = rt.decode_device(seqs, toks, steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    toks = [int(i) for i in out[-1]]
    e0, e1 = events()
    e0.record(stream)
    for _ in range(steps):
        ids, _ = rt.step(seqs, ids=toks)
        toks = [int(i) for i in ids]
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    w_bytes, kv_tok = algorithmic_bytes(d, quant, cfg)
    ctx0 = [L + warmup for L in lens]
    kv = sum(sum((c + i + 1) * kv_tok for c in ctx0) for i in range(steps)) + steps * n * kv_tok
    res = {"ms": ms, "ms_e2e": ms_e2e, "bytes_per_step": w_bytes + kv / steps, "io": rt.step_io_bytes(n),
           "setup_s": t_setup, "mean_context": float(np.mean(ctx0)) + steps / 2, "cfg": cfg}
    rt.close()
    return res


def gemv_workload(reps=20):
    """Quant-GEMV bandwidth of the op-level kernels: ocrvl_op_matvec (k_gemv)
    on lm_head-sized matrices with one input vector, per quantization type, and
    ocrvl_op_rowsum (k_rowsum).  Weight bytes are random (every byte pattern is
    a valid Q4/Q6/Q8 row); successive calls use different copies so that the
    weights stream from HBM.  Algorithmic bytes per call: packed rows + f32
    scales (+ int32 row sums for the int8-activation types) + input + output."""
    import ctypes as C

    import torch

    from rapidocrvl_b200 import _lib, gguf

    L = _lib.load()
    rows, cols = 103424, 1024
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    peak, src = hbm_peak()
    res = {}
    g = torch.Generator(device="cuda").manual_seed(5)
    for name, typ in (("q4", gguf.Q4_ROW), ("q6", gguf.Q6_ROW), ("q8", gguf.Q8_ROW)):
        pitch = gguf.packed_row_bytes(typ, cols)
        copies = max(2, -(-300_000_000 // (rows * pitch)))
        ws = [torch.randint(0, 256, (rows, pitch), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
        sc = torch.rand(rows, device="cuda", generator=g) * 1e-3 + 1e-4
        rs = [torch.empty(rows, dtype=torch.int32, device="cuda") for _ in range(copies)]
        x = torch.randn(cols, device="cuda", generator=g)
        out = torch.empty(rows, device="cuda")
        for i in range(copies):
            _lib.check(L.ocrvl_op_rowsum(typ, rows, cols, ptr(ws[i]), ptr(rs[i]), sh))
        for i in range(3):  # warm-up
            _lib.check(L.ocrvl_op_matvec(typ, rows, cols, ptr(ws[i % copies]), ptr(sc), ptr(rs[i % copies]), 1, ptr(x),
                                         None, 0.0, ptr(out), sh))
        ev0, ev1 = events()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(reps):
            _lib.check(L.ocrvl_op_matvec(typ, rows, cols, ptr(ws[i % copies]), ptr(sc), ptr(rs[i % copies]), 1, ptr(x),
                                         None, 0.0, ptr(out), sh))
        ev1.record(stream)
        torch.cuda.synchronize()
        us = ev0.elapsed_time(ev1) * 1e3 / reps
        nbytes = rows * (pitch + 4 + (4 if typ != gguf.Q8_ROW else 0)) + cols * 4 + rows * 4
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"kernel": "k_gemv", "us_per_call": us, "algorithmic_bytes": nbytes, "achieved_gbs": gbs,
                     "frac": gbs / peak}
        if name == "q4":
            e0, e1 = events()
            e0.record(stream)
            for i in range(reps):
                _lib.check(L.ocrvl_op_rowsum(typ, rows, cols, ptr(ws[i % copies]), ptr(rs[i % copies]), sh))
            e1.record(stream)
            torch.cuda.synchronize()
            us_r = e0.elapsed_time(e1) * 1e3 / reps
            rb = rows * (pitch + 4)
            res["rowsum_q4"] = {"kernel": "k_rowsum", "us_per_call": us_r, "algorithmic_bytes": rb,
                                "achieved_gbs": rb / (us_r * 1e-6) / 1e9, "frac": rb / (us_r * 1e-6) / 1e9 / peak}
        del ws, rs
        torch.cuda.empty_cache()
    res["peak_gbs"] = peak
    res["peak_source"] = src
    res["shape"] = f"{rows} x {cols}, one input vector, {reps} calls over rotating weight copies (> 2x L2)"
    return res


def sample_workload(reps=20):
    """The device sampler (ocrvl_op_sample, k_sample) on rows of vocab
    103,424 logits (randn * 2): top-k 50 at temperature 0.8 and the full
    vocabulary at temperature 1.0, for 1 and 64 rows, device-timed over
    `reps` calls after 3 warm-up calls (the rows stay in L2: the sampler
    reads each row once or twice and is bound by its sequential sums and one
    SM's issue rate, not by HBM)."""
    import ctypes as C

    import torch

    from rapidocrvl_b200 import _lib

    L = _lib.load()
    V = 103424
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    g = torch.Generator(device="cuda").manual_seed(11)
    res = {}
    for m in (1, 64):
        x = torch.randn(m, V, device="cuda", generator=g) * 2
        st = torch.arange(m, dtype=torch.int64, device="cuda")
        out = torch.empty(m, dtype=torch.int32, device="cuda")
        work = torch.empty(m, V, device="cuda")
        for name, temp, k in (("top_k50", 0.8, 50), ("full_vocab", 1.0, 0)):
            wk = ptr(work) if k == 0 else None

            def call():
                _lib.check(L.ocrvl_op_sample(m, V, ptr(x), temp, k, ptr(st), ptr(out), None, None, wk, sh))

            for _ in range(3):
                call()
            ev0, ev1 = events()
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(reps):
                call()
            ev1.record(stream)
            torch.cuda.synchronize()
            res[f"{name}_rows{m}_us"] = ev0.elapsed_time(ev1) * 1e3 / reps
    res["shape"] = f"vocab {V}, randn*2 logits, {reps} calls per case"
    return res


def sweep_workload(n_requests, rank, world, device, new_tokens=256, max_live=64):
    """configs4: Q8, n_requests requests (prompts U[1024, 8192], seed 3),
    new_tokens greedy tokens each, partitioned over the ranks by predicted KV
    bytes; each rank runs a continuous batch of up to max_live sequences."""
    import numpy as np
    import torch

    from rapidocrvl_b200 import LoadOptions, Runtime, config, partition, scheduler, synth

    d = synth.ensure("bench", "q8")
    cfg = config.load(d)
    rng = np.random.default_rng(3)
    prompts = rng.integers(1024, 8193, size=n_requests).tolist()
    firsts = rng.integers(0, cfg.vocab_size, size=n_requests).tolist()
    costs = [partition.request_cost(cfg, p, new_tokens) for p in prompts]
    mine = partition.shard(costs, rank, world)
    w_bytes, kv_tok = algorithmic_bytes(d, "q8", cfg)
    # live sequences at their longest, plus a margin for the one joining
    live_peak = sorted((prompts[i] + new_tokens + 16 for i in mine), reverse=True)[:max_live + 1]
    rt = Runtime.load(d, LoadOptions(quantization="q8", device=device, max_position=8192 + new_tokens + 64,
                                     kv_pool_bytes=int(sum(live_peak) * kv_tok) + (512 << 20)))
    reqs = [scheduler.Request(i, prompts[i], new_tokens, int(firsts[i])) for i in mine]
    stream = torch.cuda.ExternalStream(rt.stream_handle)
    fill_s = [0.0]

    def prefill(seq, r):
        t0 = time.time()
        seq.fill_synthetic(r.prompt_tokens, 7919 * r.index + 1)
        fill_s[0] += time.time() - t0

    stats = scheduler.run(rt, reqs, prefill, max_live=max_live, stream=stream)
    bytes_total = stats.steps * w_bytes + stats.kv_positions_read * kv_tok + stats.tokens * kv_tok
    res = {"ms": stats.step_ms, "steps": stats.steps, "tokens": stats.tokens, "requests": len(mine),
           "bytes_total": bytes_total, "mean_batch": stats.tokens / max(1, stats.steps), "fill_s": fill_s[0],
           "io": rt.step_io_bytes(min(max_live, max(1, len(mine))))}
    rt.close()
    return res


def run_cuda(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900))
        pg = dist
    from rapidocrvl_b200 import synth

    if rank == 0:
        for q in ("q4", "q8"):
            synth.ensure("bench", q)
    if pg:
        pg.barrier()

    def max_over_ranks(vals):
        if not pg:
            return vals
        t = torch.tensor(vals, device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return [float(x) for x in t]

    def sum_over_ranks(vals):
        if not pg:
            return vals
        t = torch.tensor(vals, device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.SUM)
        return [float(x) for x in t]

    want = args.workload
    line = None
    if want in ("all", "configs1"):
        if pg:
            pg.barrier()
        r = bs1_workload(args.quant, args.prompt, args.steps, args.warmup, rank, local, "configs1",
                         clocks_for=visible_bus_ids(local))
        ms, ms_e2e = max_over_ranks([r["ms"], r["ms_e2e"]])
        cfg = r["cfg"]
        h2d, d2h = r["io"]
        line = {
            "metric": METRIC, "value": world * args.steps / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8/f32" if args.quant != "q8" else "f32",
            "data": "synthetic (seeded N(0,0.02) BF16 weights converted to GGUF; uniform random prompt ids)",
            "config": workload_config(args, cfg),
            "roofline": roofline(r["bytes_per_step"], ms / args.steps, "k_step (one persistent launch per token)"),
            "e2e": {"value": world * args.steps / (ms_e2e / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": 1,
            "gpu_launches_note": "value: the device-fed loop runs all K steps in one persistent k_step launch; "
                                 "e2e: one k_step launch per token",
            "clocks": r["clocks"],
        }
        traffic_path = os.path.join(ROOT, "profiles", "k_step_traffic.json")
        if os.path.exists(traffic_path):
            with open(traffic_path) as f:
                tj = json.load(f)
            if tj.get("quant") == args.quant:
                # one ncu capture at a fixed context, moved to this run's mean
                # context by the K/V bytes per position (traffic grows with it)
                mean_ctx = args.prompt + args.warmup + (args.steps + 1) / 2
                line["roofline"]["traffic"] = (tj["dram_bytes_per_step"]
                                               + (mean_ctx - tj["context"]) * tj["kv_bytes_per_position"])
                line["roofline"]["traffic_source"] = tj.get("source")
        if rank == 0 and world == 1 and os.environ.get("OCRVL_BENCH_NO_CPU") is None:
            steps, dt, t_pre, threads = cpu_reference_decode(r["dir"], args.quant, cfg, r["prompt"], args.steps, 0,
                                                             budget_s=15.0)
            line["cpu_baseline"] = {
                "value": steps / dt, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{steps} greedy decode steps at context {args.prompt}+ after a {args.prompt}-token CPU "
                          f"prefill ({t_pre:.1f} s, untimed); C++ restatement of the reference Go CPU path, "
                          f"{threads} OpenMP threads"}
    extra = {}
    if world == 1 and want in ("all", "configs0"):
        r = bs1_workload("q8", 32, 64, 8, rank, local, "configs0")
        extra["configs0"] = {
            "workload": "configs[0]: Q8 decoder, batch 1, 32-token prompt, 8+64 greedy decode tokens",
            "value": 64 / (r["ms"] / 1e3), "unit": UNIT, "ms_per_step": r["ms"] / 64,
            "roofline": roofline(r["bytes_per_step"], r["ms"] / 64, "k_step (one persistent launch per token)"),
            "e2e": {"value": 64 / (r["ms_e2e"] / 1e3), "unit": UNIT, "h2d_bytes_per_step": r["io"][0],
                    "d2h_bytes_per_step": r["io"][1]}}
    if world == 1 and want in ("all", "configs3"):
        steps3 = 128 if want == "all" else args.steps
        warm3 = 4 if want == "all" else args.warmup
        r = batched_workload("q4", 64, args.ctx_hi, steps3, warm3, rank, local)
        extra["configs3"] = {
            "workload": f"configs[3]: Q4 decoder, 64 sequences, contexts U[256,{args.ctx_hi}] (seed 2), 16-token "
                        f"pages, {warm3}+{steps3} steps of one token per sequence",
            "value": 64 * steps3 / (r["ms"] / 1e3), "unit": UNIT, "ms_per_step": r["ms"] / steps3,
            "mean_context": r["mean_context"], "setup_s": round(r["setup_s"], 1),
            "kv": "seeded synthetic K/V written on the device (ocrvl_seq_fill_synthetic)",
            "roofline": roofline(r["bytes_per_step"], r["ms"] / steps3, "k_step_b (one persistent launch per step)"),
            "e2e": {"value": 64 * steps3 / (r["ms_e2e"] / 1e3), "unit": UNIT, "h2d_bytes_per_step": r["io"][0],
                    "d2h_bytes_per_step": r["io"][1]},
            "gpu_launches": steps3}
    if world == 1 and want in ("all", "gemv"):
        extra["gemv"] = gemv_workload()
    if world == 1 and want in ("all", "sample"):
        extra["sample"] = sample_workload(reps=max(1, args.steps) if want == "sample" else 20)
    if want in ("all", "configs4"):
        if pg:
            pg.barrier()
        r = sweep_workload(args.requests, rank, world, local)
        ms_max, = max_over_ranks([r["ms"]])
        tokens, bytes_total = sum_over_ranks([float(r["tokens"]), float(r["bytes_total"])])
        peak, src = hbm_peak()
        extra["configs4"] = {
            "workload": f"configs[4]: Q8 decoder, {args.requests} requests with prompts U[1024, 8192] (seed 3), 256 "
                        f"greedy tokens each, partitioned over {world} GPU(s) by predicted KV bytes, continuous "
                        f"batching of up to 64 live sequences per GPU",
            "value": tokens / (ms_max / 1e3), "unit": UNIT, "n_gpus": world, "scaling": "strong",
            "ms_max_over_ranks": ms_max, "rank0": {k: r[k] for k in ("steps", "tokens", "requests", "mean_batch")},
            "prefill": "seeded synthetic K/V written on the device, untimed",
            "roofline_per_gpu": {"bound": "hbm", "achieved": bytes_total / world / (ms_max / 1e3) / 1e9, "peak": peak,
                                 "unit": "GB/s", "frac": bytes_total / world / (ms_max / 1e3) / 1e9 / peak,
                                 "peak_source": src},
            "e2e": {"value": tokens / (ms_max / 1e3), "unit": UNIT, "h2d_bytes_per_step": r["io"][0],
                    "d2h_bytes_per_step": r["io"][1],
                    "note": "every step is a C-ABI ocrvl_step with host ids in and out"}}
    if line is None and want == "gemv":
        obj = extra["gemv"]
        line = {"metric": METRIC, "value": obj["q4"]["achieved_gbs"], "unit": "GB/s", "n_gpus": world,
                "steps": 20, "warmup": 3, "ms_per_step": obj["q4"]["us_per_call"] / 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic random weights",
                "config": {"workload": "quant-GEMV (k_gemv) Q4, " + obj["shape"]}, "gemv": obj}
    elif line is None and want == "sample":
        obj = extra["sample"]
        line = {"metric": "device sampler time per call (vocab 103424, top-k 50, one row)",
                "value": obj["top_k50_rows1_us"], "unit": "us", "n_gpus": world, "steps": max(1, args.steps),
                "warmup": 3, "ms_per_step": obj["top_k50_rows1_us"] / 1e3, "higher_is_better": False,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic logits",
                "config": {"workload": "k_sample, " + obj["shape"]}, "sample": obj}
    elif line is None:
        # a single non-headline workload: its object is the line
        (name, obj), = extra.items()
        line = {"metric": METRIC, "value": obj["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": obj.get("ms_per_step", obj.get("ms_max_over_ranks")),
                "higher_is_better": True, "scaling": obj.get("scaling", "weak"), "vs_baseline": None,
                "dtype": "i8/f32", "data": "synthetic", "config": {"workload": obj["workload"]},
                "roofline": obj.get("roofline", obj.get("roofline_per_gpu")), "e2e": obj["e2e"],
                "gpu_launches": obj.get("gpu_launches")}
    else:
        line.update(extra)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_cuda(args)


if __name__ == "__main__":
    sys.exit(main())
