"""Decode-step benchmark (Q4, batch 1, 512-token
prompt, 256 greedy new tokens, context 512 -> 768).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

A step is one greedy decode token.  ``value`` is device-timed (CUDA events on
the engine's stream around K steps of the device-fed decode loop, inputs
resident in HBM); ``e2e`` times the same K-token workload through the
reference-facing C ABI (ocrvl_step with host buffers: token in, token out,
one call per token).  Under torchrun each rank decodes its own request on its
own GPU (request-parallel replicas, no collective on the data path); the
reported time is the max over ranks.  ``--impl reference`` times the CPU
restatement of the reference's decode path on the host cores instead.
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
    ap.add_argument("--workload", default="configs1", choices=["configs1", "configs3"],
                    help="configs1: batch 1, 512-token prompt (headline); configs3: 64 sequences, contexts U[256, 4096]")
    ap.add_argument("--ctx-hi", type=int, default=4096,
                    help="configs3: contexts drawn U[256, ctx_hi] (4096 is the workload; smaller for profiling captures)")
    ap.add_argument("--kv", default="prefill", choices=["prefill", "synthetic"],
                    help="configs3 caches: prompt prefill through steps, or seeded K/V imported directly")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def workload_config(args, cfg):
    return {
        "workload": f"configs[1]: {args.quant.upper()} decoder (hidden {cfg.hidden_size}, {cfg.num_hidden_layers} layers, "
                    f"{cfg.num_attention_heads}q/{cfg.num_key_value_heads}kv heads, head_dim {cfg.head_dim}, "
                    f"SwiGLU {cfg.intermediate_size}, vocab {cfg.vocab_size}), batch 1 per GPU, {args.prompt}-token "
                    f"prompt, {args.warmup}+{args.steps} greedy decode tokens",
        "quant": args.quant,
        "batch_per_gpu": 1,
        "prompt_tokens": args.prompt,
        "context": [args.prompt + args.warmup, args.prompt + args.warmup + args.steps],
        "parallelism": "request-parallel replicas (one sequence per GPU, no collective)",
        "l2": "no flush: per-step working set (all weights + KV) > 126 MB L2",
    }


def algorithmic_bytes(model_dir, quant, cfg):
    """Weight bytes streamed per token: rows*(packed row + f32
    scale) for every quantized matrix incl. lm_head, the 2L+1 f32 norm
    vectors and one f32 embedding row."""
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


def cpu_reference_decode(model_dir, quant, cfg, prompt, steps, warmup, seed_kv=None, budget_s=None):
    """Times the CPU restatement of the reference decode path (oracle/) on all
    host threads.  With seed_kv (GPU prefill K/V) the prompt is not recomputed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle

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
    return steps, dt, t_pre


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from rapidocrvl_b200 import config, synth

    d = synth.ensure("bench", args.quant)
    cfg = config.load(d)
    prompt = synth.random_prompt(args.prompt, cfg.vocab_size, 0)
    steps, dt, t_pre = cpu_reference_decode(d, args.quant, cfg, prompt, args.steps, args.warmup)
    v = steps / dt
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic (seeded N(0,0.02) BF16 weights -> GGUF; uniform prompt ids)",
        "config": workload_config(args, cfg),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{steps} greedy decode steps at context {args.prompt + args.warmup}+ after a "
                                   f"{args.prompt}-token CPU prefill ({t_pre:.1f} s, untimed); C++ restatement of the "
                                   f"reference Go CPU path (no Go toolchain on this image), all host threads"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_cuda(args):
    import numpy as np
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        pg = dist
    from rapidocrvl_b200 import LoadOptions, Runtime, config, synth

    if rank == 0:
        d = synth.ensure("bench", args.quant)
    if pg:
        pg.barrier()
    d = synth.ensure("bench", args.quant)
    cfg = config.load(d)
    total = args.prompt + args.warmup + 2 * args.steps + 8
    rt = Runtime.load(d, LoadOptions(quantization=args.quant, device=local, max_position=max(4096, total),
                                     kv_pool_bytes=2 << 30))
    prompt = synth.random_prompt(args.prompt, cfg.vocab_size, rank)

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
    # warm-up (device loop and host-call path)
    out = rt.decode_device([seq_dev], [tok_dev], args.warmup)
    tok_dev = int(out[-1, 0])
    for _ in range(args.warmup):
        ids, _ = rt.step([seq_e2e], ids=[tok_e2e])
        tok_e2e = int(ids[0])
    bus_ids = []
    try:
        r = subprocess.run(["nvidia-smi", "--query-gpu=pci.bus_id", "--format=csv,noheader"], capture_output=True,
                           text=True, timeout=20)
        allb = [x.strip() for x in r.stdout.splitlines() if x.strip()]
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = [int(v) for v in vis.split(",")] if vis else list(range(len(allb)))
        bus_ids = [allb[idx[local]]] if local < len(idx) and idx[local] < len(allb) else allb[:1]
    except Exception:
        bus_ids = []
    # ---- device-timed value ----
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(bus_ids) as clocks:
        ev0.record(stream)
        out = rt.decode_device([seq_dev], [tok_dev], args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        # ---- e2e through the C ABI, host buffers, one call per token ----
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            ids, _ = rt.step([seq_e2e], ids=[tok_e2e])
            tok_e2e = int(ids[0])
        e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1)
    if pg:
        t = torch.tensor([ms, ms_e2e], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
        pg.barrier()
    w_bytes, kv_tok = algorithmic_bytes(d, args.quant, cfg)
    ctx0 = args.prompt + args.warmup
    # step i attends ctx0+i+1 positions and appends one
    kv_read = sum((ctx0 + i + 1) * kv_tok for i in range(args.steps))
    bytes_per_step = w_bytes + (kv_read + args.steps * kv_tok) / args.steps
    step_s = ms / 1e3 / args.steps
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            peak, peak_src = float(json.load(f)["hbm_gbs"]), "measured"
    achieved = bytes_per_step / step_s / 1e9
    h2d, d2h = rt.step_io_bytes(1)
    value = world * args.steps / (ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "i8/f32" if args.quant != "q8" else "f32",
        "data": "synthetic (seeded N(0,0.02) BF16 weights converted to GGUF; uniform random prompt ids)",
        "config": workload_config(args, cfg),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else "fallback",
                     "kernel": "k_step (one persistent launch per token)",
                     "algorithmic_bytes_per_step": bytes_per_step, "traffic": None},
        "e2e": {"value": world * args.steps / (ms_e2e / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    traffic_path = os.path.join(ROOT, "profiles", "k_step_traffic.json")
    if os.path.exists(traffic_path):
        with open(traffic_path) as f:
            tj = json.load(f)
        if tj.get("quant") == args.quant:
            # one ncu capture at a fixed context, moved to this run's mean
            # context by the K/V bytes per position (traffic grows with it)
            mean_ctx = ctx0 + (args.steps + 1) / 2
            line["roofline"]["traffic"] = (tj["dram_bytes_per_step"]
                                           + (mean_ctx - tj["context"]) * tj["kv_bytes_per_position"])
            line["roofline"]["traffic_source"] = tj.get("source")
    if rank == 0 and world == 1 and os.environ.get("OCRVL_BENCH_NO_CPU") is None:
        steps, dt, t_pre = cpu_reference_decode(d, args.quant, cfg, prompt, args.steps, 0, budget_s=15.0)
        line["cpu_baseline"] = {
            "value": steps / dt, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} greedy decode steps at context {args.prompt}+ after a {args.prompt}-token CPU "
                      f"prefill ({t_pre:.1f} s, untimed); C++ restatement of the reference Go CPU path, all host "
                      f"threads (OpenMP)"}
    rt.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_batched(args):
    """64 sequences, contexts drawn U[256, 4096] (seed 2), one new
    token per sequence per step; the projections run as int8 tensor-core
    GEMMs (Q4).  Value = generated tokens/s of the device-fed loop."""
    import numpy as np
    import torch

    from rapidocrvl_b200 import LoadOptions, Runtime, config, synth

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    d = synth.ensure("bench", args.quant)
    cfg = config.load(d)
    n = 64
    rng = np.random.default_rng(2 + rank)
    lens = rng.integers(256, args.ctx_hi + 1, size=n).tolist()
    total_new = args.warmup + args.steps + 1
    rt = Runtime.load(d, LoadOptions(quantization=args.quant, device=local, max_position=8192,
                                     kv_pool_bytes=int(sum(lens) + n * (total_new + 32)) * 36864 + (256 << 20)))
    seqs = [rt.new_sequence(L + total_new + 8) for L in lens]
    prompts = [synth.random_prompt(L, cfg.vocab_size, 1000 * rank + j) for j, L in enumerate(lens)]
    t0 = time.time()
    if args.kv == "synthetic":
        # seeded K/V imported straight into the caches (ocrvl_seq_import_kv):
        # the decode timing does not depend on the cached values, and setting
        # up takes one call per sequence instead of max(lens) prefill launches
        kvd = cfg.num_key_value_heads * cfg.head_dim
        krng = np.random.default_rng(5 + rank)
        shape = (cfg.num_hidden_layers, max(lens), kvd)
        kpool = krng.standard_normal(shape, dtype=np.float32)
        vpool = krng.standard_normal(shape, dtype=np.float32)
        for j, L in enumerate(lens):  # sequence j: positions j .. j+L-2 of the pools (wrapping)
            idx = (np.arange(L - 1) + j) % shape[1]
            seqs[j].import_kv(kpool[:, idx], vpool[:, idx])
    else:
        for p in range(max(lens) - 1):
            live = [j for j in range(n) if p < lens[j] - 1]
            rt.step([seqs[j] for j in live], ids=[prompts[j][p] for j in live], need_logits=False)
    ids, _ = rt.step(seqs, ids=[pr[-1] for pr in prompts])
    t_pre = time.time() - t0
    first = [int(i) for i in ids]
    out = rt.decode_device(seqs, first, args.warmup)
    first = [int(i) for i in out[-1]]
    stream = torch.cuda.ExternalStream(rt.stream_handle)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    out = rt.decode_device(seqs, first, args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    w_bytes, kv_tok = algorithmic_bytes(d, args.quant, cfg)
    ctx0 = [L + args.warmup for L in lens]
    kv_read = sum(sum((c + i + 1) * kv_tok for c in ctx0) for i in range(args.steps))
    bytes_per_step = w_bytes + (kv_read + args.steps * n * kv_tok) / args.steps
    step_s = ms / 1e3 / args.steps
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak = 6650.0
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            peak = float(json.load(f)["hbm_gbs"])
    achieved = bytes_per_step / step_s / 1e9
    line = {
        "metric": METRIC, "value": n * args.steps / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic (seeded weights; uniform prompt ids)",
        "config": {"workload": f"configs[3]: {args.quant.upper()}, 64 sequences, contexts U[256,{args.ctx_hi}] (seed 2), "
                               f"16-token pages, {args.warmup}+{args.steps} steps of one token per sequence",
                   "kv": "prompt prefill" if args.kv == "prefill" else "seeded N(0,1) K/V imported",
                   "setup_s": round(t_pre, 1), "mean_context": float(np.mean(ctx0)) + args.steps / 2,
                   "l2": "no flush: per-step KV (~5.6 GB) + weights > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "kernel": "k_step_b (one persistent launch per step)",
                     "algorithmic_bytes_per_step": bytes_per_step, "traffic": None},
        "gpu_launches": args.steps,
    }
    traffic_path = os.path.join(ROOT, "profiles", "k_step_b_traffic.json")
    if os.path.exists(traffic_path):
        with open(traffic_path) as f:
            tj = json.load(f)
        if tj.get("quant") == args.quant:
            # one ncu capture of a smaller case, scaled by the algorithmic bytes
            # (the K/V stream dominates both)
            line["roofline"]["traffic"] = tj["dram_bytes_per_step"] * bytes_per_step / tj["algorithmic_bytes_per_step"]
            line["roofline"]["traffic_source"] = tj.get("source") + ", scaled by algorithmic bytes"
    rt.close()
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "configs3":
        return run_batched(args)
    return run_cuda(args)


if __name__ == "__main__":
    sys.exit(main())
