"""Checkpoint -> GGUF converter, the command-line tool of the decode path.

    python -m rapidocrvl_b200.convert --model-dir DIR [--out PATH]
        [--quant f32|q8|q6|q4] [--progress|--no-progress] [--json]

Mirrors cmd/paddleocrvl-convert (cmd/paddleocrvl-convert/main.go:18-66):
reads ``model.safetensors`` (or the shards of
``model.safetensors.index.json``) and ``config.json`` from the model
directory, writes ``<model-dir>/model.gguf`` (f32) or
``model-<quant>.gguf`` by default, through a temporary file replaced on
success, and logs (or, with ``--json``, prints) a summary: output path,
quantization, bytes, sha256, elapsed ms, tensor counts from the written
file's metadata.  Quantized tensors are the text decoder's 2-D linear
weights (``is_quantized_text_tensor``); everything else is stored f32.
The Go tool's GOMAXPROCS and GC flags have no counterpart here.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

from . import config as cfgmod
from . import gguf, safetensors


def normalize_quant(q: str) -> str:
    q = (q or "").strip().lower()
    return q or "f32"


def default_output(model_dir: str, quant: str) -> str:
    name = {"q8": "model-q8.gguf", "q6": "model-q6.gguf", "q4": "model-q4.gguf"}.get(quant, "model.gguf")
    return os.path.join(model_dir, name)


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 22), b""):
            h.update(blk)
    return h.hexdigest()


def convert_dir(model_dir: str, out: str = "", quant: str = "f32", progress=None) -> dict:
    """Converts the checkpoint in ``model_dir``; returns the summary dict."""
    quant = normalize_quant(quant)
    if quant not in ("f32", "q8", "q6", "q4"):
        raise ValueError(f"unsupported quantization {quant!r} (f32, q8, q6 or q4)")
    dst = out or default_output(model_dir, quant)
    d = os.path.dirname(dst)
    if d:
        os.makedirs(d, exist_ok=True)
    cfg = None
    if os.path.exists(os.path.join(model_dir, "config.json")):
        cfg = cfgmod.load(model_dir)
    t0 = time.time()
    with safetensors.open_model(model_dir) as st:
        gguf.convert(st.tensors, dst, cfg, quant, shards=st.shard_count, progress=progress)
    elapsed = time.time() - t0
    g = gguf.GGUFFile(dst)
    meta = g.metadata
    return {
        "output": os.path.abspath(dst),
        "quant": quant,
        "bytes": os.path.getsize(dst),
        "sha256": sha256_file(dst),
        "elapsed_ms": int(elapsed * 1e3),
        "model_dir": os.path.abspath(model_dir),
        "config_path": os.path.abspath(model_dir),
        "source_tensors": int(meta.get("paddleocrvl.source_tensors", 0)),
        "f32_tensors": int(meta.get("paddleocrvl.f32_tensors", 0)),
        "quantized_tensors": int(meta.get("paddleocrvl.quantized_tensors", 0)),
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m rapidocrvl_b200.convert",
                                 description="Convert a safetensors checkpoint to the repo's GGUF row formats.")
    ap.add_argument("--model-dir", default=".", help="directory containing model.safetensors and config.json")
    ap.add_argument("--out", default="", help="output GGUF path; default is <model-dir>/model[-quant].gguf")
    ap.add_argument("--quant", default="f32", help="output quantization: f32, q8, q6, or q4")
    ap.add_argument("--progress", action=argparse.BooleanOptionalAction, default=True, help="log conversion progress")
    ap.add_argument("--json", action="store_true", help="emit the conversion summary as JSON")
    args = ap.parse_args(argv)
    last = [0.0]

    def progress(done, total, name, typ):
        if done == total:
            print(f"converted {done}/{total} tensors", file=sys.stderr)
            return
        now = time.time()
        if done == 0 or now - last[0] >= 2.0:
            print(f"converting {done + 1}/{total} {typ} {name}", file=sys.stderr)
            last[0] = now

    try:
        s = convert_dir(args.model_dir, args.out, args.quant, progress if args.progress else None)
    except (ValueError, OSError) as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    if args.json:
        print(json.dumps(s))
    else:
        print(f"wrote {s['output']} quant={s['quant']} bytes={s['bytes']} sha256={s['sha256']} "
              f"tensors={s['source_tensors']} f32={s['f32_tensors']} quantized={s['quantized_tensors']} "
              f"elapsed={s['elapsed_ms']}ms", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
