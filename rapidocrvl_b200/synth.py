"""Seeded synthetic ERNIE decoders for tests and benchmarks.

The benchmark configuration (hidden 1024, 18 layers, 16 q / 2 kv heads,
head_dim 128, SwiGLU 3072, vocab 103424, eps 1e-5, theta 5e5) has no public
checkpoint here, so weights are drawn N(0, 0.02) from
``torch.Generator().manual_seed(seed)`` one tensor at a time in sorted-name
order, cast to BF16 (as a safetensors checkpoint would store them), widened
back to float32 and written through the restated converter
(:func:`rapidocrvl_b200.gguf.convert`).  Norm weights are drawn the same way.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

from . import config as cfgmod
from . import gguf

BENCH_CONFIG = dict(
    vocab_size=103424,
    hidden_size=1024,
    intermediate_size=3072,
    num_hidden_layers=18,
    num_attention_heads=16,
    num_key_value_heads=2,
    head_dim=128,
    rms_norm_eps=1e-5,
    rope_theta=500000.0,
)

# Small decoder for the test-suite: head_dim 128 as in the benchmark model, but
# 4 q heads over 2 kv heads (GQA group 2, where the benchmark model has 8).
TINY_CONFIG = dict(
    vocab_size=1000,
    hidden_size=256,
    intermediate_size=384,
    num_hidden_layers=2,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=128,
    rms_norm_eps=1e-5,
    rope_theta=500000.0,
)


def make_config(**kw) -> cfgmod.Config:
    c = cfgmod.Config(**kw)
    return c


def tensor_shapes(c: cfgmod.Config) -> dict:
    shapes = {
        "model.embed_tokens.weight": (c.vocab_size, c.hidden_size),
        "model.norm.weight": (c.hidden_size,),
        "lm_head.weight": (c.vocab_size, c.hidden_size),
    }
    for i in range(c.num_hidden_layers):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = (c.hidden_size,)
        shapes[p + "post_attention_layernorm.weight"] = (c.hidden_size,)
        shapes[p + "self_attn.q_proj.weight"] = (c.q_rows, c.hidden_size)
        shapes[p + "self_attn.k_proj.weight"] = (c.kv_rows, c.hidden_size)
        shapes[p + "self_attn.v_proj.weight"] = (c.kv_rows, c.hidden_size)
        shapes[p + "self_attn.o_proj.weight"] = (c.hidden_size, c.q_rows)
        shapes[p + "mlp.gate_proj.weight"] = (c.intermediate_size, c.hidden_size)
        shapes[p + "mlp.up_proj.weight"] = (c.intermediate_size, c.hidden_size)
        shapes[p + "mlp.down_proj.weight"] = (c.hidden_size, c.intermediate_size)
    return shapes


class _Lazy:
    """A tensor drawn from a shared generator when the converter reaches it."""

    def __init__(self, gen, shape, std):
        self.gen, self.shape, self.std = gen, shape, std

    def materialize(self):
        import torch

        t = torch.randn(self.shape, generator=self.gen, dtype=torch.float32) * self.std
        return t.to(torch.bfloat16).to(torch.float32).numpy()


def build(model_dir: str, c: cfgmod.Config, quantization: str, seed: int = 0, std: float = 0.02) -> str:
    """Write config.json + model-<quant>.gguf into ``model_dir``; returns the GGUF path."""
    import torch

    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(c.to_json(), f, indent=1)
    gen = torch.Generator().manual_seed(seed)
    shapes = tensor_shapes(c)
    tensors = {name: _Lazy(gen, shapes[name], std) for name in sorted(shapes)}
    path = os.path.join(model_dir, f"model-{quantization}.gguf")
    gguf.convert(tensors, path, c, quantization)
    return path


def cache_root() -> str:
    return os.environ.get("OCRVL_MODEL_CACHE", os.path.join("/tmp", "ocrvl_models"))


# The tiny decoder with a vocabulary that is a multiple of 16 (the
# full-vocabulary sampler's whole 16-float blocks).
TINY_V1024_CONFIG = dict(TINY_CONFIG, vocab_size=1024)

KINDS = {"bench": BENCH_CONFIG, "tiny": TINY_CONFIG, "tiny-v1024": TINY_V1024_CONFIG}


def ensure(kind: str, quantization: str, seed: int = 0) -> str:
    """Return a model directory holding the seeded ``kind`` (a key of KINDS)
    decoder in ``quantization``, building it on first use."""
    kw = KINDS[kind]
    c = make_config(**kw)
    key = hashlib.sha1(json.dumps([kw, seed, 1], sort_keys=True).encode()).hexdigest()[:10]
    d = os.path.join(cache_root(), f"{kind}-{key}")
    path = os.path.join(d, f"model-{quantization}.gguf")
    if not os.path.exists(path):
        build(d, c, quantization, seed)
    return d


def random_prompt(n: int, vocab: int, seed: int) -> list:
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def all_close_hist(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64)))) if a.size else 0.0
