"""Host-side logic with no GPU: config loading, the GGUF reader's rejection of
malformed files, generation-option validation, backend selection and the
request partitioner."""
import struct

import numpy as np
import pytest

from rapidocrvl_b200 import config, gguf, partition, synth
from rapidocrvl_b200.runtime import (GenerateOptions, select_backend, validate_generate_options,
                                     validate_generation_input)


# ---- config (internal/config/config.go:51-84) -------------------------------
def test_config_defaults_and_duplicates():
    c = config.loads('{"hidden_size": 1024, "num_attention_heads": 16, "vocab_size": 5}')
    assert c.head_dim == 64 and c.num_key_value_heads == 16
    assert c.rope_theta == 10000.0 and c.rms_norm_eps == 1e-6
    assert c.mrope_section == [16, 24, 24]
    with pytest.raises(ValueError, match="duplicate key"):
        config.loads('{"hidden_size": 1, "hidden_size": 2}')
    with pytest.raises(ValueError, match="duplicate key"):
        config.loads('{"vision_config": {"a": 1, "a": 2}}')
    c = config.loads('{"rope_scaling": {"mrope_section": [8, 12, 12]}, "vision_config": {"spatial_merge_size": 2}}')
    assert c.mrope_section == [8, 12, 12] and c.spatial_merge_size == 2


def test_validate_decoder():
    config.validate_decoder(config.Config(**synth.BENCH_CONFIG))
    with pytest.raises(ValueError):
        config.validate_decoder(config.Config(**dict(synth.TINY_CONFIG, num_key_value_heads=3)))
    with pytest.raises(ValueError):
        config.validate_decoder(config.Config(**dict(synth.TINY_CONFIG, num_hidden_layers=0)))


# ---- GGUF reader (internal/gguf/gguf.go:111-251) -----------------------------
@pytest.fixture()
def small_gguf(tmp_path):
    cfg = config.Config(**synth.TINY_CONFIG)
    rng = np.random.default_rng(0)
    t = {"lm_head.weight": rng.standard_normal((cfg.vocab_size, cfg.hidden_size)).astype(np.float32),
         "model.norm.weight": np.ones(cfg.hidden_size, np.float32)}
    p = str(tmp_path / "m.gguf")
    gguf.convert(t, p, cfg, "q4")
    return p, t


def test_gguf_round_trip_layout(small_gguf):
    p, t = small_gguf
    g = gguf.GGUFFile(p)
    assert g.metadata["general.architecture"] == "paddleocrvl"
    assert g.metadata["paddleocrvl.quantization"] == "q4"
    assert list(g.tensors) == sorted(t)  # sorted-name order (convert.go:60-64)
    assert all(m.offset % gguf.ALIGNMENT == 0 for m in g.tensors.values())
    assert g.data_start % gguf.ALIGNMENT == 0
    typ, sc, pk, shape = g.row_quant("lm_head.weight")
    assert typ == gguf.Q4_ROW and shape == t["lm_head.weight"].shape
    sc2, pk2 = gguf.quantize_rows(gguf.Q4_ROW, t["lm_head.weight"])
    assert np.array_equal(sc, sc2) and np.array_equal(pk, pk2)
    assert np.array_equal(g.float32("model.norm.weight"), t["model.norm.weight"])


def _corrupt(path, tmp_path, edit):
    b = bytearray(open(path, "rb").read())
    b = edit(b)
    q = str(tmp_path / "bad.gguf")
    with open(q, "wb") as fh:
        fh.write(bytes(b))
    return q


@pytest.mark.parametrize("edit,msg", [
    (lambda b: b"XXXX" + b[4:], "bad GGUF magic"),
    (lambda b: b[:4] + struct.pack("<I", 2) + b[8:], "unsupported GGUF version"),
    (lambda b: b[:8] + struct.pack("<Q", 1 << 40) + b[16:], "tensor count too large"),
    (lambda b: b[:16] + struct.pack("<Q", 1 << 40) + b[24:], "metadata count too large"),
    (lambda b: b[:20], "truncated"),
    (lambda b: b[: len(b) - 100], "exceeds file size"),
])
def test_gguf_rejects_malformed(small_gguf, tmp_path, edit, msg):
    p, _ = small_gguf
    with pytest.raises(ValueError, match=msg):
        gguf.GGUFFile(_corrupt(p, tmp_path, edit))


def test_gguf_rejects_duplicate_tensor_and_bad_names(tmp_path):
    def build(names):
        hdr = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(names), 0))
        for n in names:
            nb = n.encode()
            hdr += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", 1) + struct.pack("<Q", 4)
            hdr += struct.pack("<IQ", gguf.F32, 0)
        hdr += b"\0" * ((-len(hdr)) % 32) + b"\0" * 64
        p = str(tmp_path / "x.gguf")
        open(p, "wb").write(bytes(hdr))
        return p

    with pytest.raises(ValueError, match="duplicated"):
        gguf.GGUFFile(build(["a", "a"]))
    with pytest.raises(ValueError, match="control character"):
        gguf.GGUFFile(build(["a\x01"]))
    with pytest.raises(ValueError, match="empty"):
        gguf.GGUFFile(build([""]))


def test_quantizable_predicate():
    """isQuantizedTextTensor (convert.go:402-434): only decoder linears and lm_head."""
    cfg = config.Config(**synth.TINY_CONFIG)
    assert gguf.is_quantized_text_tensor("lm_head.weight", (1000, 256), cfg)
    assert gguf.is_quantized_text_tensor("model.layers.1.mlp.down_proj.weight", (256, 384), cfg)
    assert not gguf.is_quantized_text_tensor("model.layers.2.mlp.down_proj.weight", (256, 384), cfg)
    assert not gguf.is_quantized_text_tensor("model.layers.0.mlp.down_proj.weight", (384, 256), cfg)
    assert not gguf.is_quantized_text_tensor("model.embed_tokens.weight", (1000, 256), cfg)
    assert not gguf.is_quantized_text_tensor("model.norm.weight", (256,), cfg)


# ---- generation options (internal/model/model.go:448-490) --------------------
def test_generate_option_validation():
    validate_generate_options(GenerateOptions(max_new_tokens=3))
    for bad in (dict(max_new_tokens=-1), dict(temperature=-0.5), dict(temperature=float("nan")),
                dict(temperature=float("inf")), dict(top_k=-1), dict(eos_token_ids=[-1]),
                dict(eos_token_ids=list(range(1025)))):
        with pytest.raises(ValueError):
            validate_generate_options(GenerateOptions(**bad))
    with pytest.raises(ValueError, match="must not be empty"):
        validate_generation_input([], GenerateOptions(max_new_tokens=1))
    validate_generation_input([], GenerateOptions(max_new_tokens=0))
    with pytest.raises(ValueError, match="negative"):
        validate_generation_input([1, -2], GenerateOptions(max_new_tokens=1))


def test_backend_selection_is_strict():
    for name in ("cpu", "vulkan", "metal"):
        with pytest.raises(ValueError, match="not provided"):
            select_backend(name)


# ---- request partitioner ------------------------------------------------------
def test_partition_assign_properties():
    cfg = config.Config(**synth.BENCH_CONFIG)
    rng = np.random.default_rng(3)
    prompts = rng.integers(1024, 8192, size=512)
    costs = [partition.request_cost(cfg, int(p), 256) for p in prompts]
    for world in (1, 2, 4, 8):
        plan = partition.assign(costs, world)
        flat = sorted(i for p in plan for i in p)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in plan]
        # LPT bound: max load <= mean + max single request
        assert max(loads) <= sum(costs) / world + max(costs)
        assert plan == partition.assign(costs, world)  # deterministic
        for r in range(world):
            assert partition.shard(costs, r, world) == plan[r]
    assert partition.assign([5, 5], 4) == [[0], [1], [], []]
    assert partition.assign([], 2) == [[], []]
    with pytest.raises(ValueError):
        partition.assign([1], 0)
    with pytest.raises(ValueError):
        partition.shard([1], 2, 2)
    assert partition.kv_bytes_per_token(cfg) == 36864
