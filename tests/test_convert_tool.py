"""The checkpoint converter as a tool (python -m rapidocrvl_b200.convert),
the counterpart of cmd/paddleocrvl-convert and
gguf.ConvertSafetensorsWithOptions (internal/gguf/convert.go:42-198): a
safetensors checkpoint (single file or sharded index; F32, BF16 or F16) in,
a GGUF file whose tensors are those of the library converter on the decoded
float32 values, and the reader's validation of malformed checkpoints
(internal/safetensors/safetensors.go:48-290)."""
import json
import os
import struct

import numpy as np
import pytest

from rapidocrvl_b200 import config as cfgmod
from rapidocrvl_b200 import convert, gguf, safetensors, synth


def _model(tmp_path, dtype="BF16", seed=0):
    c = synth.make_config(**synth.TINY_CONFIG)
    rng = np.random.default_rng(seed)
    tensors = {n: (rng.standard_normal(s) * 0.02).astype(np.float32) for n, s in synth.tensor_shapes(c).items()}
    d = tmp_path / "model"
    d.mkdir()
    with open(d / "config.json", "w") as f:
        json.dump(c.to_json(), f)
    return c, tensors, d


def _decoded(tensors, dtype):
    """The float32 values a reader of `dtype` storage sees."""
    out = {}
    for n, a in tensors.items():
        if dtype == "BF16":
            u = a.view(np.uint32).astype(np.uint64)
            out[n] = ((((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)).view(np.float32)
        elif dtype == "F16":
            out[n] = a.astype(np.float16).astype(np.float32)
        else:
            out[n] = a
    return out


def _payloads(path):
    g = gguf.GGUFFile(path)
    return {n: np.asarray(g.raw(n)).tobytes() for n in g.tensors}, g


@pytest.mark.parametrize("dtype", ["BF16", "F16", "F32"])
@pytest.mark.parametrize("quant", ["q4", "q8"])
def test_tool_matches_library_converter(tmp_path, dtype, quant):
    c, tensors, d = _model(tmp_path, dtype)
    safetensors.write_file(str(d / "model.safetensors"), tensors, dtype)
    rc = convert.main(["--model-dir", str(d), "--quant", quant, "--no-progress"])
    assert rc == 0
    out = d / f"model-{quant}.gguf"
    ref = tmp_path / "ref.gguf"
    gguf.convert(_decoded(tensors, dtype), str(ref), cfgmod.load(str(d)), quant)
    with open(out, "rb") as a, open(ref, "rb") as b:
        assert a.read() == b.read()


def test_sharded_index_and_json_summary(tmp_path, capsys):
    c, tensors, d = _model(tmp_path)
    names = sorted(tensors)
    shards = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    wm = {}
    for fn, ns in shards.items():
        safetensors.write_file(str(d / fn), {n: tensors[n] for n in ns}, "BF16")
        wm.update({n: fn for n in ns})
    with open(d / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)
    rc = convert.main(["--model-dir", str(d), "--quant", "q6", "--json", "--no-progress"])
    assert rc == 0
    summary = json.loads(capsys.readouterr().out)
    assert summary["quant"] == "q6" and summary["source_tensors"] == len(tensors)
    assert summary["quantized_tensors"] + summary["f32_tensors"] == len(tensors)
    assert summary["quantized_tensors"] == 7 * c.num_hidden_layers + 1  # q,k,v,o,gate,up,down per layer + lm_head
    got, g = _payloads(summary["output"])
    assert g.metadata["paddleocrvl.source_shards"] == 2
    # tensor payloads equal to a single-file conversion of the same values
    single = tmp_path / "single"
    single.mkdir()
    safetensors.write_file(str(single / "model.safetensors"), tensors, "BF16")
    with open(single / "config.json", "w") as f:
        json.dump(c.to_json(), f)
    s2 = convert.convert_dir(str(single), quant="q6")
    want, _ = _payloads(s2["output"])
    assert got == want


def _write_raw(path, header: dict, data: bytes):
    hj = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj + data)


@pytest.mark.parametrize(
    "header,data,msg",
    [
        ({"a": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 12]}}, b"\0" * 16, "data offsets"),
        ({"a": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 16]}}, b"\0" * 8, "data offsets"),
        ({"a": {"dtype": "Q9", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8, "unknown dtype"),
        ({"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, b"\0" * 4, "bad shape"),
        ({"a": {"shape": [1]}}, b"\0" * 4, "malformed"),
    ],
)
def test_reader_rejects_malformed_files(tmp_path, header, data, msg):
    p = tmp_path / "model.safetensors"
    _write_raw(p, header, data)
    with pytest.raises(ValueError, match=msg):
        safetensors.open_model(str(tmp_path))


def test_reader_rejects_duplicate_keys_and_unsafe_shards(tmp_path):
    p = tmp_path / "model.safetensors"
    hj = b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}, "a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}'
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj + b"\0" * 4)
    with pytest.raises(ValueError, match="duplicate"):
        safetensors.open_model(str(tmp_path))
    os.remove(p)
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"weight_map": {"a": "../evil.safetensors"}}, f)
    with pytest.raises(ValueError, match="unsafe shard"):
        safetensors.open_model(str(tmp_path))
    safetensors.write_file(str(tmp_path / "s1.safetensors"), {"b": np.zeros(2, np.float32)})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"weight_map": {"a": "s1.safetensors"}}, f)
    with pytest.raises(ValueError, match="missing"):
        safetensors.open_model(str(tmp_path))


def test_missing_checkpoint_and_bad_quant(tmp_path):
    assert convert.main(["--model-dir", str(tmp_path), "--no-progress"]) == 1
    with pytest.raises(ValueError, match="unsupported quantization"):
        convert.convert_dir(str(tmp_path), quant="q5")
