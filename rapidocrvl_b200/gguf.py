"""The repo's custom GGUF v3 row-quantized format (mirror of ``internal/gguf``).

Reader: ``GGUFFile`` restates ``gguf.Open`` and the row loaders
(internal/gguf/gguf.go:111-251, 313-569).  Writer: ``convert`` restates
``ConvertSafetensorsWithOptions`` (internal/gguf/convert.go:42-198): tensors in
sorted name order, 32-byte alignment, per-row quantization of the decoder's
linear weights and lm_head, the same metadata keys.

Row layouts (tensor types 1000/1001/1002, gguf.go:19-22): a tensor is
``[rows x f32 scale][rows x packed row]``.
  * Q8_ROW: int8 in [-127, 127], one byte per weight, scale = max|row|/127.
  * Q4_ROW: byte j holds column 2j in the low nibble and 2j+1 in the high
    nibble, nibble = q + 8 with q in [-7, 7], scale = max|row|/7.
  * Q6_ROW: four 6-bit fields per three bytes, little endian
    (v0 | v1<<6 | v2<<12 | v3<<18), field = q + 32 with q in [-31, 31],
    scale = max|row|/31.
An all-zero row stores scale 1 and zero data.

Quantizers restate the reference's scalar row quantizers
(internal/tensor/quant.go:96-147, 201-280, 291-365): float32 arithmetic,
round half away from zero, per-type clamp.  The reference's AVX2/AVX-512
quantizers for Q4 and Q6 (internal/tensor/dot_amd64.s:5887-5935 and
6004-6099) pack 16 values into 4 bytes and duplicate values 0-3 into slots 4-7
respectively, so their output does not round-trip through the reader; the
scalar semantics are the ones the reader's layout defines.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"GGUF"
VERSION = 3
ALIGNMENT = 32

F32 = 0
Q8_ROW = 1000
Q4_ROW = 1001
Q6_ROW = 1002

META_U32 = 4
META_U64 = 10
META_STR = 8

MAX_TENSOR_COUNT = 1 << 20
MAX_KV_COUNT = 1 << 20
MAX_STRING = 16 << 20
MAX_DIMS = 8

TYPE_NAMES = {F32: "F32", Q8_ROW: "Q8_ROW", Q4_ROW: "Q4_ROW", Q6_ROW: "Q6_ROW"}
QUANT_TYPES = {"q8": Q8_ROW, "q6": Q6_ROW, "q4": Q4_ROW}


def packed_row_bytes(typ: int, cols: int) -> int:
    if typ == Q8_ROW:
        return cols
    if typ == Q4_ROW:
        return (cols + 1) // 2
    if typ == Q6_ROW:
        return (cols * 6 + 7) // 8
    if typ == F32:
        return cols * 4
    raise ValueError(f"unsupported GGUF tensor type {typ}")


def tensor_bytes(typ: int, shape) -> int:
    """TensorBytes (gguf.go:586-631)."""
    if typ == F32:
        n = 1
        for d in shape:
            n *= int(d)
        return n * 4
    if len(shape) != 2:
        return 0
    rows, cols = int(shape[0]), int(shape[1])
    return rows * 4 + rows * packed_row_bytes(typ, cols)


def _align(n: int, a: int = ALIGNMENT) -> int:
    return (n + a - 1) // a * a


# ---------------------------------------------------------------------------
# Quantizers (numpy, float32 arithmetic)
# ---------------------------------------------------------------------------
def _round_half_away(x: np.ndarray) -> np.ndarray:
    """roundToInt (quant.go:436-441): int(x+0.5) / int(x-0.5) in float32."""
    half = np.float32(0.5)
    return np.where(x >= 0, np.trunc(x + half), np.trunc(x - half)).astype(np.int32)


def _row_scales(w: np.ndarray, qmax: float):
    m = np.max(np.abs(w), axis=1).astype(np.float32)
    zero = m == 0
    scale = (m / np.float32(qmax)).astype(np.float32)
    scale[zero] = np.float32(1.0)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    return scale, inv, zero


def quantize_rows(typ: int, w: np.ndarray):
    """Quantize a [rows, cols] float32 matrix; returns (scales f32[rows], packed u8[rows, pb])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if typ == Q8_ROW:
        scale, inv, zero = _row_scales(w, 127.0)
        q = np.clip(_round_half_away(w * inv[:, None]), -127, 127)
        q[zero] = 0
        return scale, q.astype(np.int8).view(np.uint8)
    if typ == Q4_ROW:
        scale, inv, zero = _row_scales(w, 7.0)
        nib = (np.clip(_round_half_away(w * inv[:, None]), -7, 7) + 8).astype(np.uint8)
        if cols % 2:
            nib = np.concatenate([nib, np.zeros((rows, 1), np.uint8)], axis=1)
            nib[:, -1] = 0
        packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
        packed[zero] = 0
        return scale, packed
    if typ == Q6_ROW:
        scale, inv, zero = _row_scales(w, 31.0)
        v = (np.clip(_round_half_away(w * inv[:, None]), -31, 31) + 32).astype(np.uint32)
        packed = pack_q6_fields(v)
        packed[zero] = 0
        return scale, packed
    raise ValueError(f"unsupported quantized type {typ}")


def unpack_rows(typ: int, packed: np.ndarray, cols: int) -> np.ndarray:
    """Packed rows -> int8 weights (unpackQ4RowFast / unpackQ6RowFast)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    rows = packed.shape[0]
    if typ == Q8_ROW:
        return packed.view(np.int8)[:, :cols].copy()
    if typ == Q4_ROW:
        lo = (packed & 0x0F).astype(np.int16) - 8
        hi = (packed >> 4).astype(np.int16) - 8
        out = np.empty((rows, packed.shape[1] * 2), np.int16)
        out[:, 0::2] = lo
        out[:, 1::2] = hi
        return out[:, :cols].astype(np.int8)
    if typ == Q6_ROW:
        return (q6_fields(packed, cols).astype(np.int16) - 32).astype(np.int8)
    raise ValueError(f"unsupported quantized type {typ}")


def pack_q6_fields(v: np.ndarray) -> np.ndarray:
    """Pack [rows, cols] 6-bit fields, four per three bytes little endian
    (putQ6, quant.go:2886-2895); a partial last group leaves its unused bits 0."""
    v = np.asarray(v, dtype=np.uint32) & 0x3F
    rows, cols = v.shape
    pad = (-cols) % 4
    if pad:
        v = np.concatenate([v, np.zeros((rows, pad), np.uint32)], axis=1)
    g = v.reshape(rows, -1, 4)
    word = g[:, :, 0] | (g[:, :, 1] << 6) | (g[:, :, 2] << 12) | (g[:, :, 3] << 18)
    b = np.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], axis=2).astype(np.uint8)
    return b.reshape(rows, -1)[:, : packed_row_bytes(Q6_ROW, cols)].copy()


def q6_fields(packed: np.ndarray, cols: int) -> np.ndarray:
    """The [rows, cols] 6-bit fields of packed Q6 rows (getQ6, quant.go:2897-2906)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    rows, nb = packed.shape
    padded = np.zeros((rows, (nb + 2) // 3 * 3), np.uint32)
    padded[:, :nb] = packed
    g = padded.reshape(rows, -1, 3)
    word = g[:, :, 0] | (g[:, :, 1] << 8) | (g[:, :, 2] << 16)
    vals = np.stack([(word >> s) & 0x3F for s in (0, 6, 12, 18)], axis=2).reshape(rows, -1)
    return vals[:, :cols].astype(np.uint8)


# ---------------------------------------------------------------------------
# Reader
# ---------------------------------------------------------------------------
@dataclass
class TensorMeta:
    shape: tuple
    type: int
    offset: int


class GGUFFile:
    """Memory-mapped reader (gguf.Open + Q8Row/Q4Row/Q6Row/Float32)."""

    def __init__(self, path: str):
        self.path = path
        self.metadata = {}
        self.tensors = {}
        size = os.path.getsize(path)
        if size < 24:
            raise ValueError("truncated GGUF header")
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        hdr_limit = min(size, 256 << 20)
        pos = 0

        def take(n):
            nonlocal pos
            if pos + n > hdr_limit:
                raise ValueError("truncated GGUF header")
            b = self._mm[pos : pos + n].tobytes()
            pos += n
            return b

        def u32():
            return struct.unpack("<I", take(4))[0]

        def u64():
            return struct.unpack("<Q", take(8))[0]

        def string():
            n = u64()
            if n > MAX_STRING:
                raise ValueError(f"GGUF string too large: {n} bytes")
            return take(n).decode("utf-8", errors="surrogateescape")

        if take(4) != MAGIC:
            raise ValueError("bad GGUF magic")
        ver = u32()
        if ver != VERSION:
            raise ValueError(f"unsupported GGUF version {ver}")
        nt = u64()
        if nt > MAX_TENSOR_COUNT:
            raise ValueError(f"GGUF tensor count too large: {nt}")
        nkv = u64()
        if nkv > MAX_KV_COUNT:
            raise ValueError(f"GGUF metadata count too large: {nkv}")
        for _ in range(nkv):
            key = string()
            _check_name(key, "metadata key")
            typ = u32()
            if typ == META_U32:
                val = u32()
            elif typ == META_U64:
                val = u64()
            elif typ == META_STR:
                val = string()
            else:
                raise ValueError(f"unsupported GGUF metadata type {typ}")
            if key in self.metadata:
                raise ValueError(f"GGUF metadata key {key} is duplicated")
            self.metadata[key] = val
        for _ in range(nt):
            name = string()
            _check_name(name, "tensor name")
            if name in self.tensors:
                raise ValueError(f"GGUF tensor {name} is duplicated")
            nd = u32()
            if nd > MAX_DIMS:
                raise ValueError(f"GGUF tensor {name} has too many dimensions: {nd}")
            shape = tuple(u64() for _ in range(nd))
            typ = u32()
            off = u64()
            self.tensors[name] = TensorMeta(shape, typ, off)
        self.data_start = _align(pos)
        if self.data_start > size:
            raise ValueError("GGUF header exceeds file size")
        for name, m in self.tensors.items():
            nbytes = tensor_bytes(m.type, m.shape)
            if nbytes <= 0:
                raise ValueError(f"GGUF tensor {name} has invalid type or shape")
            if self.data_start + m.offset + nbytes > size:
                raise ValueError(f"GGUF tensor {name} exceeds file size")

    def raw(self, name: str) -> np.ndarray:
        m = self.tensors.get(name)
        if m is None:
            raise KeyError(f"missing tensor {name}")
        start = self.data_start + m.offset
        return self._mm[start : start + tensor_bytes(m.type, m.shape)]

    def float32(self, name: str) -> np.ndarray:
        m = self.tensors[name]
        if m.type != F32:
            raise ValueError(f"unsupported GGUF tensor type {m.type} for {name}")
        return self.raw(name).view(np.float32).reshape(m.shape)

    def row_quant(self, name: str):
        """Returns (type, scales f32[rows], packed u8[rows, pb], shape)."""
        m = self.tensors[name]
        if m.type not in (Q8_ROW, Q4_ROW, Q6_ROW):
            raise ValueError(f"unsupported GGUF tensor type {m.type} for {name}")
        if len(m.shape) != 2:
            raise ValueError(f"{TYPE_NAMES[m.type]} tensor {name} must be 2D")
        rows, cols = int(m.shape[0]), int(m.shape[1])
        raw = self.raw(name)
        scales = raw[: rows * 4].view(np.float32)
        packed = raw[rows * 4 :].reshape(rows, packed_row_bytes(m.type, cols))
        return m.type, scales, packed, (rows, cols)


def _check_name(s: str, what: str):
    if not s:
        raise ValueError(f"GGUF has empty {what}")
    if any(ord(ch) < 0x20 or ord(ch) == 0x7F for ch in s):
        raise ValueError(f"GGUF {what} contains control character")


# ---------------------------------------------------------------------------
# Writer / converter
# ---------------------------------------------------------------------------
def is_quantized_text_tensor(name: str, shape, cfg) -> bool:
    """isQuantizedTextTensor (convert.go:402-434)."""
    if cfg is None or len(shape) != 2:
        return False
    if name == "lm_head.weight":
        return shape[0] == cfg.vocab_size and shape[1] == cfg.hidden_size
    if not name.startswith("model.layers."):
        return False
    rest = name[len("model.layers.") :]
    if "." not in rest:
        return False
    layer_text, suffix = rest.split(".", 1)
    if not layer_text.isdigit() or int(layer_text) >= cfg.num_hidden_layers:
        return False
    q, kv, hs, inter = cfg.q_rows, cfg.kv_rows, cfg.hidden_size, cfg.intermediate_size
    want = {
        "self_attn.q_proj.weight": (q, hs),
        "self_attn.k_proj.weight": (kv, hs),
        "self_attn.v_proj.weight": (kv, hs),
        "self_attn.o_proj.weight": (hs, q),
        "mlp.gate_proj.weight": (inter, hs),
        "mlp.up_proj.weight": (inter, hs),
        "mlp.down_proj.weight": (hs, inter),
    }.get(suffix)
    return want is not None and tuple(int(d) for d in shape) == want


def _metadata(cfg, quant: str, n_tensors: int, n_f32: int, n_quant: int, n_shards: int = 1):
    file_type = {"q8": 7, "q6": 6, "q4": 3}.get(quant, 0)
    kvs = [
        ("general.architecture", META_STR, "paddleocrvl"),
        ("general.name", META_STR, "PaddleOCR-VL-0.9B"),
        ("general.alignment", META_U32, ALIGNMENT),
        ("general.file_type", META_U32, file_type),
        ("paddleocrvl.gguf_version", META_U32, VERSION),
        ("paddleocrvl.quantization", META_STR, quant or "f32"),
        ("paddleocrvl.source_tensors", META_U64, n_tensors),
        ("paddleocrvl.source_shards", META_U64, n_shards),
        ("paddleocrvl.f32_tensors", META_U64, n_f32),
        ("paddleocrvl.quantized_tensors", META_U64, n_quant),
    ]
    if cfg is not None:
        kvs += [
            ("paddleocrvl.vocab_size", META_U64, cfg.vocab_size),
            ("paddleocrvl.text_layers", META_U64, cfg.num_hidden_layers),
            ("paddleocrvl.hidden_size", META_U64, cfg.hidden_size),
            ("paddleocrvl.vision_layers", META_U64, cfg.vision_num_hidden_layers),
        ]
    return kvs


def _pack_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def convert(tensors, dst: str, cfg, quantization: str = "q8", shards: int = 1, progress=None) -> None:
    """Write ``tensors`` (name -> float32 ndarray, or an object with ``shape``
    and ``materialize()``, materialized in sorted name order) as a GGUF file.
    ``shards``: the source checkpoint's file count (metadata); ``progress``:
    called as progress(done, total, name, type_name) before each tensor and
    once at the end (ConvertOptions.Progress, internal/gguf/convert.go:37-40)."""
    quant = (quantization or "f32").strip().lower()
    if quant not in ("f32", "q8", "q6", "q4"):
        raise ValueError(f"unsupported quantization {quantization!r}")
    names = sorted(tensors)
    infos = []
    off = 0
    n_f32 = n_q = 0
    for name in names:
        shape = tuple(int(d) for d in tensors[name].shape)
        typ = F32
        if quant != "f32" and is_quantized_text_tensor(name, shape, cfg):
            typ = QUANT_TYPES[quant]
        if typ == F32:
            n_f32 += 1
        else:
            n_q += 1
        off = _align(off)
        infos.append((name, shape, typ, off))
        off += tensor_bytes(typ, shape)
    hdr = bytearray()
    hdr += MAGIC + struct.pack("<I", VERSION)
    kvs = _metadata(cfg, quant, len(names), n_f32, n_q, shards)
    hdr += struct.pack("<QQ", len(infos), len(kvs))
    for key, typ, val in kvs:
        hdr += _pack_str(key) + struct.pack("<I", typ)
        if typ == META_STR:
            hdr += _pack_str(val)
        elif typ == META_U32:
            hdr += struct.pack("<I", val)
        else:
            hdr += struct.pack("<Q", val)
    for name, shape, typ, o in infos:
        hdr += _pack_str(name) + struct.pack("<I", len(shape))
        for d in shape:
            hdr += struct.pack("<Q", d)
        hdr += struct.pack("<IQ", typ, o)
    hdr += b"\0" * (_align(len(hdr)) - len(hdr))
    tmp = dst + ".tmp"
    with open(tmp, "wb") as f:
        f.write(hdr)
        cur = 0
        for i, (name, shape, typ, o) in enumerate(infos):
            if progress is not None:
                progress(i, len(infos), name, TYPE_NAMES.get(typ, str(typ)))
            if cur < o:
                f.write(b"\0" * (o - cur))
                cur = o
            t = tensors[name]
            arr = np.asarray(t.materialize() if hasattr(t, "materialize") else t, dtype=np.float32)
            if typ == F32:
                b = np.ascontiguousarray(arr).tobytes()
            else:
                sc, packed = quantize_rows(typ, arr.reshape(shape))
                b = sc.astype(np.float32).tobytes() + packed.tobytes()
            f.write(b)
            cur += len(b)
    if progress is not None:
        progress(len(infos), len(infos), "", "")
    os.replace(tmp, dst)
