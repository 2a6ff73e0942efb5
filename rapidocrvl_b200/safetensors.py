"""Reader of safetensors checkpoints for the GGUF converter.

Restates the reference's reader (internal/safetensors/safetensors.go):
``open_model(dir)`` takes ``model.safetensors`` or, failing that, the shards
listed by ``model.safetensors.index.json`` (OpenModel, OpenSetFile,
OpenSetIndex, safetensors.go:48-148); a file is an 8-byte little-endian
header length, a JSON header (name -> dtype, shape, data_offsets; an optional
``__metadata__`` entry) and the tensor bytes (Open, safetensors.go:175-238).
Tensors are decoded to float32 on demand: F32 as is, BF16 by widening the
16 bits to the upper half of a float32, F16 by IEEE half conversion
(readEncodedFloat32At / decodeBF16 / decodeF16).  Names, shard file names,
offsets and sizes are validated before any data is read.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np

MAX_HEADER_BYTES = 100 << 20   # a JSON header larger than this is rejected
MAX_INDEX_BYTES = 64 << 20
MAX_TENSORS = 1 << 20
DTYPE_SIZE = {"F32": 4, "BF16": 2, "F16": 2, "F64": 8, "I64": 8, "I32": 4, "I16": 2, "I8": 1, "U8": 1, "BOOL": 1}


def _reject_duplicate_keys(pairs):
    out = {}
    for k, v in pairs:
        if k in out:
            raise ValueError(f"duplicate JSON key {k!r}")
        out[k] = v
    return out


def _check_name(name: str) -> None:
    if not name or len(name) > 4096 or any(ord(ch) < 0x20 for ch in name):
        raise ValueError(f"invalid tensor name {name!r}")


def _safe_shard(name: str) -> bool:
    if name in ("", ".", "..") or "/" in name or "\\" in name:
        return False
    return all(ch.isascii() and (ch.isalnum() or ch in "._-") for ch in name)


class Tensor:
    """One tensor of an open file: shape, dtype, and its float32 values on
    demand (``materialize``), so the converter reads one tensor at a time."""

    def __init__(self, f: "File", name: str, dtype: str, shape, begin: int, end: int):
        self.file, self.name, self.dtype = f, name, dtype
        self.shape = tuple(int(d) for d in shape)
        self.begin, self.end = begin, end

    def raw(self) -> memoryview:
        return memoryview(self.file.map)[self.file.data_start + self.begin:self.file.data_start + self.end]

    def materialize(self) -> np.ndarray:
        raw = self.raw()
        if self.dtype == "F32":
            out = np.frombuffer(raw, dtype="<f4").copy()
        elif self.dtype == "BF16":
            out = (np.frombuffer(raw, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
        elif self.dtype == "F16":
            out = np.frombuffer(raw, dtype="<f2").astype(np.float32)
        else:
            raise ValueError(f"unsupported dtype {self.dtype} for {self.name}")
        return out.reshape(self.shape)


class File:
    """One safetensors file, memory-mapped."""

    def __init__(self, path: str):
        self.path = path
        self._fh = open(path, "rb")
        size = os.fstat(self._fh.fileno()).st_size
        head = self._fh.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: truncated safetensors file")
        (hlen,) = struct.unpack("<Q", head)
        if hlen > MAX_HEADER_BYTES or 8 + hlen > size:
            raise ValueError(f"{path}: safetensors header too large: {hlen} bytes")
        header = json.loads(self._fh.read(hlen), object_pairs_hook=_reject_duplicate_keys)
        if not isinstance(header, dict):
            raise ValueError(f"{path}: header is not a JSON object")
        self.data_start = 8 + hlen
        data_bytes = size - self.data_start
        self.map = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
        self.tensors = {}
        entries = {k: v for k, v in header.items() if k != "__metadata__"}
        if len(entries) > MAX_TENSORS:
            raise ValueError(f"{path}: too many tensors ({len(entries)})")
        for name, meta in entries.items():
            _check_name(name)
            try:
                dtype, shape, (b, e) = meta["dtype"], meta["shape"], meta["data_offsets"]
            except (KeyError, TypeError, ValueError) as exc:
                raise ValueError(f"{path}: malformed entry for {name}") from exc
            if dtype not in DTYPE_SIZE:
                raise ValueError(f"{path}: unknown dtype {dtype} for {name}")
            if any((not isinstance(d, int)) or d < 0 for d in shape):
                raise ValueError(f"{path}: bad shape {shape} for {name}")
            nbytes = int(np.prod(shape, dtype=np.int64)) * DTYPE_SIZE[dtype] if shape else DTYPE_SIZE[dtype]
            if not (0 <= b <= e <= data_bytes) or e - b != nbytes:
                raise ValueError(f"{path}: data offsets [{b}, {e}) of {name} do not match its shape / the file")
            self.tensors[name] = Tensor(self, name, dtype, shape, b, e)

    def close(self) -> None:
        if isinstance(self.map, mmap.mmap):
            self.map.close()
        self._fh.close()


class Set:
    """The tensors of a model (one file or the shards of an index)."""

    def __init__(self, files, tensors):
        self.files, self.tensors = files, tensors

    @property
    def shard_count(self) -> int:
        return len(self.files)

    def close(self) -> None:
        for f in self.files.values():
            f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def open_file_set(path: str) -> Set:
    f = File(path)
    return Set({os.path.basename(path): f}, dict(f.tensors))


def open_index(path: str) -> Set:
    if os.path.getsize(path) > MAX_INDEX_BYTES:
        raise ValueError(f"safetensors index too large: {path}")
    with open(path, "rb") as fh:
        idx = json.loads(fh.read(), object_pairs_hook=_reject_duplicate_keys)
    wm = idx.get("weight_map") if isinstance(idx, dict) else None
    if not wm:
        raise ValueError(f"{path} has empty weight_map")
    if len(wm) > MAX_TENSORS:
        raise ValueError(f"{path}: too many tensors ({len(wm)})")
    d = os.path.dirname(path)
    files, tensors = {}, {}
    try:
        for name, shard in wm.items():
            _check_name(name)
            if not isinstance(shard, str) or not _safe_shard(shard):
                raise ValueError(f"unsafe shard path {shard!r}")
            if shard not in files:
                files[shard] = File(os.path.join(d, shard))
            t = files[shard].tensors.get(name)
            if t is None:
                raise ValueError(f"{name} listed in index but missing from {shard}")
            tensors[name] = t
    except Exception:
        for f in files.values():
            f.close()
        raise
    return Set(files, tensors)


def open_model(src: str) -> Set:
    """A file, or a directory holding model.safetensors or
    model.safetensors.index.json (OpenModel)."""
    if os.path.isfile(src):
        return open_file_set(src)
    single = os.path.join(src, "model.safetensors")
    if os.path.exists(single):
        return open_file_set(single)
    index = os.path.join(src, "model.safetensors.index.json")
    if os.path.exists(index):
        return open_index(index)
    raise FileNotFoundError(f"no model.safetensors or model.safetensors.index.json in {src}")


def write_file(path: str, tensors: dict, dtype: str = "F32") -> None:
    """Writes float32 arrays as one safetensors file in `dtype` (F32, BF16
    (round to nearest even) or F16): the fixture writer of the converter's
    tests and of synthetic checkpoints."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name], dtype=np.float32)
        if dtype == "F32":
            b = a.astype("<f4").tobytes()
        elif dtype == "BF16":
            u = a.view(np.uint32).astype(np.uint64)
            b = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2")).tobytes()
        elif dtype == "F16":
            b = a.astype("<f2").tobytes()
        else:
            raise ValueError(f"unsupported dtype {dtype}")
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
