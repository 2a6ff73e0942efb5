"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
the checker / CPU baseline; never by the product package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


class OrcConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int),
        ("hidden_size", C.c_int),
        ("intermediate_size", C.c_int),
        ("num_layers", C.c_int),
        ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_double),
        ("mrope_section", C.c_int * 3),
    ]


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(_HERE, f) for f in ("oracle.cpp", "oracle.h")]
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(map(os.path.getmtime, srcs)):
            build()
        L = C.CDLL(_LIB_PATH)
        P, I, F, D = C.c_void_p, C.c_int, C.c_float, C.c_double
        L.orc_load.restype = P
        L.orc_load.argtypes = [C.c_char_p, C.POINTER(OrcConfig), C.c_char_p, I]
        L.orc_free.argtypes = [P]
        L.orc_set_threads.argtypes = [I]
        L.orc_quant_type.argtypes = [P]
        L.orc_seq_new.restype = P
        L.orc_seq_new.argtypes = [P, I]
        L.orc_seq_free.argtypes = [P]
        L.orc_seq_len.argtypes = [P]
        L.orc_seq_kv.argtypes = [P, I, P, P]
        L.orc_seq_import_kv.argtypes = [P, I, P, P]
        L.orc_forward.argtypes = [P, P, P, I, I, I, I, P, P, P]
        L.orc_forward_dump.argtypes = [P, P, P, I, I, I, P, P, P]
        L.orc_generate.argtypes = [P, P, I, I, P, I, P, I]
        L.orc_decode_steps.argtypes = [P, P, I, I, I]
        L.orc_embed.argtypes = [P, I, P]
        L.orc_quantize_row.restype = F
        L.orc_quantize_row.argtypes = [I, P, I, P]
        L.orc_unpack_row.argtypes = [I, P, I, P]
        L.orc_quantize_x.restype = F
        L.orc_quantize_x.argtypes = [P, I, P]
        L.orc_dot_u8s8.restype = C.c_int32
        L.orc_dot_u8s8.argtypes = [P, P, I]
        L.orc_vnni_finalize.restype = F
        L.orc_vnni_finalize.argtypes = [C.c_int32, C.c_int32, F, F]
        L.orc_dot_q8_f32.restype = F
        L.orc_dot_q8_f32.argtypes = [P, P, I]
        L.orc_matvec.argtypes = [I, I, I, P, P, P, P]
        L.orc_matvec_add_rmsnorm.argtypes = [I, I, I, P, P, P, P, P, F, I, P]
        L.orc_swiglu.argtypes = [I, I, I, P, P, P, P, P, P]
        L.orc_rmsnorm.argtypes = [P, P, I, F, P]
        L.orc_fast_rsqrt.restype = F
        L.orc_fast_rsqrt.argtypes = [F]
        L.orc_fast_exp.restype = F
        L.orc_fast_exp.argtypes = [F]
        L.orc_rope.argtypes = [P, I, I, P, P]
        L.orc_rope_table.argtypes = [C.POINTER(OrcConfig), I, I, I, P, P]
        L.orc_softmax.argtypes = [P, I]
        L.orc_attention.argtypes = [P, P, P, I, I, I, I, P]
        L.orc_argmax_matvec.argtypes = [I, I, I, P, P, P, P]
        U64P = C.POINTER(C.c_uint64)
        L.orc_rng_float64.restype = D
        L.orc_rng_float64.argtypes = [U64P]
        L.orc_topk_select.argtypes = [P, I, I, P, P]
        L.orc_sample_candidates.argtypes = [P, P, I, D, U64P]
        L.orc_sample_full.argtypes = [P, I, F, U64P]
        L.orc_pick_cumulative.argtypes = [P, I, F]
        L.orc_sample_token.argtypes = [P, I, D, I, U64P]
        L.orc_generate_sampled.argtypes = [P, P, I, I, P, I, D, I, C.c_int64, P, I]
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    """OpenMP threads of the oracle (n > 0 sets them); returns the count in effect."""
    return int(lib().orc_set_threads(int(n)))


def _seed64(seed: int) -> int:
    """The int64 whose two's-complement bits are uint64(seed)."""
    u = int(seed) & 0xFFFFFFFFFFFFFFFF
    return u - (1 << 64) if u >= 1 << 63 else u


class RNG:
    """fastRNG (model.go:1829-1852) held in a uint64; ``state`` is readable."""

    def __init__(self, seed: int):
        self._s = C.c_uint64(int(seed) & 0xFFFFFFFFFFFFFFFF)

    @property
    def state(self) -> int:
        return int(self._s.value)

    def float64(self) -> float:
        return float(lib().orc_rng_float64(C.byref(self._s)))


def topk_select(logits, k):
    """topKSelectWithWork: (ids, scores) of the k best, descending, ties -> lower id."""
    x = np.ascontiguousarray(logits, np.float32)
    k = min(int(k), len(x))
    ids = np.zeros(k, np.int32)
    sc = np.zeros(k, np.float32)
    lib().orc_topk_select(ptr(x), len(x), k, ptr(ids), ptr(sc))
    return ids, sc


def sample_candidates(ids, scores, temperature, rng: RNG) -> int:
    i = np.ascontiguousarray(ids, np.int32)
    s = np.ascontiguousarray(scores, np.float32)
    return int(lib().orc_sample_candidates(ptr(i), ptr(s), len(i), float(temperature), C.byref(rng._s)))


def pick_cumulative(cdf, pick) -> int:
    """pickCumulativeFloat32: first index with pick <= cdf[i], or -1."""
    c = np.ascontiguousarray(cdf, np.float32)
    return int(lib().orc_pick_cumulative(ptr(c), len(c), float(pick)))


def sample_full(logits, temperature, rng: RNG) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_full(ptr(x), len(x), float(temperature), C.byref(rng._s)))


def sample_token(logits, temperature, top_k, rng: RNG) -> int:
    """The generation loop's sampler on one row of logits (-2: unsupported vocab)."""
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_token(ptr(x), len(x), float(temperature), int(top_k), C.byref(rng._s)))


def ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def make_config(c) -> OrcConfig:
    oc = OrcConfig()
    oc.vocab_size = c.vocab_size
    oc.hidden_size = c.hidden_size
    oc.intermediate_size = c.intermediate_size
    oc.num_layers = c.num_hidden_layers
    oc.num_heads = c.num_attention_heads
    oc.num_kv_heads = c.num_key_value_heads
    oc.head_dim = c.head_dim
    oc.rms_norm_eps = c.rms_norm_eps
    oc.rope_theta = c.rope_theta
    for i in range(3):
        oc.mrope_section[i] = c.mrope_section[i]
    return oc


class OracleModel:
    """Oracle decoder loaded from a GGUF file."""

    def __init__(self, gguf_path: str, cfg):
        self.cfg = cfg
        self._oc = make_config(cfg)
        err = C.create_string_buffer(512)
        self.h = lib().orc_load(gguf_path.encode(), C.byref(self._oc), err, 512)
        if not self.h:
            raise RuntimeError("oracle load failed: " + err.value.decode())

    def close(self):
        if self.h:
            lib().orc_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def generate(self, ids, max_new, eos=None):
        ids = np.asarray(ids, dtype=np.int32)
        out = np.zeros(len(ids) + max_new + 1, dtype=np.int32)
        e = None if eos is None else np.asarray(eos, dtype=np.int32)
        n = lib().orc_generate(self.h, ptr(ids), len(ids), max_new, None if e is None else ptr(e),
                               0 if e is None else len(e), ptr(out), len(out))
        if n < 0:
            raise RuntimeError(f"oracle generate failed ({n})")
        return out[:n].tolist()

    def generate_sampled(self, ids, max_new, temperature, top_k, seed, eos=None):
        """GenerateWithOptions with temperature / top_k / seed (orc_generate_sampled)."""
        ids = np.asarray(ids, dtype=np.int32)
        out = np.zeros(len(ids) + max_new + 1, dtype=np.int32)
        e = None if eos is None else np.asarray(eos, dtype=np.int32)
        n = lib().orc_generate_sampled(self.h, ptr(ids), len(ids), max_new, None if e is None else ptr(e),
                                       0 if e is None else len(e), float(temperature), int(top_k),
                                       _seed64(seed), ptr(out), len(out))
        if n < 0:
            raise RuntimeError(f"oracle generate failed ({n})")
        return out[:n].tolist()

    def new_seq(self, max_tokens):
        return OracleSeq(self, max_tokens)

    def embed(self, tok):
        out = np.zeros(self.cfg.hidden_size, np.float32)
        if lib().orc_embed(self.h, int(tok), ptr(out)) != 0:
            raise ValueError("token id outside vocab")
        return out


class OracleSeq:
    def __init__(self, model: OracleModel, max_tokens: int):
        self.m = model
        self.h = lib().orc_seq_new(model.h, max_tokens)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_seq_free(self.h)
            self.h = None

    def __len__(self):
        return lib().orc_seq_len(self.h)

    def forward(self, emb, pos, need_logits=True, want_logits=False):
        """Returns (token, logits|None, final_norm)."""
        c = self.m.cfg
        emb = np.ascontiguousarray(emb, dtype=np.float32)
        tok = C.c_int(-1)
        logits = np.zeros(c.vocab_size, np.float32) if want_logits else None
        fin = np.zeros(c.hidden_size, np.float32)
        t, h, w = pos if isinstance(pos, (tuple, list)) else (pos, pos, pos)
        rc = lib().orc_forward(self.m.h, self.h, ptr(emb), t, h, w, int(need_logits), C.byref(tok),
                               None if logits is None else ptr(logits), ptr(fin))
        if rc != 0:
            raise RuntimeError(f"oracle forward failed ({rc})")
        return tok.value, logits, fin

    def forward_dump(self, emb, pos):
        """orc_forward_dump: (token, logits, per-layer dict of intermediates)."""
        c = self.m.cfg
        H, I = c.hidden_size, c.intermediate_size
        qr, kr = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
        per = 4 * H + 2 * qr + 2 * kr + I
        dump = np.zeros(c.num_hidden_layers * per, np.float32)
        logits = np.zeros(c.vocab_size, np.float32)
        tok = C.c_int(-1)
        t, h, w = pos if isinstance(pos, (tuple, list)) else (pos, pos, pos)
        rc = lib().orc_forward_dump(self.m.h, self.h, ptr(np.ascontiguousarray(emb, np.float32)), t, h, w,
                                    C.byref(tok), ptr(logits), ptr(dump))
        if rc != 0:
            raise RuntimeError(f"oracle forward failed ({rc})")
        layers = []
        for li in range(c.num_hidden_layers):
            d = dump[li * per:(li + 1) * per]
            o = 0
            rec = {}
            for name, size in (("h_in", H), ("norm1", H), ("q", qr), ("k", kr), ("v", kr), ("head", qr),
                               ("vo", H), ("norm2", H), ("g", I)):
                rec[name] = d[o:o + size].copy()
                o += size
            layers.append(rec)
        return tok.value, logits, layers

    def kv(self, layer):
        c = self.m.cfg
        n = len(self)
        kvd = c.num_key_value_heads * c.head_dim
        k = np.zeros((max(n, 1), kvd), np.float32)
        v = np.zeros((max(n, 1), kvd), np.float32)
        lib().orc_seq_kv(self.h, layer, ptr(k), ptr(v))
        return k[:n], v[:n]

    def import_kv(self, k, v):
        """Cache of n positions, k and v [num_layers][n][kv_heads*head_dim] f32."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if k.shape != v.shape or k.ndim != 3:
            raise ValueError("K/V must be [num_layers][n][kvd]")
        if lib().orc_seq_import_kv(self.h, int(k.shape[1]), ptr(k), ptr(v)) != 0:
            raise RuntimeError("oracle import_kv failed")

    def decode_steps(self, tok, pos, steps):
        return lib().orc_decode_steps(self.m.h, self.h, int(tok), int(pos), int(steps))
