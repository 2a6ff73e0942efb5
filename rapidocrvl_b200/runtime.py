"""Host-side mirror of the reference's ``internal/model`` Runtime API for the
decode path, running on the CUDA engine (libocrvl_cuda.so).

Reference surface mirrored here (internal/model/model.go):
  * LoadOptions / LoadWithOptions (342-346, 546-605): quantization + backend.
  * GenerateOptions / ValidateGenerateOptions / GenerateResult (415-490).
  * Runtime.Generate / GenerateWithOptions (1484-1572): greedy generation.
  * forwardEmbeddingForSampling (3475-3643): ``Runtime.step`` (batched).
Backend names follow internal/backend/backend.go:85-111 with a strict
``"cuda"`` choice: no CPU fallback exists in this package.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import weakref
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from . import config as cfgmod

MAX_EOS_TOKEN_IDS = 1024
DEFAULT_EOS_TOKEN_IDS = [2]


@dataclass
class LoadOptions:
    quantization: str = "q8"
    backend: str = "cuda"
    device: int = 0
    kv_pool_bytes: int = 0
    max_position: int = 0


@dataclass
class GenerateOptions:
    max_new_tokens: int = 0
    temperature: float = 0.0
    top_k: int = 0
    seed: int = 0
    eos_token_ids: Optional[List[int]] = None


@dataclass
class GenerateResult:
    tokens: List[int] = field(default_factory=list)
    prompt_tokens: int = 0


def validate_generate_options(opts: GenerateOptions) -> None:
    """ValidateGenerateOptions (model.go:448-470)."""
    if opts.max_new_tokens < 0:
        raise ValueError("max_new_tokens must be >= 0")
    if opts.temperature < 0:
        raise ValueError("temperature must be >= 0")
    if math.isnan(opts.temperature) or math.isinf(opts.temperature):
        raise ValueError("temperature must be finite")
    if opts.top_k < 0:
        raise ValueError("top_k must be >= 0")
    eos = opts.eos_token_ids or []
    if len(eos) > MAX_EOS_TOKEN_IDS:
        raise ValueError(f"eos_token_ids length {len(eos)} exceeds limit {MAX_EOS_TOKEN_IDS}")
    if any(i < 0 for i in eos):
        raise ValueError("eos_token_ids must not contain negative ids")


def generation_needs_sampling(opts: GenerateOptions) -> bool:
    """generationNeedsSamplingScratch (model.go:1854-1856): an RNG is used."""
    return opts.max_new_tokens > 0 and opts.temperature > 0 and opts.top_k != 1


def generation_uses_argmax(opts: GenerateOptions) -> bool:
    """generationUsesArgmaxSampling (model.go:1858-1860)."""
    return opts.temperature <= 0 or opts.top_k == 1


def sampling_rng_state(opts: GenerateOptions) -> Optional[int]:
    """samplingRNGInto (model.go:1846-1852): the fastRNG state uint64(seed),
    or None when generation draws nothing."""
    return (int(opts.seed) & 0xFFFFFFFFFFFFFFFF) if generation_needs_sampling(opts) else None


def validate_generation_input(ids: Sequence[int], opts: GenerateOptions) -> None:
    """validateInputTokenIDs + validateGenerationInput (model.go:472-490)."""
    if any(i < 0 for i in ids):
        raise ValueError("input tokens must not contain negative ids")
    if opts.max_new_tokens > 0 and len(ids) == 0:
        raise ValueError("input tokens must not be empty when max_new_tokens > 0")


def expand_single_image_placeholder(ids: Sequence[int], n: int, image_token_id: int) -> List[int]:
    """expandSingleImagePlaceholderInto (model.go:2834-2859): a prompt holding
    exactly one image placeholder gets it repeated once per image embedding."""
    ids = list(ids)
    if sum(1 for t in ids if t == image_token_id) != 1 or n <= 1:
        return ids
    out: List[int] = []
    for t in ids:
        out.extend([t] * n if t == image_token_id else [t])
    return out


def multimodal_positions(ids: Sequence[int], image_grid, image_token_id: int, spatial_merge_size: int):
    """multimodalPositionsInto (model.go:1717-1783): M-RoPE (t, h, w) positions
    for a prompt whose image placeholders each stand for one merged patch of a
    (grid_t, grid_h, grid_w) image, and the rope delta for generated tokens
    (position = len(out) - 1 + delta)."""
    ids = list(ids)
    pos: List[tuple] = []
    st = 0
    next_pos = 0
    while True:
        try:
            ed = ids.index(image_token_id, st)
        except ValueError:
            break
        st_idx = next_pos
        text_len = ed - st
        pos.extend((st_idx + i,) * 3 for i in range(text_len))
        if spatial_merge_size <= 0:
            raise ValueError("config: vision_config.spatial_merge_size must be positive for image prompts")
        gt = int(image_grid[0])
        gh = int(image_grid[1]) // spatial_merge_size
        gw = int(image_grid[2]) // spatial_merge_size
        max_pos = st_idx + text_len - 1
        base = text_len + st_idx
        for t in range(gt):
            for h in range(gh):
                for w in range(gw):
                    pos.append((base + t, base + h, base + w))
                    max_pos = max(max_pos, base + t, base + h, base + w)
        next_pos = max_pos + 1
        st = ed + gt * gh * gw
    if st < len(ids):
        pos.extend((next_pos + i,) * 3 for i in range(len(ids) - st))
        next_pos = next_pos + len(ids) - st
    if not pos:
        return pos, 0
    return pos, next_pos - len(ids)


def normalize_quantization(q: str) -> str:
    q = (q or "").strip().lower()
    return q or "f32"


def select_backend(requested: str) -> str:
    """backend.Select (backend.go:85-111) restricted to this package: "cuda"
    (or "auto") needs a visible CUDA device; other backends are not here."""
    r = (requested or "auto").strip().lower()
    if r not in ("auto", "cuda"):
        raise ValueError(f"backend {requested!r} is not provided by rapidocrvl_b200 (use 'cuda')")
    n = _lib.check(_lib.load().ocrvl_device_count())
    if n <= 0:
        raise RuntimeError("no CUDA device visible for backend 'cuda'")
    return "cuda"


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Sequence_:
    """A decode sequence with its own paged KV cache on the device."""

    def __init__(self, rt: "Runtime", max_tokens: int):
        if not rt._h:
            raise RuntimeError("runtime is closed")
        self.rt = rt
        h = C.c_void_p()
        _lib.check(rt._L.ocrvl_seq_create(rt._h, int(max_tokens), C.byref(h)))
        self._h = h
        self.max_tokens = int(max_tokens)
        rt._seqs.add(self)

    def __len__(self) -> int:
        return _lib.check(self.rt._L.ocrvl_seq_len(self._h))

    def reset(self) -> None:
        _lib.check(self.rt._L.ocrvl_seq_reset(self._h))

    def close(self) -> None:
        # sequences must be released before their model (ocrvl_seq_free
        # touches the model's page pool); Runtime.close frees the live ones
        if self._h and self.rt._h:
            self.rt._L.ocrvl_seq_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def read_kv(self, layer: int):
        c = self.rt.cfg
        n = len(self)
        kvd = c.num_key_value_heads * c.head_dim
        k = np.zeros((max(n, 1), kvd), np.float32)
        v = np.zeros((max(n, 1), kvd), np.float32)
        _lib.check(self.rt._L.ocrvl_seq_read_kv(self._h, int(layer), _ptr(k), _ptr(v)))
        return k[:n], v[:n]

    def fill_synthetic(self, n: int, seed: int) -> None:
        """Sets the cache to n positions of seeded device-generated K/V
        (ocrvl_seq_fill_synthetic): the stand-in for a long prompt's prefill
        when only the decode steps after it are timed."""
        _lib.check(self.rt._L.ocrvl_seq_fill_synthetic(self._h, int(n), int(seed) & 0xFFFFFFFFFFFFFFFF))

    def import_kv(self, k, v) -> None:
        """Replaces the cache with k, v of shape [num_layers][n][kv_heads *
        head_dim] (f32) and sets the length to n (ocrvl_seq_import_kv)."""
        c = self.rt.cfg
        kvd = c.num_key_value_heads * c.head_dim
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if k.shape != v.shape or k.ndim != 3 or k.shape[0] != c.num_hidden_layers or k.shape[2] != kvd:
            raise ValueError(f"K/V must be [{c.num_hidden_layers}][n][{kvd}] f32, got {k.shape} / {v.shape}")
        _lib.check(self.rt._L.ocrvl_seq_import_kv(self._h, int(k.shape[1]), _ptr(k), _ptr(v)))


class Runtime:
    """Decoder runtime on one CUDA device (one process per GPU)."""

    def __init__(self, cfg: cfgmod.Config, opts: LoadOptions):
        cfgmod.validate_decoder(cfg)
        self.cfg = cfg
        self.backend = select_backend(opts.backend)
        self.quantization = normalize_quantization(opts.quantization)
        self._L = _lib.load()
        d = _lib.ModelDesc()
        d.vocab_size = cfg.vocab_size
        d.hidden_size = cfg.hidden_size
        d.intermediate_size = cfg.intermediate_size
        d.num_layers = cfg.num_hidden_layers
        d.num_heads = cfg.num_attention_heads
        d.num_kv_heads = cfg.num_key_value_heads
        d.head_dim = cfg.head_dim
        d.rms_norm_eps = cfg.rms_norm_eps
        d.rope_theta = cfg.rope_theta
        for i in range(3):
            d.mrope_section[i] = cfg.mrope_section[i]
        d.max_position = opts.max_position
        d.kv_pool_bytes = opts.kv_pool_bytes
        h = C.c_void_p()
        self._h = None
        self._seqs = weakref.WeakSet()
        _lib.check(self._L.ocrvl_init(int(opts.device), C.byref(d), C.byref(h)))
        self._h = h
        self.device = opts.device

    # -- loading ---------------------------------------------------------
    @classmethod
    def load(cls, model_dir: str, opts: Optional[LoadOptions] = None) -> "Runtime":
        """LoadWithOptions: config.json + model-<quant>.gguf from model_dir."""
        opts = opts or LoadOptions()
        cfg = cfgmod.load(model_dir)
        q = normalize_quantization(opts.quantization)
        if q not in ("q8", "q6", "q4"):
            raise ValueError(f"quantization {q!r} is not supported by the CUDA decode path (q8, q6, q4)")
        path = os.path.join(model_dir, f"model-{q}.gguf")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not found (convert the checkpoint to {q} GGUF first)")
        rt = cls(cfg, opts)
        rt.load_gguf(path)
        rt.finalize()
        return rt

    def load_gguf(self, path: str) -> None:
        _lib.check(self._L.ocrvl_load_gguf(self._h, path.encode()))

    def load_tensor(self, name: str, typ: int, shape, scales: Optional[np.ndarray], data: np.ndarray) -> None:
        rows = int(shape[0])
        cols = int(shape[1]) if len(shape) > 1 else 1
        data = np.ascontiguousarray(data)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        _lib.check(self._L.ocrvl_load_tensor(self._h, name.encode(), int(typ), rows, cols, _ptr(sc), _ptr(data)))

    def finalize(self) -> None:
        _lib.check(self._L.ocrvl_finalize(self._h))

    @property
    def quant_type(self) -> int:
        return _lib.check(self._L.ocrvl_quant_type(self._h))

    def trace(self) -> np.ndarray:
        """Per-phase [start, prologue end, end, barrier exit] ns of the last
        step (needs OCRVL_TRACE=1 in the environment at load time)."""
        buf = np.zeros(4 * 256, np.uint64)
        n = _lib.check(self._L.ocrvl_trace_read(self._h, _ptr(buf), len(buf)))
        return buf[:n].reshape(-1, 4)

    def close(self) -> None:
        if getattr(self, "_h", None):
            for sq in list(self._seqs):
                sq.close()
            self._L.ocrvl_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- decoding ----------------------------------------------------------
    def new_sequence(self, max_tokens: int) -> Sequence_:
        return Sequence_(self, max_tokens)

    def step(self, seqs, ids=None, embeds=None, positions=None, need_logits=True, return_logits=False):
        """One decode step over ``seqs`` (1..8 sequences).  Returns
        (ids, logits|None): greedy ids per sequence (-1 when need_logits is
        False) and optionally the full logits."""
        n = len(seqs)
        arr = (C.c_void_p * n)(*[s._h for s in seqs])
        ids_a = None if ids is None else _i32(ids)
        emb = None if embeds is None else np.ascontiguousarray(embeds, dtype=np.float32)
        pos = None if positions is None else _i32(positions).reshape(n, 3)
        out = np.zeros(n, np.int32)
        logits = np.zeros((n, self.cfg.vocab_size), np.float32) if (return_logits and need_logits) else None
        _lib.check(self._L.ocrvl_step(self._h, arr, n, _ptr(ids_a), _ptr(emb), _ptr(pos), int(bool(need_logits)),
                                      _ptr(out), _ptr(logits)))
        return out, logits

    def step_sample(self, seqs, ids=None, embeds=None, positions=None, temperature=0.0, top_k=0, rng_states=None):
        """One decode step whose next ids are drawn on the device by the
        reference's generation-loop sampler (``ocrvl_step_sample``).
        ``rng_states``: one fastRNG state per sequence (a uint64 numpy array,
        advanced in place); unused for argmax.  Returns the ids."""
        n = len(seqs)
        arr = (C.c_void_p * n)(*[s._h for s in seqs])
        ids_a = None if ids is None else _i32(ids)
        emb = None if embeds is None else np.ascontiguousarray(embeds, dtype=np.float32)
        pos = None if positions is None else _i32(positions).reshape(n, 3)
        st = None
        if rng_states is not None:
            st = rng_states
            if not (isinstance(st, np.ndarray) and st.dtype == np.uint64 and st.flags.c_contiguous and st.size == n):
                raise ValueError("rng_states must be a contiguous uint64 array with one state per sequence")
        out = np.zeros(n, np.int32)
        _lib.check(self._L.ocrvl_step_sample(self._h, arr, n, _ptr(ids_a), _ptr(emb), _ptr(pos), float(temperature),
                                             int(top_k), _ptr(st), _ptr(out)))
        return out

    def decode_device(self, seqs, first_ids, steps: int) -> np.ndarray:
        """Greedy decode of ``steps`` tokens per sequence with device-side
        token feedback (no host round trip per token).  Returns [steps, n] ids."""
        n = len(seqs)
        arr = (C.c_void_p * n)(*[s._h for s in seqs])
        first = _i32(first_ids)
        out = np.zeros((steps, n), np.int32)
        _lib.check(self._L.ocrvl_decode_greedy_device(self._h, arr, n, _ptr(first), int(steps), _ptr(out)))
        return out

    @property
    def stream_handle(self) -> int:
        return int(self._L.ocrvl_model_stream(self._h) or 0)

    def step_io_bytes(self, n: int):
        h2d, d2h = C.c_int64(), C.c_int64()
        _lib.check(self._L.ocrvl_step_io_bytes(self._h, int(n), C.byref(h2d), C.byref(d2h)))
        return h2d.value, d2h.value

    def generate(self, ids: Sequence[int], max_new: int) -> List[int]:
        return self.generate_with_options(ids, GenerateOptions(max_new_tokens=max_new)).tokens

    def generate_with_options(self, ids: Sequence[int], opts: GenerateOptions) -> GenerateResult:
        validate_generate_options(opts)
        validate_generation_input(ids, opts)
        eos = DEFAULT_EOS_TOKEN_IDS if opts.eos_token_ids is None else list(opts.eos_token_ids)
        ids_a = _i32(list(ids))
        if opts.max_new_tokens == 0:
            return GenerateResult(tokens=list(ids), prompt_tokens=len(ids))
        for t in ids_a:
            if t >= self.cfg.vocab_size:
                raise ValueError(f"token id {int(t)} outside vocab")
        out = np.zeros(len(ids_a) + opts.max_new_tokens, np.int32)
        n = C.c_int(0)
        # an explicit empty list means "no EOS" (only None selects the default)
        eos_a = _i32(eos) if eos else np.zeros(1, np.int32)
        seed = int(opts.seed) & 0xFFFFFFFFFFFFFFFF
        seed = seed - (1 << 64) if seed >= 1 << 63 else seed
        _lib.check(self._L.ocrvl_generate(self._h, _ptr(ids_a), len(ids_a), int(opts.max_new_tokens),
                                          _ptr(eos_a), len(eos), float(opts.temperature), int(opts.top_k), seed,
                                          _ptr(out), len(out), C.byref(n)))
        return GenerateResult(tokens=out[: n.value].tolist(), prompt_tokens=len(ids_a))

    def generate_with_image_embeds(self, ids: Sequence[int], image_embeds, image_grid,
                                   opts: GenerateOptions) -> GenerateResult:
        """GenerateWithImageEmbeds (model.go:1582-1707): image placeholders
        take the given embeddings (one row each, in order), M-RoPE positions
        come from :func:`multimodal_positions`, and generated tokens sit at
        len(out) - 1 + rope delta.  One ``ocrvl_step`` per token, or
        ``ocrvl_step_sample`` when the options sample."""
        validate_generate_options(opts)
        validate_generation_input(ids, opts)
        if opts.max_new_tokens == 0:
            return GenerateResult(tokens=list(ids), prompt_tokens=len(ids))
        c = self.cfg
        emb = np.ascontiguousarray(np.asarray(image_embeds, dtype=np.float32).reshape(-1, c.hidden_size))
        eos = DEFAULT_EOS_TOKEN_IDS if opts.eos_token_ids is None else list(opts.eos_token_ids)
        inp = expand_single_image_placeholder(ids, len(emb), c.image_token_id)
        positions, delta = multimodal_positions(inp, image_grid, c.image_token_id, c.spatial_merge_size)
        n_img = sum(1 for t in inp if t == c.image_token_id)
        if n_img > len(emb):
            raise ValueError(f"too many image placeholder tokens: need {len(emb)}")
        if n_img < len(emb):
            raise ValueError(f"not enough image placeholder tokens: got {n_img} need {len(emb)}")
        state = sampling_rng_state(opts)
        rng = None if state is None else np.array([state], np.uint64)

        def step(ids=None, embeds=None, pos=None, last=True):
            if last and rng is not None:
                return int(self.step_sample([seq], ids=ids, embeds=embeds, positions=[pos],
                                            temperature=opts.temperature, top_k=opts.top_k, rng_states=rng)[0])
            r, _ = self.step([seq], ids=ids, embeds=embeds, positions=[pos], need_logits=last)
            return int(r[0])

        seq = self.new_sequence(len(inp) + opts.max_new_tokens)
        try:
            cursor = 0
            nxt = -1
            for i, t in enumerate(inp):
                last = i == len(inp) - 1
                if t == c.image_token_id:
                    nxt = step(embeds=emb[cursor:cursor + 1], pos=positions[i], last=last)
                    cursor += 1
                else:
                    nxt = step(ids=[t], pos=positions[i], last=last)
            out = list(inp)
            for i in range(opts.max_new_tokens):
                out.append(nxt)
                if nxt in eos or i + 1 >= opts.max_new_tokens:
                    break
                p = len(out) - 1 + delta
                nxt = step(ids=[nxt], pos=(p, p, p))
            return GenerateResult(tokens=out, prompt_tokens=len(inp))
        finally:
            seq.close()
