"""The CPU oracle (and the numpy GGUF quantizers) against the reference's own
known-answer tests.  Each test names the reference test it restates; the
literal inputs, expected values and tolerances are the reference's.
"""
import ctypes as C
import math

import numpy as np
import pytest

from rapidocrvl_b200 import config, gguf, synth
from rapidocrvl_b200.runtime import expand_single_image_placeholder, multimodal_positions

import pyoracle
from pyoracle import ptr

W23 = np.array([[1, -2, 3], [0.5, 0.25, -0.75]], np.float32)
X3 = np.array([2, -1, 0.5], np.float32)


def _float_matvec(w, x):
    # tensor.MatVec (ops.go): plain float32 row dots
    out = np.zeros(w.shape[0], np.float32)
    for r in range(w.shape[0]):
        s = np.float32(0)
        for c in range(w.shape[1]):
            s = np.float32(s + np.float32(w[r, c] * x[c]))
        out[r] = s
    return out


def _oracle_quantize(L, typ, w):
    rows, cols = w.shape
    pb = gguf.packed_row_bytes(typ, cols)
    packed = np.zeros((rows, pb), np.uint8)
    sc = np.zeros(rows, np.float32)
    for r in range(rows):
        row = np.ascontiguousarray(w[r])
        buf = np.zeros(pb, np.uint8)
        sc[r] = L.orc_quantize_row(typ, ptr(row), cols, ptr(buf))
        packed[r] = buf
    return sc, packed


@pytest.mark.parametrize("typ,tol", [(gguf.Q8_ROW, 0.05), (gguf.Q4_ROW, 0.5), (gguf.Q6_ROW, 0.12)])
def test_matvec_approx(oracle_lib, typ, tol):
    """TestQ8MatVecApprox / TestQ4MatVecApprox / TestQ6MatVecApprox
    (internal/tensor/quant_test.go:9-24, 43-58, 68-83)."""
    want = _float_matvec(W23, X3)
    sc, packed = _oracle_quantize(oracle_lib, typ, W23)
    got = np.zeros(2, np.float32)
    oracle_lib.orc_matvec(typ, 2, 3, ptr(sc), ptr(packed), ptr(X3), ptr(got))
    assert np.all(np.abs(got - want) <= tol), (got, want)


def test_quantize_q8_bytes_match_int8(oracle_lib):
    """TestQuantizeQ8RowBytesIntoMatchesInt8 (quant_test.go:26-41): the byte
    form of a Q8 row is the int8 form reinterpreted."""
    w = np.array([[1, -2, 3, 0.5, 0.25, -0.75, 0]], np.float32)
    sc, packed = _oracle_quantize(oracle_lib, gguf.Q8_ROW, w)
    q = np.zeros(7, np.int8)
    oracle_lib.orc_unpack_row(gguf.Q8_ROW, ptr(packed[0]), 7, ptr(q))
    assert np.array_equal(q.view(np.uint8), packed[0])
    assert sc[0] == np.float32(3) / np.float32(127)
    assert q.tolist() == [42, -85, 127, 21, 11, -32, 0]


def test_q4_odd_cols_clears_tail_nibble(oracle_lib):
    """TestQuantizeQ4RowIntoOddColsClearsTailNibble (quant_test.go:60-66)."""
    data = np.array([0xFF, 0xFF], np.uint8)
    w = np.array([1, -1, 0.5], np.float32)
    oracle_lib.orc_quantize_row(gguf.Q4_ROW, ptr(w), 3, ptr(data))
    assert data[1] & 0xF0 == 0
    _, packed = gguf.quantize_rows(gguf.Q4_ROW, w[None])
    assert packed[0, 1] & 0xF0 == 0
    assert np.array_equal(packed[0], data)


def test_q6_pack_round_trip_odd_cols(oracle_lib):
    """TestQ6PackRoundTripOddCols (quant_test.go:85-97): 11 fields (i*7)&63."""
    fields = np.array([[(i * 7) & 0x3F for i in range(11)]], np.uint32)
    packed = gguf.pack_q6_fields(fields)
    assert packed.shape == (1, (11 * 6 + 7) // 8)
    assert gguf.q6_fields(packed, 11).tolist() == fields.tolist()
    out = np.zeros(11, np.int8)
    oracle_lib.orc_unpack_row(gguf.Q6_ROW, ptr(packed[0]), 11, ptr(out))
    assert (out.astype(np.int32) + 32).tolist() == fields[0].tolist()


def test_quant_helpers(oracle_lib):
    """TestQuantHelpers (quant_test.go:99-127): round half away from zero,
    the Q4 nibble tables and the Q6/Q8 value maps."""
    xs = np.array([1.49, 1.50, -1.49, -1.50, 0], np.float32)
    assert gguf._round_half_away(xs).tolist() == [1, 2, -1, -2, 0]
    lo_hi = gguf.unpack_rows(gguf.Q4_ROW, np.array([[0xF0, 0x08]], np.uint8), 4)[0]
    assert lo_hi.tolist() == [-8, 7, 0, -8]
    out = np.zeros(4, np.int8)
    oracle_lib.orc_unpack_row(gguf.Q4_ROW, ptr(np.array([0xF0, 0x08], np.uint8)), 4, ptr(out))
    assert out.tolist() == [-8, 7, 0, -8]
    q6 = gguf.unpack_rows(gguf.Q6_ROW, gguf.pack_q6_fields(np.array([[0, 32, 63]])), 3)[0]
    assert q6.tolist() == [-32, 0, 31]
    q8 = gguf.unpack_rows(gguf.Q8_ROW, np.array([[0x80, 0, 127]], np.uint8), 3)[0]
    assert q8.tolist() == [-128, 0, 127]
    w = np.array([-1, 2.5, -3, 0.25, 1, -0.5, 7, -6, 4], np.float32)
    sc, _ = _oracle_quantize(oracle_lib, gguf.Q8_ROW, w[None])
    assert sc[0] == np.float32(7) / np.float32(127)  # maxAbsFloat32 = 7


def test_vnni_core_known_answers(oracle_lib):
    """TestDotQ8VNNICoreDebug / ...Tail (internal/tensor/vnni_test.go:8-24)."""
    a = np.ones(8, np.int8)
    xq = np.full(8, 129, np.uint8)
    assert oracle_lib.orc_dot_u8s8(ptr(a), ptr(xq), 8) == 1032
    assert oracle_lib.orc_dot_u8s8(ptr(a[:3].copy()), ptr(xq[:3].copy()), 3) == 387


@pytest.mark.parametrize("n", [32, 64, 128, 256, 1024])
def test_vnni_matches_float_dot(oracle_lib, n):
    """TestDotQ8VNNICorrectness (vnni_test.go:26-54): int8-activation dot vs
    the float Q8 dot within 5 % (or 0.01 absolute)."""
    i = np.arange(n)
    w = ((i % 17) - 8).astype(np.float32)
    x = (((i % 13) - 6) / np.float32(13)).astype(np.float32)
    sc, packed = _oracle_quantize(oracle_lib, gguf.Q8_ROW, w[None])
    q = packed[0].view(np.int8).copy()
    xq = np.zeros(n, np.uint8)
    sx = oracle_lib.orc_quantize_x(ptr(x), n, ptr(xq))
    rowsum = int(q.astype(np.int32).sum())
    dot = oracle_lib.orc_dot_u8s8(ptr(q), ptr(xq), n)
    vnni = oracle_lib.orc_vnni_finalize(dot, rowsum, sx, float(sc[0]))
    ref = oracle_lib.orc_dot_q8_f32(ptr(q), ptr(x), n) * sc[0]
    assert abs(vnni - ref) <= max(abs(ref) * 0.05, 0.01)


def test_quantize_x_rules(oracle_lib):
    """quantizeXForVNNI (quant.go:2087-2115): scale = max|x|/127, xq =
    clamp(rne(x/scale) + 128); an all-zero x gives scale 1 and xq = 128."""
    x = np.array([0.0, 1.0, -1.0, 0.5, -0.25, 127 / 254], np.float32)
    xq = np.zeros(len(x), np.uint8)
    s = oracle_lib.orc_quantize_x(ptr(x), len(x), ptr(xq))
    assert s == np.float32(1) / np.float32(127)
    inv = np.float32(1) / np.float32(s)
    want = np.clip(np.rint(x * inv) + 128, 0, 255).astype(np.uint8)
    assert xq.tolist() == want.tolist()
    z = np.zeros(40, np.float32)
    zq = np.zeros(40, np.uint8)
    assert oracle_lib.orc_quantize_x(ptr(z), 40, ptr(zq)) == 1.0
    assert np.all(zq == 128)


def _scalar_mrope(x, heads, dim, pos, theta, sections=(16, 24, 24)):
    # applyMRoPE (internal/model/model.go:7363-7389): float64 angles, f32 cos/sin
    x = x.copy()
    half = dim // 2
    for h in range(heads):
        base = h * dim
        end, axis = sections[0], 0
        for i in range(half):
            while axis + 1 < len(sections) and i >= end:
                axis += 1
                end += sections[axis]
            p = pos[axis]
            ang = float(p) * math.pow(theta, -float(2 * i) / float(dim))
            cs, sn = np.float32(math.cos(ang)), np.float32(math.sin(ang))
            a, b = x[base + i], x[base + half + i]
            x[base + i] = np.float32(a * cs) - np.float32(b * sn)
            x[base + half + i] = np.float32(b * cs) + np.float32(a * sn)
    return x


def test_mrope_table_matches_scalar(oracle_lib):
    """TestRuntimeMRoPEMatchesScalarReference (internal/model/rope_test.go:10-35):
    head_dim 128, theta 1e4, sections [16,24,24], pos (7,3,11), 1e-6."""
    cfg = config.Config(**dict(synth.TINY_CONFIG, rope_theta=10000.0))
    oc = pyoracle.make_config(cfg)
    x = np.array([math.sin(i * 0.17) for i in range(2 * 128)], np.float32)
    cs = np.zeros(64, np.float32)
    sn = np.zeros(64, np.float32)
    oracle_lib.orc_rope_table(C.byref(oc), 7, 3, 11, ptr(cs), ptr(sn))
    got = x.copy()
    oracle_lib.orc_rope(ptr(got), 2, 128, ptr(cs), ptr(sn))
    want = _scalar_mrope(x, 2, 128, (7, 3, 11), 10000.0)
    assert np.max(np.abs(got - want)) <= 1e-6


def test_attention_fixture(oracle_lib):
    """TestAttentionWithNormCacheFallbackMatchesCPU's cache and projections
    (internal/model/vulkan_fallback_test.go:1578-1658): 2 query heads, 1 kv
    head, head_dim 2; cached (k, v) = ([0.25, -0.5], [1, 2]) plus the current
    token's k = x[1:3], v = x[0:2] for x = [2, -1, 0.5, 3]; 1e-5."""
    x = np.array([2, -1, 0.5, 3], np.float32)
    q = x.copy()  # identity q_proj
    k = np.array([[0.25, -0.5], [x[1], x[2]]], np.float32)
    v = np.array([[1, 2], [x[0], x[1]]], np.float32)
    out = np.zeros(4, np.float32)
    oracle_lib.orc_attention(ptr(q), ptr(k), ptr(v), 2, 2, 1, 2, ptr(out))
    want = []
    for h in range(2):
        s = np.array([np.dot(q[2 * h:2 * h + 2].astype(np.float64), k[t].astype(np.float64)) for t in range(2)])
        s = s / math.sqrt(2.0)
        p = np.exp(s - s.max())
        p /= p.sum()
        want.extend(list(p @ v.astype(np.float64)))
    assert np.max(np.abs(out - np.array(want))) <= 1e-5


def test_multimodal_positions_single_image():
    """TestMultimodalPositionsSingleImage (internal/model/position_test.go:10-33)."""
    got, delta = multimodal_positions([10, 101305, 100295, 100295, 100295, 100295, 11], [1, 4, 4], 100295, 2)
    assert got == [(0, 0, 0), (1, 1, 1), (2, 2, 2), (2, 2, 3), (2, 3, 2), (2, 3, 3), (4, 4, 4)]
    assert delta == -2


def test_multimodal_positions_multiple_images():
    """TestMultimodalPositionsMultipleImages (position_test.go:35-66)."""
    got, delta = multimodal_positions([1, 7, 7, 7, 7, 2, 3, 7, 7, 7, 7, 4], [1, 4, 4], 7, 2)
    assert got == [(0, 0, 0), (1, 1, 1), (1, 1, 2), (1, 2, 1), (1, 2, 2), (3, 3, 3), (4, 4, 4), (5, 5, 5),
                   (5, 5, 6), (5, 6, 5), (5, 6, 6), (7, 7, 7)]
    assert delta == -4


def test_multimodal_positions_text_only_and_empty():
    assert multimodal_positions([5, 6, 7], [1, 4, 4], 9, 2) == ([(0, 0, 0), (1, 1, 1), (2, 2, 2)], 0)
    assert multimodal_positions([], [1, 4, 4], 9, 2) == ([], 0)


def test_expand_single_image_placeholder():
    """expandSingleImagePlaceholderInto (model.go:2834-2859)."""
    assert expand_single_image_placeholder([1, 9, 2], 3, 9) == [1, 9, 9, 9, 2]
    assert expand_single_image_placeholder([1, 9, 9, 2], 3, 9) == [1, 9, 9, 2]  # two placeholders: unchanged
    assert expand_single_image_placeholder([1, 9, 2], 1, 9) == [1, 9, 2]


def _convert_lm_head(tmp_path, quant):
    cfg = config.loads('{"vocab_size": 2, "hidden_size": 3, "intermediate_size": 4, "num_hidden_layers": 0,'
                       ' "num_attention_heads": 1, "num_key_value_heads": 1, "head_dim": 3,'
                       ' "vision_config": {"num_hidden_layers": 0}}')
    values = np.array([1, -2, 3, 0.5, 0.25, -0.75], np.float32).reshape(2, 3)
    dst = str(tmp_path / f"model-{quant}.gguf")
    gguf.convert({"lm_head.weight": values}, dst, cfg, quant)
    return gguf.GGUFFile(dst), values


@pytest.mark.parametrize("quant,typ,nbytes,tol", [("q8", gguf.Q8_ROW, 6, 0.03), ("q4", gguf.Q4_ROW, 4, 0.25),
                                                   ("q6", gguf.Q6_ROW, 6, 0.08)])
def test_convert_round_trip(tmp_path, quant, typ, nbytes, tol):
    """TestConvertSafetensors{Q8,Q4,Q6}RoundTrip (internal/gguf/convert_test.go:15-65, 305-405)."""
    g, values = _convert_lm_head(tmp_path, quant)
    t, scales, packed, shape = g.row_quant("lm_head.weight")
    assert t == typ and shape == (2, 3) and packed.size == nbytes and scales.size == 2
    if quant == "q8":
        assert g.metadata["paddleocrvl.quantized_tensors"] == 1
        assert g.metadata["paddleocrvl.f32_tensors"] == 0
    deq = gguf.unpack_rows(typ, packed, 3).astype(np.float32) * scales[:, None]
    assert np.max(np.abs(deq - values)) <= tol


def test_numpy_quantizers_match_oracle(oracle_lib):
    """The converter's vectorised quantizers equal the oracle's scalar row
    quantizers byte for byte (odd widths, an all-zero row)."""
    rng = np.random.default_rng(5)
    for typ in (gguf.Q8_ROW, gguf.Q4_ROW, gguf.Q6_ROW):
        for cols in (1, 3, 7, 8, 33, 256, 1023):
            w = (rng.standard_normal((5, cols)) * 0.02).astype(np.float32)
            w[1] = 0
            sc_np, pk_np = gguf.quantize_rows(typ, w)
            sc_o, pk_o = _oracle_quantize(oracle_lib, typ, w)
            assert np.array_equal(sc_np.view(np.uint32), sc_o.view(np.uint32)), (typ, cols)
            assert np.array_equal(pk_np, pk_o), (typ, cols)
            un = np.zeros(cols, np.int8)
            for r in range(5):
                oracle_lib.orc_unpack_row(typ, ptr(pk_o[r]), cols, ptr(un))
                assert np.array_equal(un, gguf.unpack_rows(typ, pk_np[r:r + 1], cols)[0])
