// CPU oracle: C++ restatement of RapidAI/RapidOCRvl's Go CPU decode path.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).  Reference paths below are relative
// to the reference project root (Go module paddleocrvl-go).
//
// Float summation orders are canonical and documented per function; where the
// reference's amd64 assembly fixes an order (dotQ8FMA, sumSquaresF32FMA, the
// VNNI finalize epilogues, ropeFMA, siluMulInPlaceFMA, expF32VecFMA) the
// restatement follows it.  Work that the reference splits over GOMAXPROCS
// goroutines and then sums (fused AddRMSNorm sum of squares) uses a fixed
// partition of 8 workers.  Build with -ffp-contract=off: every fused
// multiply-add below is an explicit fmaf().
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace {

constexpr int kWorkers = 8;  // canonical GOMAXPROCS partition for fused sums

// ---------------------------------------------------------------------------
// Scalar helpers
// ---------------------------------------------------------------------------
inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

// fastRsqrtF32, internal/tensor/ops.go:1374-1381 (no FMA: Go amd64 v1).
float fast_rsqrt(float x) {
  float half = x * 0.5f;
  uint32_t i = 0x5f3759dfu - (f2u(x) >> 1);
  float y = u2f(i);
  y = y * (1.5f - (half * y) * y);
  return y * (1.5f - (half * y) * y);
}

const float kLog2e = u2f(0x3FB8AA3Bu);
const float kC1 = u2f(0x3F317218u);
const float kC2 = u2f(0x3E75FDF0u);
const float kC3 = u2f(0x3D635847u);
const float kC4 = u2f(0x3C1D955Bu);
const float kC5 = u2f(0x3AAF0217u);

// FastExpF32, internal/tensor/ops.go:1099-1112 (scalar, unfused polynomial,
// exponent added to the bit pattern).
float fast_exp(float x) {
  const float magic = 12582912.0f;
  float t = x * kLog2e;
  int32_t n = (int32_t)((t + magic) - magic);
  float f = t - (float)n;
  float f2 = f * f;
  float poly = (1.0f + kC1 * f) + f2 * ((kC2 + kC3 * f) + f2 * (kC4 + kC5 * f));
  uint32_t bits = f2u(poly) + ((uint32_t)n << 23);
  return u2f(bits);
}

// Vector exp of expF32VecFMA / siluMulInPlaceFMA (dot_amd64.s:6134-6151,
// 5670-5687): RNE range reduction, FMA Horner pairs, scale by 2^n built as
// ((n+127)<<23).
float exp_fma(float d) {
  float t = d * kLog2e;
  float n = nearbyintf(t);
  float f = t - n;
  float f2 = f * f;
  float p1 = fmaf(f, kC1, 1.0f);
  float p2 = fmaf(f, kC3, kC2);
  float p3 = fmaf(f, kC5, kC4);
  p2 = fmaf(f2, p3, p2);
  p1 = fmaf(f2, p2, p1);
  int32_t ni = (int32_t)n;
  float pow2 = u2f((uint32_t)(ni + 127) << 23);
  return p1 * pow2;
}

// 16-lane horizontal tree used by every ZMM reduction in the reference:
// VEXTRACTF64X4/VADDPS, VEXTRACTF128/VADDPS, VMOVHLPS/VADDPS, VSHUFPS/VADDSS.
float tree16(const float *v) {
  float a[8], b[4], c[2];
  for (int i = 0; i < 8; i++) a[i] = v[i] + v[i + 8];
  for (int i = 0; i < 4; i++) b[i] = a[i] + a[i + 4];
  for (int i = 0; i < 2; i++) c[i] = b[i] + b[i + 2];
  return c[0] + c[1];
}

// dotQ8FMA order (internal/tensor/dot_fma_amd64.s:666-799): 8 ZMM
// accumulators over 128-element blocks, then 64/32/16 blocks on the first
// 4/2/1 accumulators, pairwise accumulator reduce, tree16, scalar tail.
float dot_q8_f32(const int8_t *w, const float *x, int n) {
  float acc[8][16];
  memset(acc, 0, sizeof(acc));
  int c = 0;
  float s = 0.0f;
  if (n >= 16) {
    for (; n - c >= 128; c += 128)
      for (int a = 0; a < 8; a++)
        for (int l = 0; l < 16; l++)
          acc[a][l] = fmaf((float)w[c + 16 * a + l], x[c + 16 * a + l], acc[a][l]);
    for (; n - c >= 64; c += 64)
      for (int a = 0; a < 4; a++)
        for (int l = 0; l < 16; l++)
          acc[a][l] = fmaf((float)w[c + 16 * a + l], x[c + 16 * a + l], acc[a][l]);
    for (; n - c >= 32; c += 32)
      for (int a = 0; a < 2; a++)
        for (int l = 0; l < 16; l++)
          acc[a][l] = fmaf((float)w[c + 16 * a + l], x[c + 16 * a + l], acc[a][l]);
    for (; n - c >= 16; c += 16)
      for (int l = 0; l < 16; l++) acc[0][l] = fmaf((float)w[c + l], x[c + l], acc[0][l]);
    float r[16];
    for (int l = 0; l < 16; l++) {
      float z0 = acc[0][l] + acc[1][l], z2 = acc[2][l] + acc[3][l];
      float z4 = acc[4][l] + acc[5][l], z6 = acc[6][l] + acc[7][l];
      r[l] = (z0 + z2) + (z4 + z6);
    }
    s = tree16(r);
  }
  for (; c < n; c++) s = s + (float)w[c] * x[c];
  return s;
}

// sumSquaresF32FMA order (dot_amd64.s:7395-7455): 4 ZMM accumulators, slot
// = index mod 64, FMA chains; reduce (Z0+Z1)+(Z2+Z3), tree16; scalar tail.
float sum_squares(const float *x, int n) {
  float acc[4][16];
  memset(acc, 0, sizeof(acc));
  int c = 0;
  float s = 0.0f;
  if (n >= 16) {
    for (; n - c >= 128; c += 128)
      for (int k = 0; k < 8; k++)
        for (int l = 0; l < 16; l++) {
          float v = x[c + 16 * k + l];
          acc[k & 3][l] = fmaf(v, v, acc[k & 3][l]);
        }
    for (; n - c >= 32; c += 32)
      for (int k = 0; k < 2; k++)
        for (int l = 0; l < 16; l++) {
          float v = x[c + 16 * k + l];
          acc[k][l] = fmaf(v, v, acc[k][l]);
        }
    for (; n - c >= 16; c += 16)
      for (int l = 0; l < 16; l++) acc[0][l] = fmaf(x[c + l], x[c + l], acc[0][l]);
    float r[16];
    for (int l = 0; l < 16; l++) r[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
    s = tree16(r);
  }
  for (; c < n; c++) s = s + x[c] * x[c];
  return s;
}

// RMSNorm, internal/tensor/ops.go:1015-1037 with mulScaleFMA
// (dot_fma_amd64.s:1142-1228): out = (x*w)*scale.
void rmsnorm(const float *x, const float *w, int n, float eps, float *out) {
  float ss = sum_squares(x, n);
  float scale = fast_rsqrt(ss / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = (x[i] * w[i]) * scale;
}

// quantizeXForVNNI (quant.go:2087-2115 -> dot_amd64.go:228-252 ->
// dot_vnni_amd64.s:434-500): scale = max|x|/127, xq = clamp(rne(x/scale)+128).
float quantize_x(const float *x, int n, uint8_t *xq) {
  float m = 0.0f;
  for (int i = 0; i < n; i++) m = std::max(m, fabsf(x[i]));
  if (m == 0.0f) {
    memset(xq, 128, (size_t)n);
    return 1.0f;
  }
  float scale = m / 127.0f;
  float inv = 1.0f / scale;
  for (int i = 0; i < n; i++) {
    float v = nearbyintf(x[i] * inv) + 128.0f;
    v = std::min(std::max(v, 0.0f), 255.0f);
    xq[i] = (uint8_t)(int)v;
  }
  return scale;
}

// Integer dot of int8 weights with offset-128 uint8 activations (the
// VPDPBUSD core, dot_vnni_amd64.s).  Exact.
#if defined(__x86_64__)
__attribute__((target("avx512f,avx512bw,avx512vnni"))) int32_t dot_u8s8_vnni(
    const int8_t *w, const uint8_t *xq, int n) {
  __m512i acc = _mm512_setzero_si512();
  int c = 0;
  for (; c + 64 <= n; c += 64) {
    __m512i a = _mm512_loadu_si512((const void *)(xq + c));
    __m512i b = _mm512_loadu_si512((const void *)(w + c));
    acc = _mm512_dpbusd_epi32(acc, a, b);
  }
  int32_t s = _mm512_reduce_add_epi32(acc);
  for (; c < n; c++) s += (int32_t)w[c] * (int32_t)xq[c];
  return s;
}
bool have_vnni() {
  static int v = -1;
  if (v < 0) v = __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") ? 1 : 0;
  return v == 1;
}
#endif
int32_t dot_u8s8(const int8_t *w, const uint8_t *xq, int n) {
#if defined(__x86_64__)
  if (have_vnni()) return dot_u8s8_vnni(w, xq, n);
#endif
  int32_t s = 0;
  for (int c = 0; c < n; c++) s += (int32_t)w[c] * (int32_t)xq[c];
  return s;
}

// finalizeDotQ8VNNI vector lane (dot_vnni_amd64.s:1043-1090).
inline float vnni_finalize(int32_t dot, int32_t rowsum, float scale_x, float scale_w) {
  float d = (float)dot - 128.0f * (float)rowsum;
  return (d * scale_x) * scale_w;
}

// ---------------------------------------------------------------------------
// Quantized matrices (internal/tensor/quant.go:5-29)
// ---------------------------------------------------------------------------
struct QMat {
  int rows = 0, cols = 0, type = 0;
  std::vector<float> scale;
  std::vector<int8_t> w;     // unpacked int8, row-major
  std::vector<int32_t> rs;   // per-row sum of w (VNNI offset correction)
};

int packed_row_bytes(int type, int cols) {
  switch (type) {
    case ORC_Q8: return cols;
    case ORC_Q4: return (cols + 1) / 2;
    case ORC_Q6: return (cols * 6 + 7) / 8;
    case ORC_F32: return cols * 4;
  }
  return -1;
}

// getQ6, quant.go:2896-2906.
uint8_t get_q6(const uint8_t *row, int nbytes, int col) {
  int bit = col * 6, idx = bit / 8, shift = bit % 8;
  uint32_t x = row[idx];
  if (idx + 1 < nbytes) x |= (uint32_t)row[idx + 1] << 8;
  return (uint8_t)((x >> shift) & 0x3F);
}

// unpackQ4RowFast (quant.go:2358-2368) and unpackQ6RowFast (2640-2656).
void unpack_row(int type, const uint8_t *p, int cols, int8_t *out) {
  if (type == ORC_Q8) {
    memcpy(out, p, (size_t)cols);
  } else if (type == ORC_Q4) {
    for (int c = 0; c < cols; c++) {
      uint8_t b = p[c / 2];
      out[c] = (int8_t)((c & 1 ? (b >> 4) : (b & 0x0F)) - 8);
    }
  } else if (type == ORC_Q6) {
    int nb = packed_row_bytes(ORC_Q6, cols);
    int c = 0, j = 0;
    for (; c + 4 <= cols; c += 4, j += 3) {
      uint32_t v = p[j] | ((uint32_t)p[j + 1] << 8) | ((uint32_t)p[j + 2] << 16);
      out[c] = (int8_t)((v & 0x3F) - 32);
      out[c + 1] = (int8_t)(((v >> 6) & 0x3F) - 32);
      out[c + 2] = (int8_t)(((v >> 12) & 0x3F) - 32);
      out[c + 3] = (int8_t)(((v >> 18) & 0x3F) - 32);
    }
    for (; c < cols; c++) out[c] = (int8_t)(get_q6(p, nb, c) - 32);
  }
}

void build_qmat(QMat &m, int type, int rows, int cols, const float *scales, const uint8_t *data) {
  m.rows = rows; m.cols = cols; m.type = type;
  m.scale.assign(scales, scales + rows);
  m.w.resize((size_t)rows * cols);
  m.rs.assign(rows, 0);
  int pb = packed_row_bytes(type, cols);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    int8_t *o = &m.w[(size_t)r * cols];
    unpack_row(type, data + (size_t)r * pb, cols, o);
    int32_t s = 0;
    for (int c = 0; c < cols; c++) s += o[c];
    m.rs[r] = s;
  }
}

// The int8-activation path needs Unpacked+RowSum (Q4/Q6 from GGUF) and
// Cols >= 32 (quant.go:514, 895; argmax_quant.go:267); otherwise the float
// dot over the unpacked int8 weights runs (dotQ4Unpacked/dotQ6Unpacked reuse
// the Q8 dot kernel).
bool uses_vnni(const QMat &m) { return (m.type == ORC_Q4 || m.type == ORC_Q6) && m.cols >= 32; }

// matVecMaybeQuant CPU branches (model.go:7071-7088 -> quant.go:443-561).
void matvec(const QMat &m, const float *x, float *out) {
  if (uses_vnni(m)) {
    std::vector<uint8_t> xq(m.cols);
    float sx = quantize_x(x, m.cols, xq.data());
#pragma omp parallel for schedule(static)
    for (int r = 0; r < m.rows; r++)
      out[r] = vnni_finalize(dot_u8s8(&m.w[(size_t)r * m.cols], xq.data(), m.cols), m.rs[r], sx, m.scale[r]);
  } else {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < m.rows; r++)
      out[r] = dot_q8_f32(&m.w[(size_t)r * m.cols], x, m.cols) * m.scale[r];
  }
}

// Fused matvec + residual + RMSNorm (fused_matvec2.go:339-1623).  The sum of
// squares follows the reference's per-worker partials over kWorkers chunks:
//  * Q8 (float path, fused_matvec2.go:364-412): 8 scalar slots per chunk,
//    (((s0+s1)+(s2+s3))+(s4+s5))+(s6+s7), sequential tail.
//  * Q4/Q6 (VNNI finalize, dot_vnni_amd64.s:1207-1290): 16 lanes over 16-row
//    blocks, tree16; chunks shorter than 16 rows use the sequential scalar tail.
// Partials are then summed in worker order.  Returns false when a chunk has
// >=16 rows that are not a multiple of 16 (the reference's vector finalize
// leaves those rows unprocessed; such shapes are rejected here).
bool matvec_add_rmsnorm(const QMat &m, const float *x, float *residual, const float *nw,
                        float eps, bool in_place, float *norm_out) {
  int n = m.rows;
  std::vector<float> v(n);
  matvec(m, x, v.data());
  for (int i = 0; i < n; i++) v[i] = residual[i] + v[i];
  int workers = std::min(kWorkers, n);
  int chunk = (n + workers - 1) / workers;
  float ss = 0.0f;
  for (int wk = 0; wk < workers; wk++) {
    int s = wk * chunk, e = std::min(n, s + chunk);
    if (s >= e) continue;
    float part = 0.0f;
    if (!uses_vnni(m)) {
      float sl[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int i = s;
      for (; i + 7 < e; i += 8)
        for (int j = 0; j < 8; j++) sl[j] = sl[j] + v[i + j] * v[i + j];
      part = (((sl[0] + sl[1]) + (sl[2] + sl[3])) + (sl[4] + sl[5])) + (sl[6] + sl[7]);
      for (; i < e; i++) part = part + v[i] * v[i];
    } else {
      int len = e - s;
      if (len >= 16 && len % 16 != 0) return false;
      if (len < 16) {
        for (int i = s; i < e; i++) part = part + v[i] * v[i];
      } else {
        float lanes[16];
        memset(lanes, 0, sizeof(lanes));
        for (int i = s; i < e; i += 16)
          for (int l = 0; l < 16; l++) lanes[l] = lanes[l] + v[i + l] * v[i + l];
        part = tree16(lanes);
      }
    }
    ss = ss + part;
  }
  float scale = fast_rsqrt(ss / (float)n + eps);
  for (int i = 0; i < n; i++) {
    if (in_place) residual[i] = v[i];
    norm_out[i] = (v[i] * nw[i]) * scale;
  }
  return true;
}

// siluMulInPlaceFMA (dot_amd64.s:5652-5695): out = (g / (1 + exp(-g))) * u.
inline float silu_mul(float g, float u) {
  float e = exp_fma(0.0f - g);
  return (g / (e + 1.0f)) * u;
}

// SwiGLUGateUp*Scratch (quant.go:757-1000): both projections share x.
void swiglu(const QMat &g, const QMat &u, const float *x, float *out) {
  std::vector<float> gv(g.rows), uv(u.rows);
  matvec(g, x, gv.data());
  matvec(u, x, uv.data());
  for (int r = 0; r < g.rows; r++) out[r] = silu_mul(gv[r], uv[r]);
}

// ropeFMA (dot_amd64.s:5405-5440) via ApplyMRoPETable (weighted_sum.go:231).
void rope(float *x, int heads, int dim, const float *cs, const float *sn) {
  int half = dim / 2;
  for (int h = 0; h < heads; h++) {
    float *p = x + (size_t)h * dim;
    for (int i = 0; i < half; i++) {
      float a = p[i], b = p[half + i];
      p[i] = (a * cs[i]) - (b * sn[i]);
      p[half + i] = fmaf(a, sn[i], b * cs[i]);
    }
  }
}

// SoftmaxInPlace (ops.go:1199-1363) with ExpVec -> expF32VecFMA
// (dot_amd64.s:6116-6210).  For n >= 16 the vector loop covers the first
// 16*floor(n/16) entries only; the remaining entries keep their raw scores
// and are scaled by 1/sum with the rest (reference behaviour on amd64).
void softmax(float *x, int n) {
  auto mx = [](float a, float b) { return b > a ? b : a; };
  if (n <= 0) return;
  if (n == 1) { x[0] = 1.0f; return; }
  if (n == 2) {
    float a = x[0], b = x[1];
    if (a >= b) { float e = fast_exp(b - a); float inv = 1.0f / (1.0f + e); x[0] = inv; x[1] = e * inv; }
    else { float e = fast_exp(a - b); float inv = 1.0f / (1.0f + e); x[0] = e * inv; x[1] = inv; }
    return;
  }
  if (n <= 8) {
    float m = x[0];
    // max is exact in any order
    for (int i = 1; i < n; i++) m = mx(m, x[i]);
    float e[8];
    for (int i = 0; i < n; i++) e[i] = fast_exp(x[i] - m);
    float sum;
    switch (n) {
      case 3: sum = (e[0] + e[1]) + e[2]; break;
      case 4: sum = (e[0] + e[1]) + (e[2] + e[3]); break;
      case 5: sum = ((e[0] + e[1]) + (e[2] + e[3])) + e[4]; break;
      case 6: sum = ((e[0] + e[1]) + (e[2] + e[3])) + (e[4] + e[5]); break;
      case 7: sum = (((e[0] + e[1]) + (e[2] + e[3])) + (e[4] + e[5])) + e[6]; break;
      default: sum = (((e[0] + e[1]) + (e[2] + e[3])) + (e[4] + e[5])) + (e[6] + e[7]); break;
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] = e[i] * inv;
    return;
  }
  float m = -INFINITY;
  for (int i = 0; i < n; i++) m = mx(m, x[i]);
  float sum = 0.0f;
  if (n < 16) {
    for (int i = 0; i < n; i++) { float e = fast_exp(x[i] - m); x[i] = e; sum = sum + e; }
  } else {
    float lanes[16];
    memset(lanes, 0, sizeof(lanes));
    int nv = n & ~15;
    for (int i = 0; i < nv; i++) {
      float e = exp_fma(x[i] - m);
      x[i] = e;
      lanes[i & 15] = lanes[i & 15] + e;
    }
    sum = tree16(lanes);
  }
  float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

// 128-element score dot: 8 ZMM products (one element per slot) reduced as in
// dotQ8FMA; other head sizes use the same 128-slot structure.
float dot_f32(const float *a, const float *b, int n) {
  float acc[8][16];
  memset(acc, 0, sizeof(acc));
  int c = 0;
  float s = 0.0f;
  if (n >= 16) {
    for (; n - c >= 128; c += 128)
      for (int k = 0; k < 8; k++)
        for (int l = 0; l < 16; l++) acc[k][l] = fmaf(a[c + 16 * k + l], b[c + 16 * k + l], acc[k][l]);
    for (; n - c >= 16; c += 16)
      for (int l = 0; l < 16; l++) acc[0][l] = fmaf(a[c + l], b[c + l], acc[0][l]);
    float r[16];
    for (int l = 0; l < 16; l++) {
      float z0 = acc[0][l] + acc[1][l], z2 = acc[2][l] + acc[3][l];
      float z4 = acc[4][l] + acc[5][l], z6 = acc[6][l] + acc[7][l];
      r[l] = (z0 + z2) + (z4 + z6);
    }
    s = tree16(r);
  }
  for (; c < n; c++) s = s + a[c] * b[c];
  return s;
}

// Decode attention (model.go:3973-4042 / 3774-3833): per q-head h with
// kv-head h/group, scores (q.k)*1/sqrt(dim), SoftmaxInPlace (or the
// cacheAttentionLen2..6 paths, same formulas), value sum in token order:
// o = w0*v0, then o = fma(w_t, v_t, o).
void attention(const float *q, const float *kc, const float *vc, int n, int heads, int kvh,
               int dim, float *out) {
  int kvdim = kvh * dim;
  int group = heads / kvh;
  float scale = (float)(1.0 / sqrt((double)dim));
#pragma omp parallel for schedule(static)
  for (int h = 0; h < heads; h++) {
    int g = h / group;
    float *o = out + (size_t)h * dim;
    if (n == 1) {
      memcpy(o, vc + (size_t)g * dim, sizeof(float) * dim);
      continue;
    }
    std::vector<float> s(n);
    for (int t = 0; t < n; t++) s[t] = dot_f32(q + (size_t)h * dim, kc + (size_t)t * kvdim + g * dim, dim) * scale;
    softmax(s.data(), n);
    const float *v0 = vc + (size_t)g * dim;
    for (int d = 0; d < dim; d++) o[d] = s[0] * v0[d];
    for (int t = 1; t < n; t++) {
      const float *vt = vc + (size_t)t * kvdim + g * dim;
      for (int d = 0; d < dim; d++) o[d] = fmaf(s[t], vt[d], o[d]);
    }
  }
}

int argmax_matvec(const QMat &m, const float *x, float *best) {
  std::vector<float> sc(m.rows);
  matvec(m, x, sc.data());
  int bi = 0;
  float bv = sc[0];
  for (int r = 1; r < m.rows; r++)
    if (sc[r] > bv) { bv = sc[r]; bi = r; }
  if (best) *best = bv;
  return bi;
}

// ---------------------------------------------------------------------------
// Sampling (internal/model/model.go:1821-2828; internal/tensor/topk.go,
// cumsum.go, weighted_sum.go:314-328 -> dot_amd64.s:6886-6996).  The
// generation loop's CPU path (model.go:1536-1544, 3632-3642): top_k in
// [2, vocab) takes the lm_head top-k candidates (MatVecTopK*WithWork) and
// sampleCandidateScoresScratch; top_k <= 0 or >= vocab samples the full
// logits (sampleTokenScratch -> sampleFullLogitsScratch) with a weight
// scratch; temperature <= 0 or top_k == 1 is the argmax.  One RNG draw per
// sampled token.
// ---------------------------------------------------------------------------

// fastRNG.Float64 (model.go:1833-1840): splitmix64 step, top 53 bits.
double rng_float64(uint64_t &state) {
  state += 0x9e3779b97f4a7c15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  z ^= z >> 31;
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

// topKSelectWithWork (topk.go:326-347): partial selection sort, the k
// highest scores with ties to the lower id, in descending order.
void topk_select(const float *logits, int n, int k, int *ids, float *scores) {
  if (k > n) k = n;
  std::vector<int> id(n);
  std::vector<float> sc(logits, logits + n);
  for (int i = 0; i < n; i++) id[i] = i;
  for (int i = 0; i < k; i++) {
    int best = i;
    for (int j = i + 1; j < n; j++)
      if (sc[j] > sc[best] || (sc[j] == sc[best] && id[j] < id[best])) best = j;
    if (best != i) {
      std::swap(sc[i], sc[best]);
      std::swap(id[i], id[best]);
    }
  }
  for (int i = 0; i < k; i++) {
    ids[i] = id[i];
    scores[i] = sc[i];
  }
}

inline float max32_local(float a, float b) { return b > a ? b : a; }  // model.go:2468-2473

// sampleCandidateScoresSmall (model.go:1978-2034), temperature != 1, <= 4 candidates.
int sample_small(const int *ids, const float *s, int k, float inv, float mx, uint64_t &rng) {
  if (k == 0) return 0;
  if (k == 1) return ids[0];
  if (k == 2) {
    float s0 = s[0] * inv, s1 = s[1] * inv;
    if (s0 >= s1) {
      double w1 = fast_exp(s1 - s0);
      return rng_float64(rng) * (1 + w1) <= 1 ? ids[0] : ids[1];
    }
    double w0 = fast_exp(s0 - s1);
    return rng_float64(rng) * (w0 + 1) <= w0 ? ids[0] : ids[1];
  }
  double w[4];
  for (int i = 0; i < k; i++) w[i] = fast_exp(s[i] * inv - mx);
  double pick = rng_float64(rng) * (k == 3 ? (w[0] + w[1]) + w[2] : (w[0] + w[1]) + (w[2] + w[3]));
  double acc = w[0];
  if (pick <= acc) return ids[0];
  acc += w[1];
  if (pick <= acc) return ids[1];
  if (k == 3) return ids[2];
  acc += w[2];
  if (pick <= acc) return ids[2];
  return ids[3];
}

// sampleCandidateScoresTemp1Small (model.go:2140-2209), <= 4 candidates.
int sample_temp1_small(const int *ids, const float *s, int k, float mx, uint64_t &rng) {
  if (k == 0) return 0;
  if (k == 1) return ids[0];
  if (k == 2) {
    float s0 = s[0], s1 = s[1];
    if (s0 >= s1) {
      double w1 = fast_exp(s1 - s0);
      return rng_float64(rng) * (1 + w1) <= 1 ? ids[0] : ids[1];
    }
    double w0 = fast_exp(s0 - s1);
    return rng_float64(rng) * (w0 + 1) <= w0 ? ids[0] : ids[1];
  }
  float w[4];
  for (int i = 0; i < k; i++) w[i] = fast_exp(s[i] - mx);
  if (k == 3) {
    float pick = (float)rng_float64(rng) * ((w[0] + w[1]) + w[2]);
    if (pick <= w[0]) return ids[0];
    if (pick <= w[0] + w[1]) return ids[1];
    return ids[2];
  }
  float pick = (float)rng_float64(rng) * ((w[0] + w[1]) + (w[2] + w[3]));
  float acc = w[0];
  if (pick <= acc) return ids[0];
  acc += w[1];
  if (pick <= acc) return ids[1];
  acc += w[2];
  if (pick <= acc) return ids[2];
  return ids[3];
}

// sampleCandidateScoresScratch (model.go:1929-1976) with a weight scratch:
// temperature 1 -> float32 weights and sums (sampleCandidateScoresTemp1Scratch
// + pickWeightedRawFloat32, model.go:2036-2061, 2418-2462); otherwise float32
// weights summed in float64 (pickWeightedFloat32, model.go:2342-2416).
int sample_candidates(const int *ids, const float *s, int k, double temp, uint64_t &rng) {
  if (k == 0) return 0;
  if (temp == 1) {
    float mx = s[0];
    for (int i = 1; i < k; i++) mx = max32_local(mx, s[i]);
    if (k <= 4) return sample_temp1_small(ids, s, k, mx, rng);
    std::vector<float> w(k);
    float sum = 0;
    for (int i = 0; i < k; i++) {
      w[i] = fast_exp(s[i] - mx);
      sum += w[i];
    }
    float pick = (float)rng_float64(rng) * sum;
    float acc = 0;
    for (int i = 0; i < k; i++) {
      acc += w[i];
      if (pick <= acc) return ids[i];
    }
    return ids[k - 1];
  }
  float inv = (float)(1 / temp);
  float raw = s[0];
  for (int i = 1; i < k; i++) raw = max32_local(raw, s[i]);
  float mx = raw * inv;
  if (k <= 4) return sample_small(ids, s, k, inv, mx, rng);
  std::vector<float> w(k);
  double sum = 0;
  for (int i = 0; i < k; i++) {
    w[i] = fast_exp(s[i] * inv - mx);
    sum += (double)w[i];
  }
  double pick = rng_float64(rng) * sum;
  double acc = 0;
  for (int i = 0; i < k; i++) {
    acc += (double)w[i];
    if (pick <= acc) return ids[i];
  }
  return ids[k - 1];
}

// pickCumulativeFloat32 (model.go:2326-2340): binary search for the first
// cdf entry >= pick; -1 past the end.
int pick_cumulative(const float *cdf, int n, float pick) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (int)((unsigned)(lo + hi) >> 1);
    if (pick <= cdf[mid]) hi = mid;
    else lo = mid + 1;
  }
  return lo < n ? lo : -1;
}

// sampleFullLogitsScratch / sampleFullLogitsTemp1Scratch with a weight
// scratch (model.go:2215-2307): weights = ExpScaledVec(logits, 1/temp,
// -max*inv) (expScaledVecFMA: x*scale, + bias, vector exp; 16 lane sums,
// tree16), CumulativeSum (cumsum.go:9-58: one chain below 4096, else four
// blocks of ceil(n/4) with the earlier blocks' sums added), pick =
// float32(u) * sum, pickCumulativeFloat32's binary search (model.go:
// 2326-2340).  The vector kernel processes whole 16-float blocks only and
// leaves the last n % 16 weights unset (stale scratch), so only n % 16 == 0
// is restated; returns -2 otherwise.
int sample_full(const float *logits, int n, float temp, uint64_t &rng) {
  if (n < 16 || n % 16 != 0) return -2;
  float inv = temp == 1 ? 1.0f : 1.0f / temp;
  float mx = logits[0];
  for (int i = 1; i < n; i++) mx = std::max(mx, logits[i]);
  float bias = -(mx * inv);
  std::vector<float> w(n);
  float lanes[16] = {0};
  for (int i = 0; i < n; i += 16)
    for (int l = 0; l < 16; l++) {
      w[i + l] = exp_fma(logits[i + l] * inv + bias);
      lanes[l] = lanes[l] + w[i + l];
    }
  float sum = tree16(lanes);
  if (n < 4096) {
    float cs = 0;
    for (int i = 0; i < n; i++) w[i] = cs = cs + w[i];
  } else {
    int bs = (n + 3) / 4;
    float bsum[4] = {0, 0, 0, 0};
    for (int b = 0; b < 4; b++) {
      int st = b * bs, en = std::min(n, st + bs);
      float cs = 0;
      for (int i = st; i < en; i++) w[i] = cs = cs + w[i];
      if (st < en) bsum[b] = cs;
    }
    float off = bsum[0];
    for (int b = 1; b < 4; b++) {
      int st = b * bs, en = std::min(n, st + bs);
      for (int i = st; i < en; i++) w[i] = w[i] + off;
      off = off + bsum[b];
    }
  }
  float pick = (float)rng_float64(rng) * sum;
  int idx = pick_cumulative(w.data(), n, pick);
  return idx >= 0 ? idx : n - 1;
}

// First index of the maximum (the greedy path's tie rule).
int argmax_first(const float *x, int n) {
  int bi = 0;
  for (int i = 1; i < n; i++)
    if (x[i] > x[bi]) bi = i;
  return bi;
}

// The generation loop's choice of sampler (model.go:1536-1544, 1854-1868,
// 3611-3642, 7202-7205): <0 unsupported.
int sample_token(const float *logits, int n, double temperature, int top_k, uint64_t &rng) {
  if (temperature <= 0 || top_k == 1) return argmax_first(logits, n);
  if (top_k > 1 && top_k < n) {
    std::vector<int> ids(top_k);
    std::vector<float> sc(top_k);
    topk_select(logits, n, top_k, ids.data(), sc.data());
    return sample_candidates(ids.data(), sc.data(), top_k, temperature, rng);
  }
  return sample_full(logits, n, (float)temperature, rng);
}

// ---------------------------------------------------------------------------
// GGUF reader (internal/gguf/gguf.go:111-251, 435-569)
// ---------------------------------------------------------------------------
struct TensorMeta {
  std::vector<int64_t> shape;
  uint32_t type;
  uint64_t offset;
};

struct GGUF {
  FILE *f = nullptr;
  uint64_t data_start = 0;
  std::map<std::string, TensorMeta> tensors;
  ~GGUF() { if (f) fclose(f); }
};

int64_t tensor_bytes(const TensorMeta &m) {
  if (m.type == ORC_F32) {
    int64_t c = 1;
    for (auto d : m.shape) c *= d;
    return c * 4;
  }
  if (m.shape.size() != 2) return 0;
  int64_t rows = m.shape[0], cols = m.shape[1];
  int pb = packed_row_bytes((int)m.type, (int)cols);
  if (pb < 0) return 0;
  return rows * 4 + rows * (int64_t)pb;
}

bool rd(FILE *f, void *p, size_t n, uint64_t &pos) {
  if (fread(p, 1, n, f) != n) return false;
  pos += n;
  return true;
}
bool rd_str(FILE *f, std::string &s, uint64_t &pos) {
  uint64_t n;
  if (!rd(f, &n, 8, pos) || n > (16u << 20)) return false;
  s.resize(n);
  return n == 0 || rd(f, &s[0], n, pos);
}

bool gguf_open(GGUF &g, const char *path, std::string &err) {
  g.f = fopen(path, "rb");
  if (!g.f) { err = "cannot open GGUF"; return false; }
  uint64_t pos = 0;
  char magic[4];
  uint32_t ver;
  uint64_t nt, nkv;
  if (!rd(g.f, magic, 4, pos) || memcmp(magic, "GGUF", 4) != 0) { err = "bad GGUF magic"; return false; }
  if (!rd(g.f, &ver, 4, pos) || ver != 3) { err = "unsupported GGUF version"; return false; }
  if (!rd(g.f, &nt, 8, pos) || nt > (1u << 20)) { err = "GGUF tensor count too large"; return false; }
  if (!rd(g.f, &nkv, 8, pos) || nkv > (1u << 20)) { err = "GGUF metadata count too large"; return false; }
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key;
    uint32_t typ;
    if (!rd_str(g.f, key, pos) || !rd(g.f, &typ, 4, pos)) { err = "truncated GGUF metadata"; return false; }
    if (typ == 4) { uint32_t v; if (!rd(g.f, &v, 4, pos)) return false; }
    else if (typ == 10) { uint64_t v; if (!rd(g.f, &v, 8, pos)) return false; }
    else if (typ == 8) { std::string v; if (!rd_str(g.f, v, pos)) return false; }
    else { err = "unsupported GGUF metadata type"; return false; }
  }
  for (uint64_t i = 0; i < nt; i++) {
    std::string name;
    uint32_t nd;
    TensorMeta m;
    if (!rd_str(g.f, name, pos) || !rd(g.f, &nd, 4, pos) || nd > 8) { err = "bad GGUF tensor info"; return false; }
    m.shape.resize(nd);
    for (uint32_t j = 0; j < nd; j++) { uint64_t d; if (!rd(g.f, &d, 8, pos)) return false; m.shape[j] = (int64_t)d; }
    if (!rd(g.f, &m.type, 4, pos) || !rd(g.f, &m.offset, 8, pos)) { err = "bad GGUF tensor info"; return false; }
    if (g.tensors.count(name)) { err = "GGUF tensor duplicated"; return false; }
    g.tensors[name] = m;
  }
  g.data_start = (pos + 31) / 32 * 32;
  fseek(g.f, 0, SEEK_END);
  uint64_t fsz = (uint64_t)ftell(g.f);
  for (auto &kv : g.tensors) {
    int64_t sz = tensor_bytes(kv.second);
    if (sz <= 0 || g.data_start + kv.second.offset + (uint64_t)sz > fsz) {
      err = "GGUF tensor " + kv.first + " exceeds file size";
      return false;
    }
  }
  return true;
}

bool gguf_read(GGUF &g, const std::string &name, TensorMeta &m, std::vector<uint8_t> &raw, std::string &err) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) { err = "missing tensor " + name; return false; }
  m = it->second;
  int64_t sz = tensor_bytes(m);
  raw.resize((size_t)sz);
  fseeko(g.f, (off_t)(g.data_start + m.offset), SEEK_SET);
  if (fread(raw.data(), 1, (size_t)sz, g.f) != (size_t)sz) { err = "short read " + name; return false; }
  return true;
}

// ---------------------------------------------------------------------------
// Model (Runtime, model.go:63-113) and KV cache (model.go:373-379, 5593-5612)
// ---------------------------------------------------------------------------
struct Layer {
  std::vector<float> ln1, ln2;
  QMat q, k, v, o, gate, up, down;
};

struct Model {
  orc_config cfg;
  int qtype = 0;
  std::vector<float> embed, final_norm;
  QMat lm_head;
  std::vector<Layer> layers;
  std::vector<double> freq;
  std::vector<uint8_t> axis;
};

struct Seq {
  Model *m;
  int cap = 0, len = 0;
  std::vector<std::vector<float>> k, v;  // per layer [cap][kvdim]
};

// initTextRoPE (model.go:877-902).
void init_rope(Model &m) {
  int half = m.cfg.head_dim / 2;
  m.freq.resize(half);
  m.axis.resize(half);
  int sec[3] = {m.cfg.mrope_section[0], m.cfg.mrope_section[1], m.cfg.mrope_section[2]};
  int section_end = sec[0], axis = 0;
  for (int i = 0; i < half; i++) {
    while (axis + 1 < 3 && i >= section_end) { axis++; section_end += sec[axis]; }
    m.axis[i] = (uint8_t)std::min(axis, 2);
    m.freq[i] = pow(m.cfg.rope_theta, -(double)(2 * i) / (double)m.cfg.head_dim);
  }
}

// buildMRoPETable (model.go:7318-7357).
void rope_table(const Model &m, int T, int H, int W, float *cs, float *sn) {
  int half = m.cfg.head_dim / 2;
  for (int i = 0; i < half; i++) {
    int p = T;
    if (m.axis[i] == 1) p = H; else if (m.axis[i] == 2) p = W;
    double ang = (double)p * m.freq[i];
    cs[i] = (float)cos(ang);
    sn[i] = (float)sin(ang);
  }
}

void append_kv(Seq &s, int li, const float *k, const float *v) {
  int kvd = s.m->cfg.num_kv_heads * s.m->cfg.head_dim;
  if (s.len >= s.cap) {
    // kvCache.append grows the slice when under-sized.
    int ncap = std::max(1, s.cap * 2);
    for (size_t l = 0; l < s.k.size(); l++) { s.k[l].resize((size_t)ncap * kvd); s.v[l].resize((size_t)ncap * kvd); }
    s.cap = ncap;
  }
  memcpy(&s.k[li][(size_t)s.len * kvd], k, sizeof(float) * kvd);
  memcpy(&s.v[li][(size_t)s.len * kvd], v, sizeof(float) * kvd);
}

// forwardEmbeddingForSampling, CPU branches (model.go:3475-3643, 3850-4066,
// 5714-5800).  Returns 0 or <0 on a shape error.
// dump (nullable): per layer [h_in H | norm1 H | q, k, v before RoPE | head
// QH*D | h + o H | norm2 H | g I] (orc_dump_floats per layer).
int forward(Model &m, Seq &s, const float *emb, int T, int H, int W, bool need_logits,
            int *token, float *logits, float *final_out, float *dump = nullptr) {
  const orc_config &c = m.cfg;
  int hid = c.hidden_size, D = c.head_dim;
  int qrows = c.num_heads * D, kvrows = c.num_kv_heads * D;
  std::vector<float> h(emb, emb + hid), norm(hid), q(qrows), k(kvrows), v(kvrows), head(qrows),
      g(c.intermediate_size), scratch(hid), fin(hid);
  bool has_rope = T != 0 || H != 0 || W != 0;
  std::vector<float> cs(D / 2, 1.0f), sn(D / 2, 0.0f);
  if (has_rope) rope_table(m, T, H, W, cs.data(), sn.data());
  bool vnni = m.qtype != ORC_Q8;
  int cache_len = s.len;  // same for every layer
  for (int li = 0; li < c.num_layers; li++) {
    Layer &L = m.layers[li];
    bool last = li + 1 == c.num_layers;
    float *dl = dump ? dump + (size_t)li * (4 * hid + 2 * qrows + 2 * kvrows + qrows + c.intermediate_size) : nullptr;
    if (dl) memcpy(dl, h.data(), sizeof(float) * hid);
    rmsnorm(h.data(), L.ln1.data(), hid, c.rms_norm_eps, norm.data());
    if (dl) memcpy(dl + hid, norm.data(), sizeof(float) * hid);
    if (last && !need_logits) {
      // attentionCacheOnly (model.go:3650-3668)
      matvec(L.k, norm.data(), k.data());
      matvec(L.v, norm.data(), v.data());
      if (has_rope) rope(k.data(), c.num_kv_heads, D, cs.data(), sn.data());
      append_kv(s, li, k.data(), v.data());
      s.len = cache_len + 1;
      return 0;
    }
    bool in_place;
    if (cache_len == 0) {
      // first token (model.go:3857-3909): V expanded to every q-head
      matvec(L.k, norm.data(), k.data());
      matvec(L.v, norm.data(), v.data());
      if (has_rope) rope(k.data(), c.num_kv_heads, D, cs.data(), sn.data());
      append_kv(s, li, k.data(), v.data());
      int group = c.num_heads / c.num_kv_heads;
      for (int hh = 0; hh < c.num_heads; hh++) memcpy(&head[(size_t)hh * D], &v[(size_t)(hh / group) * D], sizeof(float) * D);
      in_place = !vnni;  // Q8: MatVecQ8AddRMSNorm; Q4/Q6: ...OutOnly
    } else {
      matvec(L.q, norm.data(), q.data());
      matvec(L.k, norm.data(), k.data());
      matvec(L.v, norm.data(), v.data());
      if (dl) {
        memcpy(dl + 2 * hid, q.data(), sizeof(float) * qrows);
        memcpy(dl + 2 * hid + qrows, k.data(), sizeof(float) * kvrows);
        memcpy(dl + 2 * hid + qrows + kvrows, v.data(), sizeof(float) * kvrows);
      }
      if (has_rope) {
        rope(q.data(), c.num_heads, D, cs.data(), sn.data());
        rope(k.data(), c.num_kv_heads, D, cs.data(), sn.data());
      }
      append_kv(s, li, k.data(), v.data());
      int n = cache_len + 1;
      attention(q.data(), s.k[li].data(), s.v[li].data(), n, c.num_heads, c.num_kv_heads, D, head.data());
      // cache.len <= 6 -> matVecOutAddRMSNormCPU (in place for every type);
      // longer caches -> Q8 in place, Q4/Q6 ...OutOnly (model.go:4043-4062).
      in_place = n <= 6 || !vnni;
    }
    if (dl) memcpy(dl + 2 * hid + qrows + 2 * kvrows, head.data(), sizeof(float) * qrows);
    // v = h + o and its fused-order norm; h takes v only in the in-place form
    std::vector<float> vo(h);
    if (!matvec_add_rmsnorm(L.o, head.data(), vo.data(), L.ln2.data(), c.rms_norm_eps, true, norm.data()))
      return -2;
    if (in_place) h = vo;
    if (dl) {
      memcpy(dl + 2 * hid + 2 * qrows + 2 * kvrows, vo.data(), sizeof(float) * hid);
      memcpy(dl + 3 * hid + 2 * qrows + 2 * kvrows, norm.data(), sizeof(float) * hid);
    }
    swiglu(L.gate, L.up, norm.data(), g.data());
    if (dl) memcpy(dl + 4 * hid + 2 * qrows + 2 * kvrows, g.data(), sizeof(float) * c.intermediate_size);
    if (!last) {
      if (!matvec_add_rmsnorm(L.down, g.data(), h.data(), m.layers[li + 1].ln1.data(), c.rms_norm_eps, true, scratch.data()))
        return -2;
    } else {
      if (!matvec_add_rmsnorm(L.down, g.data(), h.data(), m.final_norm.data(), c.rms_norm_eps, false, fin.data()))
        return -2;
    }
  }
  s.len = cache_len + 1;
  if (!need_logits) return 0;
  if (final_out) memcpy(final_out, fin.data(), sizeof(float) * hid);
  if (logits) matvec(m.lm_head, fin.data(), logits);
  if (token) *token = argmax_matvec(m.lm_head, fin.data(), nullptr);
  return 0;
}

thread_local std::string g_err;

}  // namespace

// ---------------------------------------------------------------------------
// C API
// ---------------------------------------------------------------------------
extern "C" {

void *orc_load(const char *path, const orc_config *cfg, char *err, int errlen) {
  auto fail = [&](const std::string &e) -> void * {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", e.c_str());
    return nullptr;
  };
  GGUF g;
  std::string e;
  if (!gguf_open(g, path, e)) return fail(e);
  Model *m = new Model();
  m->cfg = *cfg;
  const orc_config &c = *cfg;
  std::vector<uint8_t> raw;
  TensorMeta meta;
  auto load_f32 = [&](const std::string &name, std::vector<float> &out, size_t want) -> bool {
    if (!gguf_read(g, name, meta, raw, e)) return false;
    if (meta.type != ORC_F32) { e = "tensor " + name + " is not F32"; return false; }
    out.resize(raw.size() / 4);
    memcpy(out.data(), raw.data(), raw.size());
    if (out.size() != want) { e = "tensor " + name + " has wrong size"; return false; }
    return true;
  };
  auto load_q = [&](const std::string &name, QMat &out, int rows, int cols) -> bool {
    if (!gguf_read(g, name, meta, raw, e)) return false;
    if (meta.type != ORC_Q8 && meta.type != ORC_Q4 && meta.type != ORC_Q6) { e = "tensor " + name + " is not quantized"; return false; }
    if (meta.shape.size() != 2 || meta.shape[0] != rows || meta.shape[1] != cols) { e = "tensor " + name + " has wrong shape"; return false; }
    if (m->qtype == 0) m->qtype = (int)meta.type;
    if ((int)meta.type != m->qtype) { e = "mixed quantization types"; return false; }
    build_qmat(out, (int)meta.type, rows, cols, (const float *)raw.data(), raw.data() + (size_t)rows * 4);
    return true;
  };
  int H = c.hidden_size, I = c.intermediate_size, qr = c.num_heads * c.head_dim, kvr = c.num_kv_heads * c.head_dim;
  bool ok = load_f32("model.embed_tokens.weight", m->embed, (size_t)c.vocab_size * H) &&
            load_f32("model.norm.weight", m->final_norm, H) &&
            load_q("lm_head.weight", m->lm_head, c.vocab_size, H);
  m->layers.resize(c.num_layers);
  for (int i = 0; ok && i < c.num_layers; i++) {
    std::string p = "model.layers." + std::to_string(i) + ".";
    Layer &L = m->layers[i];
    ok = load_f32(p + "input_layernorm.weight", L.ln1, H) &&
         load_f32(p + "post_attention_layernorm.weight", L.ln2, H) &&
         load_q(p + "self_attn.q_proj.weight", L.q, qr, H) &&
         load_q(p + "self_attn.k_proj.weight", L.k, kvr, H) &&
         load_q(p + "self_attn.v_proj.weight", L.v, kvr, H) &&
         load_q(p + "self_attn.o_proj.weight", L.o, H, qr) &&
         load_q(p + "mlp.gate_proj.weight", L.gate, I, H) &&
         load_q(p + "mlp.up_proj.weight", L.up, I, H) &&
         load_q(p + "mlp.down_proj.weight", L.down, H, I);
  }
  if (!ok) { delete m; return fail(e); }
  init_rope(*m);
  return m;
}

void orc_free(void *model) { delete (Model *)model; }
int orc_set_threads(int n) {
  // the CPU baseline runs on every host core whatever OMP_NUM_THREADS a
  // launcher (torchrun sets 1 for multi-process jobs) put in the environment
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}
int orc_quant_type(void *model) { return ((Model *)model)->qtype; }

void *orc_seq_new(void *model, int max_tokens) {
  Model *m = (Model *)model;
  Seq *s = new Seq();
  s->m = m;
  s->cap = std::max(1, max_tokens);
  int kvd = m->cfg.num_kv_heads * m->cfg.head_dim;
  s->k.assign(m->cfg.num_layers, std::vector<float>((size_t)s->cap * kvd));
  s->v.assign(m->cfg.num_layers, std::vector<float>((size_t)s->cap * kvd));
  return s;
}
void orc_seq_free(void *seq) { delete (Seq *)seq; }
int orc_seq_len(void *seq) { return ((Seq *)seq)->len; }
int orc_seq_import_kv(void *seq, int n, const float *k, const float *v) {
  // the cache a prompt of n tokens would leave (kvCache contents,
  // model.go:373-379), given as [layer][n][kv_heads*head_dim]
  Seq *s = (Seq *)seq;
  if (n < 0 || (n > 0 && (!k || !v))) return -1;
  int kvd = s->m->cfg.num_kv_heads * s->m->cfg.head_dim;
  if (n > s->cap) {
    for (size_t l = 0; l < s->k.size(); l++) {
      s->k[l].resize((size_t)n * kvd);
      s->v[l].resize((size_t)n * kvd);
    }
    s->cap = n;
  }
  for (size_t l = 0; l < s->k.size(); l++) {
    memcpy(s->k[l].data(), k + l * (size_t)n * kvd, (size_t)n * kvd * 4);
    memcpy(s->v[l].data(), v + l * (size_t)n * kvd, (size_t)n * kvd * 4);
  }
  s->len = n;
  return 0;
}
int orc_seq_kv(void *seq, int layer, float *k, float *v) {
  Seq *s = (Seq *)seq;
  if (layer < 0 || layer >= (int)s->k.size()) return -1;
  size_t n = (size_t)s->len * s->m->cfg.num_kv_heads * s->m->cfg.head_dim;
  memcpy(k, s->k[layer].data(), n * 4);
  memcpy(v, s->v[layer].data(), n * 4);
  return s->len;
}

int orc_forward(void *model, void *seq, const float *emb, int pT, int pH, int pW, int need_logits,
                int *token, float *logits, float *final_norm) {
  return forward(*(Model *)model, *(Seq *)seq, emb, pT, pH, pW, need_logits != 0, token, logits, final_norm);
}

int orc_forward_dump(void *model, void *seq, const float *emb, int pT, int pH, int pW, int *token, float *logits,
                     float *dump) {
  return forward(*(Model *)model, *(Seq *)seq, emb, pT, pH, pW, true, token, logits, nullptr, dump);
}

int orc_embed(void *model, int id, float *out) {
  Model *m = (Model *)model;
  if (id < 0 || id >= m->cfg.vocab_size) return -1;
  memcpy(out, &m->embed[(size_t)id * m->cfg.hidden_size], sizeof(float) * m->cfg.hidden_size);
  return 0;
}

int orc_generate(void *model, const int *ids, int n_ids, int max_new, const int *eos, int n_eos,
                 int *out, int out_cap) {
  Model *m = (Model *)model;
  if (max_new < 0) return -1;
  for (int i = 0; i < n_ids; i++)
    if (ids[i] < 0 || ids[i] >= m->cfg.vocab_size) return -1;
  if (out_cap < n_ids) return -1;
  for (int i = 0; i < n_ids; i++) out[i] = ids[i];
  if (max_new == 0) return n_ids;
  if (n_ids == 0) return -1;
  static const int def_eos[1] = {2};
  if (!eos) { eos = def_eos; n_eos = 1; }
  Seq *s = (Seq *)orc_seq_new(model, n_ids + max_new);
  std::vector<float> emb(m->cfg.hidden_size);
  int tok = 0, n = n_ids, rc = 0;
  for (int p = 0; p < n_ids && rc == 0; p++) {
    orc_embed(model, ids[p], emb.data());
    rc = forward(*m, *s, emb.data(), p, p, p, p == n_ids - 1, &tok, nullptr, nullptr);
  }
  for (int i = 0; rc == 0 && i < max_new; i++) {
    if (n >= out_cap) { rc = -1; break; }
    out[n++] = tok;
    bool stop = false;
    for (int j = 0; j < n_eos; j++) stop |= tok == eos[j];
    if (stop || i + 1 >= max_new) break;
    orc_embed(model, tok, emb.data());
    int p = n - 1;
    rc = forward(*m, *s, emb.data(), p, p, p, 1, &tok, nullptr, nullptr);
  }
  orc_seq_free(s);
  return rc == 0 ? n : rc;
}

// Sampled generation (Runtime.GenerateWithOptions, model.go:1492-1572): the
// RNG state starts at uint64(seed) (samplingRNGInto, model.go:1846-1852) and
// each generated token is drawn by sample_token from the full logits.
int orc_generate_sampled(void *model, const int *ids, int n_ids, int max_new, const int *eos, int n_eos,
                         double temperature, int top_k, int64_t seed, int *out, int out_cap) {
  Model *m = (Model *)model;
  if (max_new < 0) return -1;
  for (int i = 0; i < n_ids; i++)
    if (ids[i] < 0 || ids[i] >= m->cfg.vocab_size) return -1;
  if (out_cap < n_ids) return -1;
  for (int i = 0; i < n_ids; i++) out[i] = ids[i];
  if (max_new == 0) return n_ids;
  if (n_ids == 0) return -1;
  static const int def_eos[1] = {2};
  if (!eos) { eos = def_eos; n_eos = 1; }
  const int V = m->cfg.vocab_size;
  uint64_t rng = (uint64_t)seed;
  Seq *s = (Seq *)orc_seq_new(model, n_ids + max_new);
  std::vector<float> emb(m->cfg.hidden_size), logits(V);
  int tok = 0, n = n_ids, rc = 0;
  for (int p = 0; p < n_ids && rc == 0; p++) {
    orc_embed(model, ids[p], emb.data());
    rc = forward(*m, *s, emb.data(), p, p, p, p == n_ids - 1, &tok, logits.data(), nullptr);
  }
  for (int i = 0; rc == 0 && i < max_new; i++) {
    if (n >= out_cap) { rc = -1; break; }
    tok = sample_token(logits.data(), V, temperature, top_k, rng);
    if (tok < 0) { rc = tok; break; }
    out[n++] = tok;
    bool stop = false;
    for (int j = 0; j < n_eos; j++) stop |= tok == eos[j];
    if (stop || i + 1 >= max_new) break;
    orc_embed(model, tok, emb.data());
    int p = n - 1;
    rc = forward(*m, *s, emb.data(), p, p, p, 1, &tok, logits.data(), nullptr);
  }
  orc_seq_free(s);
  return rc == 0 ? n : rc;
}

int orc_decode_steps(void *model, void *seq, int tok, int pos, int steps) {
  Model *m = (Model *)model;
  Seq *s = (Seq *)seq;
  std::vector<float> emb(m->cfg.hidden_size);
  for (int i = 0; i < steps; i++) {
    if (orc_embed(model, tok, emb.data()) != 0) return -1;
    int p = pos + i;
    if (forward(*m, *s, emb.data(), p, p, p, 1, &tok, nullptr, nullptr) != 0) return -1;
  }
  return tok;
}

// ---- op level ----
float orc_quantize_row(int type, const float *w, int cols, uint8_t *data) {
  // maxAbsFloat32 + roundToInt (quant.go:396-441): round half away from zero
  // in float32 arithmetic, then the per-type clamp and packing.
  auto round_i = [](float x) -> int { return x >= 0 ? (int)(x + 0.5f) : (int)(x - 0.5f); };
  float m = 0.0f;
  for (int i = 0; i < cols; i++) m = std::max(m, fabsf(w[i]));
  int pb = packed_row_bytes(type, cols);
  if (m == 0.0f) { memset(data, 0, (size_t)pb); return 1.0f; }
  if (type == ORC_Q8) {  // QuantizeQ8RowBytesInto, quant.go:96-137
    float scale = m / 127.0f, inv = 1.0f / scale;
    for (int i = 0; i < cols; i++) data[i] = (uint8_t)(int8_t)std::min(127, std::max(-127, round_i(w[i] * inv)));
    return scale;
  }
  if (type == ORC_Q4) {  // QuantizeQ4RowInto scalar branch, quant.go:291-355
    float scale = m / 7.0f, inv = 1.0f / scale;
    auto nib = [&](float x) { return (uint8_t)(std::min(7, std::max(-7, round_i(x))) + 8); };
    int i = 0, j = 0;
    for (; i + 1 < cols; i += 2, j++) data[j] = (uint8_t)(nib(w[i] * inv) | (nib(w[i + 1] * inv) << 4));
    if (i < cols) data[j] = nib(w[i] * inv);
    return scale;
  }
  if (type == ORC_Q6) {  // QuantizeQ6RowInto scalar branch, quant.go:201-280
    float scale = m / 31.0f, inv = 1.0f / scale;
    auto q6 = [&](float x) { return (uint8_t)(std::min(31, std::max(-31, round_i(x))) + 32); };
    memset(data, 0, (size_t)pb);
    for (int i = 0; i < cols; i++) {
      uint8_t v = q6(w[i] * inv);
      int bit = i * 6, idx = bit / 8, sh = bit % 8;
      uint32_t x = (uint32_t)(v & 0x3F) << sh;
      data[idx] |= (uint8_t)x;
      if (idx + 1 < pb) data[idx + 1] |= (uint8_t)(x >> 8);
    }
    return scale;
  }
  return 0.0f;
}

void orc_unpack_row(int type, const uint8_t *p, int cols, int8_t *out) { unpack_row(type, p, cols, out); }
float orc_quantize_x(const float *x, int n, uint8_t *xq) { return quantize_x(x, n, xq); }
int32_t orc_dot_u8s8(const int8_t *w, const uint8_t *xq, int n) { return dot_u8s8(w, xq, n); }
float orc_vnni_finalize(int32_t dot, int32_t rowsum, float scale_x, float scale_w) {
  return vnni_finalize(dot, rowsum, scale_x, scale_w);
}
float orc_dot_q8_f32(const int8_t *w, const float *x, int n) { return dot_q8_f32(w, x, n); }

static QMat make_qmat(int type, int rows, int cols, const float *scales, const void *data) {
  QMat m;
  build_qmat(m, type, rows, cols, scales, (const uint8_t *)data);
  return m;
}

void orc_matvec(int type, int rows, int cols, const float *scales, const void *data, const float *x, float *out) {
  QMat m = make_qmat(type, rows, cols, scales, data);
  matvec(m, x, out);
}

void orc_matvec_add_rmsnorm(int type, int rows, int cols, const float *scales, const void *data,
                            const float *x, float *residual, const float *nw, float eps, int in_place,
                            float *norm_out) {
  QMat m = make_qmat(type, rows, cols, scales, data);
  matvec_add_rmsnorm(m, x, residual, nw, eps, in_place != 0, norm_out);
}

void orc_swiglu(int type, int rows, int cols, const float *gs, const void *gd, const float *us,
                const void *ud, const float *x, float *out) {
  QMat g = make_qmat(type, rows, cols, gs, gd), u = make_qmat(type, rows, cols, us, ud);
  swiglu(g, u, x, out);
}

void orc_rmsnorm(const float *x, const float *w, int n, float eps, float *out) { rmsnorm(x, w, n, eps, out); }
float orc_fast_rsqrt(float x) { return fast_rsqrt(x); }
float orc_fast_exp(float x) { return fast_exp(x); }
void orc_rope(float *x, int heads, int dim, const float *c, const float *s) { rope(x, heads, dim, c, s); }
void orc_rope_table(const orc_config *cfg, int T, int H, int W, float *cs, float *sn) {
  Model m;
  m.cfg = *cfg;
  init_rope(m);
  rope_table(m, T, H, W, cs, sn);
}
void orc_softmax(float *x, int n) { softmax(x, n); }
void orc_attention(const float *q, const float *kc, const float *vc, int n, int heads, int kvh, int dim,
                   float *out) {
  attention(q, kc, vc, n, heads, kvh, dim, out);
}
double orc_rng_float64(uint64_t *state) { return rng_float64(*state); }
void orc_topk_select(const float *logits, int n, int k, int *ids, float *scores) {
  topk_select(logits, n, k, ids, scores);
}
int orc_sample_candidates(const int *ids, const float *scores, int k, double temperature, uint64_t *state) {
  return sample_candidates(ids, scores, k, temperature, *state);
}
int orc_pick_cumulative(const float *cdf, int n, float pick) { return pick_cumulative(cdf, n, pick); }
int orc_sample_full(const float *logits, int n, float temperature, uint64_t *state) {
  return sample_full(logits, n, temperature, *state);
}
int orc_sample_token(const float *logits, int n, double temperature, int top_k, uint64_t *state) {
  return sample_token(logits, n, temperature, top_k, *state);
}
int orc_argmax_matvec(int type, int rows, int cols, const float *scales, const void *data, const float *x,
                      float *best) {
  QMat m = make_qmat(type, rows, cols, scales, data);
  return argmax_matvec(m, x, best);
}

}  // extern "C"
