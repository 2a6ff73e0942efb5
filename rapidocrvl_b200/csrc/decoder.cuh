// Decode-step device code for the ERNIE text decoder of RapidAI/RapidOCRvl
// (Runtime.forwardEmbeddingForSampling, internal/model/model.go:3475-3643).
//
// Every stage is a __device__ "phase" that walks its work items with a
// grid-stride loop, so the same code runs as a standalone kernel (op tests,
// CUDA-graph step) or inside the persistent step kernel (engine.cu), where
// phases are separated by grid barriers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "numerics.cuh"

namespace ocrvl {

constexpr int kMaxBatch = 8;      // sequences per GEMV step
constexpr int kThreads = 256;     // threads per block, every phase
constexpr int kPageTokens = 16;   // tokens per KV page
constexpr int kScoreChunk = 32;   // tokens per score work item
constexpr int kPVChunk = 64;      // tokens per softmax/value work item
constexpr int kHeadDim = 128;     // head size the attention phases support
constexpr int kFusedWorkers = 8;  // reference GOMAXPROCS partition for fused sums

enum QType { QT_Q8 = 1000, QT_Q4 = 1001, QT_Q6 = 1002 };

// One quantized matrix as stored on the device: packed rows exactly as in the
// GGUF file (pitch = packed row bytes, a multiple of 16), fp32 row scales and
// the per-row sum of the int8 weights.
struct DMat {
  const uint8_t *w;
  const float *scale;
  const int32_t *rowsum;
  int rows, cols, pitch;
};

struct LayerW {
  const float *ln1, *ln2;
  DMat qkv;  // q rows, then k rows, then v rows
  DMat o, gate, up, down;
};

struct StepParams {
  int M;                   // sequences in this step
  int any_logits;          // some sequence needs lm_head this step
  int max_n;               // max over sequences of len+1
  int tok[kMaxBatch];      // input token ids (embedding rows)
  int len[kMaxBatch];      // cache length before this step's append
  int pos[kMaxBatch][3];   // M-RoPE (T, H, W) position
  int need[kMaxBatch];     // sequence needs logits / argmax
  const int *bt[kMaxBatch];// block table (page ids) of each sequence
};

struct Ctx {
  int qtype, H, I, L, QH, KVH, D, V;
  float eps, attn_scale;
  const float *embed, *final_norm;
  const LayerW *layers;
  DMat lm_head;
  const float *rope_cos, *rope_sin;  // [rope_max][D/2]
  int rope_max;
  const int *sec_axis;               // [D/2] M-RoPE axis of each frequency
  float *kv_pool;                    // pages of [L][2][KVH][16][D] f32
  long long page_floats;
  // step work buffers
  float *h, *vbuf, *qkv, *head, *g, *scores, *partial, *logits;
  unsigned long long *argkey;
  int *tok_out;
  int max_ctx, max_chunks;
  const StepParams *sp;
  unsigned *pv_count;                // [kMaxBatch][KVH] chunk arrivals
  // persistent-kernel barrier state
  unsigned *bar_count, *bar_gen;
  int *err;
  // optional step trace: per phase [start, prologue end, phase end (max over
  // blocks), barrier exit] in %globaltimer ns
  unsigned long long *trace;
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Small block-level helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (kThreads / 32) ? red[l] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int block_sum_int(int v, int *red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (kThreads / 32) ? red[l] : 0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  int r = red[0];
  __syncthreads();
  return r;
}

// sumSquaresF32FMA order (internal/tensor/dot_amd64.s:7395-7455) for n a
// multiple of 128: 64 FMA chains (slot = index mod 64), then
// (Z0+Z1)+(Z2+Z3) and the 16-lane tree.  All threads get the result.
__device__ float ss_rmsnorm(const float *x, int n, float *red) {
  if (threadIdx.x < 64) {
    float a = 0.0f;
    for (int c = threadIdx.x; c < n; c += 64) a = __fmaf_rn(x[c], x[c], a);
    red[threadIdx.x] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float r[16];
    for (int l = 0; l < 16; l++)
      r[l] = __fadd_rn(__fadd_rn(red[l], red[16 + l]), __fadd_rn(red[32 + l], red[48 + l]));
    red[64] = tree16(r);
  }
  __syncthreads();
  float s = red[64];
  __syncthreads();
  return s;
}

// Sum of squares of the fused matvec+AddRMSNorm kernels (fused_matvec2.go):
// kFusedWorkers row chunks; per chunk either 8 unfused scalar slots
// (Q8 float path, fused_matvec2.go:364-412) or 16 lanes over 16-row blocks
// with the 16-lane tree (VNNI finalize, dot_vnni_amd64.s:1207-1259); chunk
// partials added in order.  Chunks shorter than 16 rows (VNNI) are summed
// sequentially.
__device__ float ss_fused(const float *v, int n, bool vnni, float *red) {
  int workers = n < kFusedWorkers ? n : kFusedWorkers;
  int chunk = (n + workers - 1) / workers;
  int lanes = vnni ? 16 : 8;
  int t = threadIdx.x;
  if (t < workers * lanes) {
    int wk = t / lanes, l = t % lanes;
    int s = wk * chunk, e = min(n, s + chunk);
    float a = 0.0f;
    if (vnni) {
      if (e - s >= 16) {
        for (int i = s + l; i < e; i += 16) a = __fadd_rn(a, __fmul_rn(v[i], v[i]));
      }
    } else {
      int nb = (e - s) / 8 * 8;
      for (int i = s + l; i < s + nb; i += 8) a = __fadd_rn(a, __fmul_rn(v[i], v[i]));
    }
    red[t] = a;
  }
  __syncthreads();
  if (t == 0) {
    float ss = 0.0f;
    for (int wk = 0; wk < workers; wk++) {
      int s = wk * chunk, e = min(n, s + chunk);
      float part = 0.0f;
      if (s < e) {
        const float *r = red + wk * lanes;
        if (vnni) {
          if (e - s >= 16) {
            part = tree16(r);
          } else {
            for (int i = s; i < e; i++) part = __fadd_rn(part, __fmul_rn(v[i], v[i]));
          }
        } else {
          part = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                                     __fadd_rn(r[4], r[5])),
                           __fadd_rn(r[6], r[7]));
          int nb = (e - s) / 8 * 8;
          for (int i = s + nb; i < e; i++) part = __fadd_rn(part, __fmul_rn(v[i], v[i]));
        }
      }
      ss = __fadd_rn(ss, part);
    }
    red[300] = ss;
  }
  __syncthreads();
  float r = red[300];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------
// GEMV input prologue.  Every block builds the (normalised, quantised) input
// vectors of all M sequences in shared memory itself, from L2-resident fp32
// sources, so no separate norm / quantise launch is needed.
// ---------------------------------------------------------------------------
enum { PRO_PLAIN = 0, PRO_RMSNORM = 1, PRO_ADDNORM = 2 };

struct XIn {
  // VNNI types: xq (uint8, offset 128) per sequence; Q4 stores even columns
  // then odd columns.  Q8: xf fp32 per sequence.
  uint8_t *xq;
  float *xf;
  float sx[kMaxBatch];
  int sumq[kMaxBatch];
};

// Copies n floats (n % 4 == 0, 16-byte aligned) global -> shared; every
// thread issues all of its loads before its first store.  Sources are
// activations written by other blocks earlier in the step kernel, so the
// loads go to L2 (ld.global.cg), never through the non-coherent L1/texture
// path.
__device__ __forceinline__ void g2s_f32(float *dst, const float *src, int n) {
  constexpr int U = 4;
  const int n4 = n >> 2;
  for (int base = threadIdx.x; base < n4; base += kThreads * U) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      int i = base + u * kThreads;
      if (i < n4) v[u] = __ldcg((const float4 *)src + i);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      int i = base + u * kThreads;
      if (i < n4) ((float4 *)dst)[i] = v[u];
    }
  }
}

// x = (x * w) * scale over shared x, w from global (mulScaleFMA order).
__device__ __forceinline__ void norm_apply(float *x, const float *w, int n, float scale) {
  constexpr int U = 4;
  const int n4 = n >> 2;
  for (int base = threadIdx.x; base < n4; base += kThreads * U) {
    float4 wv[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      int i = base + u * kThreads;
      if (i < n4) wv[u] = __ldg((const float4 *)w + i);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      int i = base + u * kThreads;
      if (i < n4) {
        float4 xv = ((float4 *)x)[i];
        xv.x = __fmul_rn(__fmul_rn(xv.x, wv[u].x), scale);
        xv.y = __fmul_rn(__fmul_rn(xv.y, wv[u].y), scale);
        xv.z = __fmul_rn(__fmul_rn(xv.z, wv[u].z), scale);
        xv.w = __fmul_rn(__fmul_rn(xv.w, wv[u].w), scale);
        ((float4 *)x)[i] = xv;
      }
    }
  }
}

// Shared-memory layout of the prologue: [red 320 f32][tmp n f32][x area].
__device__ void gemv_prologue(int qt, int M, const float *src, int ld, int n, int mode,
                              const float *w, float eps, float *smem, XIn &xin) {
  float *red = smem;
  float *tmp = smem + 320;
  uint8_t *area = (uint8_t *)(tmp + n);
  bool vnni = qt != QT_Q8;
  xin.xq = area;
  xin.xf = (float *)area;
  for (int m = 0; m < M; m++) {
    const float *s = src + (size_t)m * ld;
    float *dst = vnni ? tmp : xin.xf + (size_t)m * n;
    g2s_f32(dst, s, n);
    __syncthreads();
    if (mode != PRO_PLAIN) {
      float ss = mode == PRO_RMSNORM ? ss_rmsnorm(dst, n, red) : ss_fused(dst, n, vnni, red);
      float scale = fast_rsqrt(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
      norm_apply(dst, w, n, scale);
      __syncthreads();
    }
    if (vnni) {
      float mx = 0.0f;
      for (int i = threadIdx.x; i < n; i += kThreads) mx = fmaxf(mx, fabsf(dst[i]));
      mx = block_max(mx, red);
      float sx = 1.0f, inv = 0.0f;
      if (mx != 0.0f) {
        sx = __fdiv_rn(mx, 127.0f);
        inv = __fdiv_rn(1.0f, sx);
      }
      uint8_t *q = xin.xq + (size_t)m * n;
      int acc = 0;
      for (int i = threadIdx.x; i < n; i += kThreads) {
        int v = 128;
        if (mx != 0.0f) {
          float f = __fadd_rn(rintf(__fmul_rn(dst[i], inv)), 128.0f);
          f = fminf(fmaxf(f, 0.0f), 255.0f);
          v = (int)f;
        }
        acc += v;
        if (qt == QT_Q4)
          q[(i & 1) * (n / 2) + (i >> 1)] = (uint8_t)v;  // even | odd halves
        else
          q[i] = (uint8_t)v;
      }
      acc = block_sum_int(acc, (int *)red);
      xin.sx[m] = sx;
      xin.sumq[m] = acc;
      __syncthreads();
    }
  }
  __syncthreads();
}

__device__ __forceinline__ size_t gemv_smem_bytes(int qt, int M, int n) {
  size_t area = qt == QT_Q8 ? (size_t)M * n * 4 : (size_t)M * n;
  return (320 + (size_t)n) * 4 + area;
}

// ---------------------------------------------------------------------------
// Row dot products over a batch of RB rows.  All RB rows' weight loads of a
// chunk are issued before any arithmetic so that each lane keeps RB 16-byte
// loads in flight.  Results: out[r][m] = finished row value (per-type
// epilogue arithmetic applied), valid on the lane with (lane % lpr) == 0.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream4(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Q4 (int8-activation mode): per 16-byte chunk, low nibbles hold even columns
// and high nibbles odd columns; dp4a of the unsigned nibbles against the even /
// odd halves of xq gives sum((q+8)*xq), corrected by 8*sum(xq).
template <int M_, int RB>
__device__ __forceinline__ void dot_q4(const DMat &A, const int *rows, int M, const XIn &x, int li, int lpr,
                                       float (*out)[M_]) {
  const int P = A.pitch, CH = P >> 4, n = A.cols;
  uint32_t acc[RB][M_];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++) acc[r][m] = 0;
  for (int k = li; k < CH; k += lpr) {
    uint4 wv[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) wv[r] = ld_stream16(A.w + (size_t)rows[r] * P + 16 * k);
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      const uint4 xe = *(const uint4 *)(x.xq + (size_t)m * n + 16 * k);
      const uint4 xo = *(const uint4 *)(x.xq + (size_t)m * n + n / 2 + 16 * k);
      const uint32_t e4[4] = {xe.x, xe.y, xe.z, xe.w}, o4[4] = {xo.x, xo.y, xo.z, xo.w};
#pragma unroll
      for (int r = 0; r < RB; r++) {
        const uint32_t wd[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          acc[r][m] = __dp4a(wd[j] & 0x0F0F0F0Fu, e4[j], acc[r][m]);
          acc[r][m] = __dp4a((wd[j] >> 4) & 0x0F0F0F0Fu, o4[j], acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const int32_t rs = A.rowsum[rows[r]];
    const float sw = A.scale[rows[r]];
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      uint32_t a = acc[r][m];
      for (int o = lpr >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      out[r][m] = vnni_finalize((int32_t)a - 8 * x.sumq[m], rs, x.sx[m], sw);
    }
  }
}

// Q6: 48-byte chunks = 64 columns = 16 little-endian 24-bit groups of four
// 6-bit fields; fields widened to bytes for dp4a, corrected by 32*sum(xq).
__device__ __forceinline__ uint32_t q6_spread(uint32_t g) {
  return (g & 0x3Fu) | ((g << 2) & 0x3F00u) | ((g << 4) & 0x3F0000u) | ((g << 6) & 0x3F000000u);
}
template <int M_, int RB>
__device__ __forceinline__ void dot_q6(const DMat &A, const int *rows, int M, const XIn &x, int li, int lpr,
                                       float (*out)[M_]) {
  const int P = A.pitch, CH = P / 48, n = A.cols;
  uint32_t acc[RB][M_];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++) acc[r][m] = 0;
  for (int k = li; k < CH; k += lpr) {
    uint4 wv[RB][3];
#pragma unroll
    for (int r = 0; r < RB; r++)
#pragma unroll
      for (int q = 0; q < 3; q++) wv[r][q] = ld_stream16(A.w + (size_t)rows[r] * P + 48 * k + 16 * q);
#pragma unroll
    for (int r = 0; r < RB; r++) {
      const uint32_t w[12] = {wv[r][0].x, wv[r][0].y, wv[r][0].z, wv[r][0].w, wv[r][1].x, wv[r][1].y,
                              wv[r][1].z, wv[r][1].w, wv[r][2].x, wv[r][2].y, wv[r][2].z, wv[r][2].w};
      uint32_t f[16];
#pragma unroll
      for (int t = 0; t < 4; t++) {
        uint32_t w0 = w[3 * t], w1 = w[3 * t + 1], w2 = w[3 * t + 2];
        f[4 * t + 0] = q6_spread(w0 & 0xFFFFFFu);
        f[4 * t + 1] = q6_spread(__funnelshift_r(w0, w1, 24) & 0xFFFFFFu);
        f[4 * t + 2] = q6_spread(__funnelshift_r(w1, w2, 16) & 0xFFFFFFu);
        f[4 * t + 3] = q6_spread(w2 >> 8);
      }
#pragma unroll
      for (int m = 0; m < M_; m++) {
        if (m >= M) break;
        const uint4 *xv = (const uint4 *)(x.xq + (size_t)m * n + 64 * k);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          uint4 xx = xv[q];
          acc[r][m] = __dp4a(f[4 * q + 0], xx.x, acc[r][m]);
          acc[r][m] = __dp4a(f[4 * q + 1], xx.y, acc[r][m]);
          acc[r][m] = __dp4a(f[4 * q + 2], xx.z, acc[r][m]);
          acc[r][m] = __dp4a(f[4 * q + 3], xx.w, acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const int32_t rs = A.rowsum[rows[r]];
    const float sw = A.scale[rows[r]];
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      uint32_t a = acc[r][m];
      for (int o = lpr >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      out[r][m] = vnni_finalize((int32_t)a - 32 * x.sumq[m], rs, x.sx[m], sw);
    }
  }
}

// Q8 (fp32-activation mode) in dotQ8FMA order (internal/tensor/
// dot_fma_amd64.s:666-799): lane t owns slots 4t..4t+3 of every 128-column
// block (accumulator t/4, ZMM lanes 4(t%4)..+3); the accumulator pairs are
// reduced with xor-4/8/16 shuffles and the 16-lane tree with xor-2/1.
template <int M_, int RB>
__device__ __forceinline__ void dot_q8(const DMat &A, const int *rows, int M, const XIn &x, int lane,
                                       float (*out)[M_]) {
  constexpr int JB = 4;
  const int n = A.cols, NB = n >> 7;
  float acc[RB][M_][4];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++)
#pragma unroll
      for (int i = 0; i < 4; i++) acc[r][m][i] = 0.0f;
  for (int j0 = 0; j0 < NB; j0 += JB) {
    uint32_t wv[RB][JB];
#pragma unroll
    for (int r = 0; r < RB; r++)
#pragma unroll
      for (int jj = 0; jj < JB; jj++)
        wv[r][jj] = (j0 + jj < NB) ? ld_stream4(A.w + (size_t)rows[r] * A.pitch + 128 * (j0 + jj) + 4 * lane) : 0u;
#pragma unroll
    for (int jj = 0; jj < JB; jj++) {
      if (j0 + jj >= NB) break;
#pragma unroll
      for (int m = 0; m < M_; m++) {
        if (m >= M) break;
        const float4 xv = *(const float4 *)(x.xf + (size_t)m * n + 128 * (j0 + jj) + 4 * lane);
#pragma unroll
        for (int r = 0; r < RB; r++) {
          const uint32_t w = wv[r][jj];
          acc[r][m][0] = __fmaf_rn((float)(int8_t)(w & 0xFF), xv.x, acc[r][m][0]);
          acc[r][m][1] = __fmaf_rn((float)(int8_t)((w >> 8) & 0xFF), xv.y, acc[r][m][1]);
          acc[r][m][2] = __fmaf_rn((float)(int8_t)((w >> 16) & 0xFF), xv.z, acc[r][m][2]);
          acc[r][m][3] = __fmaf_rn((float)(int8_t)(w >> 24), xv.w, acc[r][m][3]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const float sw = A.scale[rows[r]];
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      float v4[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float v = acc[r][m][i];
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 16));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v4[i] = v;
      }
      float s = __fadd_rn(__fadd_rn(v4[0], v4[2]), __fadd_rn(v4[1], v4[3]));
      out[r][m] = __fmul_rn(s, sw);
    }
  }
}

// Lanes per row for a matrix: Q4 chunks of 16 bytes, Q6 chunks of 48 bytes,
// Q8 always a full warp.
__device__ __forceinline__ int lanes_per_row(int qt, const DMat &A) {
  int ch = qt == QT_Q4 ? A.pitch / 16 : qt == QT_Q6 ? A.pitch / 48 : 32;
  int l = 1;
  while (l < 32 && l * 2 <= ch) l *= 2;
  return l;
}

template <int QT, int M_, int RB>
__device__ __forceinline__ void rows_dot(const DMat &A, const int *rows, int M, const XIn &x, int lane, int lpr,
                                         float (*out)[M_]) {
  if (QT == QT_Q4)
    dot_q4<M_, RB>(A, rows, M, x, lane % lpr, lpr, out);
  else if (QT == QT_Q6)
    dot_q6<M_, RB>(A, rows, M, x, lane % lpr, lpr, out);
  else
    dot_q8<M_, RB>(A, rows, M, x, lane, out);
}

// ---------------------------------------------------------------------------
// GEMV phases
// ---------------------------------------------------------------------------
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };
enum { RESID_ALWAYS = 0, RESID_ATTN = 1, RESID_NEVER = 2, RESID_MASK = 3 };

struct GemvArgs {
  DMat A, B;                // B: up matrix for EPI_SWIGLU
  int row_begin, row_end;   // rows of A to compute
  const float *src;         // input vectors [M][ld]
  int ld;
  int mode;                 // PRO_*
  const float *norm_w;
  int epi;
  float *out;               // EPI_STORE / EPI_SWIGLU: [M][ldo]
  int ldo;
  float *resid;             // EPI_RESID: residual [M][ldo] (updated when in_place[m])
  float *vout;              // EPI_RESID: v = resid + out, [M][ldo]
  int resid_mode;           // EPI_RESID: RESID_*
  int in_place_mask;        // RESID_MASK: bit m set -> update resid
  unsigned long long *argkey;  // EPI_ARGMAX: [M]
  float *logits;            // EPI_ARGMAX: optional full scores [M][ldo]
  unsigned long long *tslot;   // optional trace slot of this phase
};

// Contiguous slab of rows [lo, hi) of a GEMV owned by block `b` of `nb`; the
// same split drives the L2 prefetch of the slab.
__device__ __forceinline__ void gemv_slab(int row_begin, int row_end, int b, int nb, int &lo, int &hi) {
  long long n = row_end - row_begin;
  lo = row_begin + (int)(n * b / nb);
  hi = row_begin + (int)(n * (b + 1) / nb);
}

__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
  uintptr_t a = (uintptr_t)p & ~(uintptr_t)15;
  uintptr_t e = ((uintptr_t)p + bytes + 15) & ~(uintptr_t)15;
  for (uintptr_t o = a; o < e; o += 32768) {
    uint32_t sz = (uint32_t)((e - o) < 32768 ? (e - o) : 32768);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(o), "r"(sz) : "memory");
  }
}

// Issues L2 prefetches of block b's slab of rows [row_begin, row_end) of A
// (packed rows, scales, row sums).  Called by one thread.
__device__ __forceinline__ void prefetch_gemv_slab(const DMat &A, int row_begin, int row_end, int b, int nb) {
  int lo, hi;
  gemv_slab(row_begin, row_end, b, nb, lo, hi);
  if (hi <= lo) return;
  prefetch_l2(A.w + (size_t)lo * A.pitch, (size_t)(hi - lo) * A.pitch);
  prefetch_l2(A.scale + lo, (size_t)(hi - lo) * 4);
  prefetch_l2(A.rowsum + lo, (size_t)(hi - lo) * 4);
}

template <int QT, int M_, int RB>
__device__ void phase_gemv_t(const Ctx &c, const GemvArgs &a, int M, float *smem) {
  const int qt = QT;
  XIn x;
  gemv_prologue(qt, M, a.src, a.ld, a.A.cols, a.mode, a.norm_w, c.eps, smem, x);
  if (a.tslot && blockIdx.x == 0 && threadIdx.x == 0) a.tslot[1] = gtimer();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lpr = lanes_per_row(qt, a.A);
  const int rpw = 32 / lpr, sub = lane / lpr;
  int in_place = 0;
  if (a.epi == EPI_RESID) {
    for (int m = 0; m < M; m++) {
      bool ip;
      if (a.resid_mode == RESID_ALWAYS) {
        ip = true;
      } else if (a.resid_mode == RESID_NEVER) {
        ip = false;
      } else if (a.resid_mode == RESID_MASK) {
        ip = (a.in_place_mask >> m) & 1;
      } else {
        // MatVecQ8AddRMSNorm is always in place; Q4/Q6 use the in-place form
        // only for caches of 2..6 tokens (matVecOutAddRMSNormCPU) and the
        // ...OutOnly form for the first token and longer caches
        // (model.go:3896-3908, 3975-3992, 4043-4062).
        int len = c.sp->len[m];
        ip = qt == QT_Q8 || (len >= 1 && len + 1 <= 6);
      }
      in_place |= (ip ? 1 : 0) << m;
    }
  }
  int blo, bhi, lo, hi;
  gemv_slab(a.row_begin, a.row_end, blockIdx.x, gridDim.x, blo, bhi);
  gemv_slab(blo, bhi, warp, kThreads / 32, lo, hi);  // this warp's contiguous rows
  const int per_group = rpw * RB;
  const int ngroups = (hi - lo + per_group - 1) / per_group;
  unsigned long long best[M_];
#pragma unroll
  for (int m = 0; m < M_; m++) best[m] = 0ull;
  for (int gi = 0; gi < ngroups; gi++) {
    int rows[RB];
    bool valid[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) {
      int row = lo + gi * per_group + r * rpw + sub;
      valid[r] = row < hi;
      rows[r] = valid[r] ? row : hi - 1;
    }
    float v[RB][M_], u[RB][M_];
    rows_dot<QT, M_, RB>(a.A, rows, M, x, lane, lpr, v);
    if (a.epi == EPI_SWIGLU) rows_dot<QT, M_, RB>(a.B, rows, M, x, lane, lpr, u);
    if ((lane % lpr) != 0) continue;
#pragma unroll
    for (int r = 0; r < RB; r++) {
      if (!valid[r]) continue;
      const int row = rows[r];
#pragma unroll
      for (int m = 0; m < M_; m++) {
        if (m >= M) break;
        size_t o = (size_t)m * a.ldo + row;
        if (a.epi == EPI_STORE) {
          a.out[o] = v[r][m];
        } else if (a.epi == EPI_RESID) {
          float t = __fadd_rn(__ldcg(a.resid + o), v[r][m]);
          a.vout[o] = t;
          if ((in_place >> m) & 1) a.resid[o] = t;
        } else if (a.epi == EPI_SWIGLU) {
          a.out[o] = silu_mul(v[r][m], u[r][m]);
        } else {
          if (a.logits) a.logits[o] = v[r][m];
          unsigned long long k = argmax_key(v[r][m], row);
          best[m] = k > best[m] ? k : best[m];
        }
      }
    }
  }
  if (a.epi == EPI_ARGMAX) {
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      unsigned long long k = best[m];
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
        k = t > k ? t : k;
      }
      if (lane == 0 && k) atomicMax(a.argkey + m, k);
    }
  }
  __syncthreads();
}

// Rows per warp batch: enough 16-byte loads in flight per lane at M = 1,
// fewer as the per-row accumulator count grows with M.
template <int QT>
__device__ void phase_gemv_q(const Ctx &c, const GemvArgs &a, int M, float *smem) {
  constexpr int R1 = QT == QT_Q4 ? 8 : 4;
  if (M <= 1)
    phase_gemv_t<QT, 1, R1>(c, a, M, smem);
  else if (M <= 2)
    phase_gemv_t<QT, 2, R1 / 2>(c, a, M, smem);
  else if (M <= 4)
    phase_gemv_t<QT, 4, (R1 / 4 > 0 ? R1 / 4 : 1)>(c, a, M, smem);
  else
    phase_gemv_t<QT, 8, 1>(c, a, M, smem);
}

__device__ void phase_gemv(const Ctx &c, const GemvArgs &a, int M, float *smem) {
  if (c.qtype == QT_Q4)
    phase_gemv_q<QT_Q4>(c, a, M, smem);
  else if (c.qtype == QT_Q6)
    phase_gemv_q<QT_Q6>(c, a, M, smem);
  else
    phase_gemv_q<QT_Q8>(c, a, M, smem);
}

// ---------------------------------------------------------------------------
// Embedding gather (tokenEmbeddingInto, model.go:3251-3258)
// ---------------------------------------------------------------------------
__device__ void phase_embed(const Ctx &c) {
  const StepParams &sp = *c.sp;
  size_t total = (size_t)sp.M * c.H;
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < total; i += (size_t)gridDim.x * kThreads) {
    int m = (int)(i / c.H), j = (int)(i % c.H);
    c.h[i] = c.embed[(size_t)sp.tok[m] * c.H + j];
  }
}

__device__ __forceinline__ float *kv_ptr(const Ctx &c, const int *bt, int layer, int kind, int kvh, int t) {
  int page = bt[t / kPageTokens];
  return c.kv_pool + (size_t)page * c.page_floats +
         ((((size_t)layer * 2 + kind) * c.KVH + kvh) * kPageTokens + (t % kPageTokens)) * c.D;
}

// ropeFMA (internal/tensor/dot_amd64.s:5405-5440): a' = a*c - b*s,
// b' = fma(a, s, b*c) over pairs (i, i+D/2) of a head.
__device__ __forceinline__ void rope_pair(float &a, float &b, float cs, float sn) {
  float na = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
  float nb = __fmaf_rn(a, sn, __fmul_rn(b, cs));
  a = na;
  b = nb;
}

// ---------------------------------------------------------------------------
// Attention phase 1: RoPE of q/k, KV append, scores.
// Items: (sequence, kv head, chunk of kScoreChunk tokens).  The item whose
// chunk holds the new token appends its rotated k and its v to the paged
// cache (kvCache.append, model.go:5593-5612).  Scores restate
// cacheAttentionScores (model.go:4623-4795): (q.k)*1/sqrt(D), the dot in
// the 8x16-slot order of the reference's 128-wide dot kernels.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope4(float4 &a, float4 &b, const float *cs, const float *sn) {
  float ax[4] = {a.x, a.y, a.z, a.w}, bx[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 4; j++) rope_pair(ax[j], bx[j], cs[j], sn[j]);
  a = make_float4(ax[0], ax[1], ax[2], ax[3]);
  b = make_float4(bx[0], bx[1], bx[2], bx[3]);
}

// cos/sin of frequencies i4*4 .. i4*4+3 for the M-RoPE position triple.
__device__ __forceinline__ void rope_cs4(const Ctx &c, const int *pos, int i4, float *cs, float *sn) {
  const int half = c.D / 2;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int i = i4 * 4 + j;
    int p = pos[c.sec_axis[i]];
    cs[j] = c.rope_cos[(size_t)p * half + i];
    sn[j] = c.rope_sin[(size_t)p * half + i];
  }
}

__device__ void phase_scores(const Ctx &c, int layer, bool append_only, float *smem) {
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH, D = c.D, H4 = D / 8;  // H4: float4 per half head
  const int qkvld = (c.QH + 2 * c.KVH) * D;
  const int nchunk = (sp.max_n + kScoreChunk - 1) / kScoreChunk;
  const int items = sp.M * c.KVH * nchunk;
  float *qs = smem;                       // [G][D]
  float *ks = smem + G * D;               // [kScoreChunk][D+1]
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    int m = it / (c.KVH * nchunk), rem = it % (c.KVH * nchunk);
    int g = rem / nchunk, ch = rem % nchunk;
    int len = sp.len[m], n = len + 1;
    int t0 = ch * kScoreChunk;
    if (t0 >= n) continue;
    int t1 = min(n, t0 + kScoreChunk);
    if (append_only && len >= t1) continue;
    const int *pos = sp.pos[m];
    const bool has_rope = pos[0] != 0 || pos[1] != 0 || pos[2] != 0;
    const float *qkv = c.qkv + (size_t)m * qkvld;
    // q heads of this group, rotated: task = (head, float4 index of the first half)
    if (!append_only) {
      for (int p = threadIdx.x; p < G * H4; p += kThreads) {
        int hh = p / H4, i4 = p % H4;
        const float4 *qh = (const float4 *)(qkv + (size_t)(g * G + hh) * D);
        float4 a = __ldcg(qh + i4), b = __ldcg(qh + i4 + H4);
        if (has_rope) {
          float cs[4], sn[4];
          rope_cs4(c, pos, i4, cs, sn);
          rope4(a, b, cs, sn);
        }
        ((float4 *)(qs + hh * D))[i4] = a;
        ((float4 *)(qs + hh * D))[i4 + H4] = b;
      }
    }
    // keys of the chunk (2 tasks per thread, loads first); the new token's
    // key comes from the projection output and is appended with its value
    {
      const int ntask = (t1 - t0) * H4;
      constexpr int U = 2;
      for (int base = threadIdx.x; base < ntask; base += kThreads * U) {
        float4 ka[U], kb[U];
        int tt[U], i4s[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
          int p = base + u * kThreads;
          tt[u] = -1;
          if (p < ntask) {
            tt[u] = p / H4;
            i4s[u] = p % H4;
            int t = t0 + tt[u];
            const float4 *src = (t == len) ? (const float4 *)(qkv + (size_t)(c.QH + g) * D)
                                           : (const float4 *)kv_ptr(c, sp.bt[m], layer, 0, g, t);
            ka[u] = __ldcg(src + i4s[u]);
            kb[u] = __ldcg(src + i4s[u] + H4);
          }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
          if (tt[u] < 0) continue;
          int t = t0 + tt[u], i4 = i4s[u];
          if (t == len) {
            if (has_rope) {
              float cs[4], sn[4];
              rope_cs4(c, pos, i4, cs, sn);
              rope4(ka[u], kb[u], cs, sn);
            }
            float4 *kd = (float4 *)kv_ptr(c, sp.bt[m], layer, 0, g, t);
            kd[i4] = ka[u];
            kd[i4 + H4] = kb[u];
            const float4 *vh = (const float4 *)(qkv + (size_t)(c.QH + c.KVH + g) * D);
            float4 *vd = (float4 *)kv_ptr(c, sp.bt[m], layer, 1, g, t);
            vd[i4] = __ldcg(vh + i4);
            vd[i4 + H4] = __ldcg(vh + i4 + H4);
          }
          float *kr = ks + tt[u] * (D + 1) + i4 * 4;
          kr[0] = ka[u].x; kr[1] = ka[u].y; kr[2] = ka[u].z; kr[3] = ka[u].w;
          float *kr2 = kr + D / 2;
          kr2[0] = kb[u].x; kr2[1] = kb[u].y; kr2[2] = kb[u].z; kr2[3] = kb[u].w;
        }
      }
    }
    __syncthreads();
    if (!append_only) {
      for (int p = threadIdx.x; p < G * kScoreChunk; p += kThreads) {
        int hh = p / kScoreChunk, tt = p % kScoreChunk, t = t0 + tt;
        if (t >= t1) continue;
        const float *q = qs + hh * D;
        const float *k = ks + tt * (D + 1);
        float r[16];
#pragma unroll
        for (int l = 0; l < 16; l++) {
          float p0 = __fmul_rn(q[l], k[l]), p1 = __fmul_rn(q[16 + l], k[16 + l]);
          float p2 = __fmul_rn(q[32 + l], k[32 + l]), p3 = __fmul_rn(q[48 + l], k[48 + l]);
          float p4 = __fmul_rn(q[64 + l], k[64 + l]), p5 = __fmul_rn(q[80 + l], k[80 + l]);
          float p6 = __fmul_rn(q[96 + l], k[96 + l]), p7 = __fmul_rn(q[112 + l], k[112 + l]);
          r[l] = __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3)),
                           __fadd_rn(__fadd_rn(p4, p5), __fadd_rn(p6, p7)));
        }
        float sc = __fmul_rn(tree16(r), c.attn_scale);
        c.scores[((size_t)m * c.QH + g * G + hh) * c.max_ctx + t] = sc;
      }
    }
    __syncthreads();
  }
}

// Softmax statistics of one head (SoftmaxInPlace, ops.go:1199-1363, and the
// cacheAttentionLen2..6 paths of model.go:4797-5081).  `mode` tells how a
// score becomes its weight:
//   0: fast_exp(s-m)*inv, 1: exp_fma(s-m)*inv for t < nv, raw s*inv above,
//   2: n == 2 special form, 3: n == 1 (weight 1).
struct SMStats {
  float m, inv;
  int mode, nv;
};

__device__ __forceinline__ float sm_weight(const SMStats &st, const float *s, int t, int n) {
  if (st.mode == 3) return 1.0f;
  if (st.mode == 2) {
    float a = __ldcg(s), b = __ldcg(s + 1);
    if (a >= b) {
      float e = fast_exp(__fsub_rn(b, a));
      float inv = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
      return t == 0 ? inv : __fmul_rn(e, inv);
    }
    float e = fast_exp(__fsub_rn(a, b));
    float inv = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return t == 0 ? __fmul_rn(e, inv) : inv;
  }
  const float v = __ldcg(s + t);
  if (st.mode == 0) return __fmul_rn(fast_exp(__fsub_rn(v, st.m)), st.inv);
  if (t < st.nv) return __fmul_rn(exp_fma(__fsub_rn(v, st.m)), st.inv);
  return __fmul_rn(v, st.inv);
}

// Statistics of one head computed by one warp.  For n >= 16 the 16 lane
// chains of expF32VecFMA are kept exactly: lane l < 16 adds the exponentials
// of tokens l, l+16, l+32, ... in order (two per 32-token step).
__device__ SMStats warp_softmax_stats(const float *s, int n) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int t0 = 0; t0 < n; t0 += 128) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      int t = t0 + 32 * u + lane;
      v[u] = t < n ? __ldcg(s + t) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) mx = fmaxf(mx, v[u]);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  SMStats st;
  st.m = mx;
  st.nv = 0;
  if (n >= 16) {
    const int nv = n & ~15;
    float acc = 0.0f;
    for (int t0 = 0; t0 < nv; t0 += 128) {
      float e[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        int t = t0 + 32 * u + lane;
        e[u] = t < nv ? exp_fma(__fsub_rn(__ldcg(s + t), mx)) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        float hi = __shfl_down_sync(0xffffffffu, e[u], 16);
        if (t0 + 32 * u < nv) {
          acc = __fadd_rn(acc, e[u]);
          if (t0 + 32 * u + 16 < nv) acc = __fadd_rn(acc, hi);
        }
      }
    }
    float lanes[16];
#pragma unroll
    for (int l = 0; l < 16; l++) lanes[l] = __shfl_sync(0xffffffffu, acc, l);
    st.inv = __fdiv_rn(1.0f, tree16(lanes));
    st.mode = 1;
    st.nv = nv;
    return st;
  }
  if (n == 1) {
    st.mode = 3;
    st.inv = 1.0f;
    return st;
  }
  if (n == 2) {
    st.mode = 2;
    st.inv = 1.0f;
    return st;
  }
  float e[15];
  for (int t = 0; t < n; t++) e[t] = fast_exp(__fsub_rn(__ldcg(s + t), mx));
  float sum;
  if (n <= 8) {
    float p01 = __fadd_rn(e[0], e[1]);
    switch (n) {
      case 3: sum = __fadd_rn(p01, e[2]); break;
      case 4: sum = __fadd_rn(p01, __fadd_rn(e[2], e[3])); break;
      case 5: sum = __fadd_rn(__fadd_rn(p01, __fadd_rn(e[2], e[3])), e[4]); break;
      case 6: sum = __fadd_rn(__fadd_rn(p01, __fadd_rn(e[2], e[3])), __fadd_rn(e[4], e[5])); break;
      case 7:
        sum = __fadd_rn(__fadd_rn(__fadd_rn(p01, __fadd_rn(e[2], e[3])), __fadd_rn(e[4], e[5])), e[6]);
        break;
      default:
        sum = __fadd_rn(__fadd_rn(__fadd_rn(p01, __fadd_rn(e[2], e[3])), __fadd_rn(e[4], e[5])),
                        __fadd_rn(e[6], e[7]));
        break;
    }
  } else {
    sum = 0.0f;
    for (int t = 0; t < n; t++) sum = __fadd_rn(sum, e[t]);
  }
  st.inv = __fdiv_rn(1.0f, sum);
  st.mode = 0;
  return st;
}

// ---------------------------------------------------------------------------
// Attention phase 2: softmax weights, value partial sums and head outputs.
// Items: (sequence, kv head, chunk of kPVChunk tokens).  Each item derives
// the softmax statistics of its G heads from all scores (one warp per head),
// writes partial[m][h][chunk][d] = sum over its tokens of w_t * v_t[d] (token
// order), and the last item to finish a (sequence, kv head) adds the partials
// of its heads in chunk order into the head output.
// ---------------------------------------------------------------------------
__device__ void phase_pv(const Ctx &c, int layer, float *smem) {
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH, D = c.D;
  const int nchunk = (sp.max_n + kPVChunk - 1) / kPVChunk;
  const int items = sp.M * c.KVH * nchunk;
  SMStats *st = (SMStats *)smem;                      // 8 entries
  float *wts = smem + 32;                             // [G][kPVChunk]
  float *vs = wts + 8 * kPVChunk;                     // [kPVChunk][D]
  __shared__ int last_flag;
  const int warp = threadIdx.x >> 5;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    int m = it / (c.KVH * nchunk), rem = it % (c.KVH * nchunk);
    int g = rem / nchunk, ch = rem % nchunk;
    int n = sp.len[m] + 1;
    int nch = (n + kPVChunk - 1) / kPVChunk;
    int t0 = ch * kPVChunk;
    if (t0 >= n) continue;
    int t1 = min(n, t0 + kPVChunk), cnt = t1 - t0;
    const float *sc = c.scores + ((size_t)m * c.QH + g * G) * c.max_ctx;
    // value rows of the chunk (loads issued first)
    {
      constexpr int U = 8;
      const int ntask = cnt * (D / 4);
      for (int base = threadIdx.x; base < ntask; base += kThreads * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
          int p = base + u * kThreads;
          if (p < ntask) v[u] = __ldcg((const float4 *)kv_ptr(c, sp.bt[m], layer, 1, g, t0 + p / (D / 4)) + p % (D / 4));
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
          int p = base + u * kThreads;
          if (p < ntask) ((float4 *)vs)[p] = v[u];
        }
      }
    }
    if (warp < G) {
      SMStats s = warp_softmax_stats(sc + (size_t)warp * c.max_ctx, n);
      if ((threadIdx.x & 31) == 0) st[warp] = s;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < G * cnt; p += kThreads) {
      int hh = p / cnt, tt = p % cnt;
      wts[hh * kPVChunk + tt] = sm_weight(st[hh], sc + (size_t)hh * c.max_ctx, t0 + tt, n);
    }
    __syncthreads();
    for (int p = threadIdx.x; p < G * D; p += kThreads) {
      int hh = p / D, d = p % D;
      const float *w = wts + hh * kPVChunk;
      float acc = __fmul_rn(w[0], vs[d]);
      for (int tt = 1; tt < cnt; tt++) acc = __fmaf_rn(w[tt], vs[tt * D + d], acc);
      c.partial[(((size_t)m * c.QH + g * G + hh) * c.max_chunks + ch) * D + d] = acc;
    }
    // last chunk item of (m, g) to finish reduces the partials
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned *cnt_p = c.pv_count + m * c.KVH + g;
      unsigned done = atomicAdd(cnt_p, 1u);
      last_flag = done == (unsigned)(nch - 1);
      if (last_flag) atomicExch(cnt_p, 0u);
    }
    __syncthreads();
    if (last_flag) {
      __threadfence();
      for (int p = threadIdx.x; p < G * D; p += kThreads) {
        int hh = p / D, d = p % D;
        const float *pp = c.partial + (((size_t)m * c.QH + g * G + hh) * c.max_chunks) * D + d;
        float acc = __ldcg(pp);
        for (int k = 1; k < nch; k++) acc = __fadd_rn(acc, __ldcg(pp + (size_t)k * D));
        c.head[((size_t)m * c.QH + g * G + hh) * D + d] = acc;
      }
    }
    __syncthreads();
  }
}

// Normalised output of a fused AddRMSNorm (the normOut vector of
// MatVec*AddRMSNorm[OutOnly]) for M sequences; one block per sequence.
__device__ void phase_addnorm_out(const Ctx &c, const float *v, int n, int M, const float *w, float *out,
                                  float *smem) {
  float *red = smem, *tmp = smem + 320;
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    for (int i = threadIdx.x; i < n; i += kThreads) tmp[i] = v[(size_t)m * n + i];
    __syncthreads();
    float ss = ss_fused(tmp, n, c.qtype != QT_Q8, red);
    float scale = fast_rsqrt(__fadd_rn(__fdiv_rn(ss, (float)n), c.eps));
    for (int i = threadIdx.x; i < n; i += kThreads) out[(size_t)m * n + i] = __fmul_rn(__fmul_rn(tmp[i], w[i]), scale);
    __syncthreads();
  }
}

// RMSNorm output (ops.go:1015-1037) for M sequences; one block per sequence.
__device__ void phase_rmsnorm_out(const Ctx &c, const float *x, int n, int M, const float *w, float *out,
                                  float *smem) {
  float *red = smem, *tmp = smem + 320;
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    for (int i = threadIdx.x; i < n; i += kThreads) tmp[i] = x[(size_t)m * n + i];
    __syncthreads();
    float ss = ss_rmsnorm(tmp, n, red);
    float scale = fast_rsqrt(__fadd_rn(__fdiv_rn(ss, (float)n), c.eps));
    for (int i = threadIdx.x; i < n; i += kThreads) out[(size_t)m * n + i] = __fmul_rn(__fmul_rn(tmp[i], w[i]), scale);
    __syncthreads();
  }
}

// lm_head argmax result -> token ids (and reset of the keys for the next step).
__device__ void phase_argmax_finish(const Ctx &c) {
  const StepParams &sp = *c.sp;
  if (blockIdx.x == 0 && threadIdx.x < sp.M) {
    unsigned long long k = c.argkey[threadIdx.x];
    c.tok_out[threadIdx.x] = sp.need[threadIdx.x] ? argmax_key_row(k) : -1;
    c.argkey[threadIdx.x] = 0ull;
  }
}

}  // namespace ocrvl
