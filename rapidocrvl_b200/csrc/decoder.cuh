// Decode-step device code for the ERNIE text decoder of RapidAI/RapidOCRvl
// (Runtime.forwardEmbeddingForSampling, internal/model/model.go:3475-3643).
//
// Every stage is a __device__ "phase" that walks its work items with a
// grid-stride loop, so the same code runs as a standalone kernel (op tests,
// per-phase launches) or inside the persistent step kernel (engine.cu), where
// phases are separated by grid barriers.  Phases read the model/step context
// through a pointer to a Ctx in global memory and keep their arguments in
// shared memory, so no large per-thread stack frames exist.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "numerics.cuh"

namespace ocrvl {

constexpr int kMaxBatch = 8;      // sequences the register-batched GEMV and the single-step kernel take
constexpr int kMaxSeqs = 64;      // sequences per decode step (the batched step kernel above kMaxBatch)
constexpr int kThreads = 256;     // threads per block, every phase
constexpr int kPageTokens = 16;   // tokens per KV page
constexpr int kAttnChunk = 32;    // tokens per attention work item
constexpr int kHeadDim = 128;     // head size the attention phase supports
constexpr int kMaxGroup = 8;      // q heads per kv head
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

// Per-sequence step record (32 bytes), so a step's parameters are a header
// plus its n records and only those bytes cross to the device.
struct SeqParams {
  int tok;                 // input token id (embedding row)
  int len;                 // cache length before this step's append
  int pos[3];              // M-RoPE (T, H, W) position
  int need;                // sequence needs logits / argmax
  const int *bt;           // block table (page ids)
};
struct StepParams {
  int M;                   // sequences in this step
  int any_logits;          // some sequence needs lm_head this step
  int max_n;               // max over sequences of len+1
  int store_logits;        // write the full logits (the caller reads them), else argmax only
  SeqParams seq[kMaxSeqs];
};
__host__ __device__ __forceinline__ size_t step_params_bytes(int n) { return 16 + (size_t)n * sizeof(SeqParams); }
static_assert(sizeof(SeqParams) == 32, "SeqParams is 32 bytes");

// TMA descriptor (CUtensorMap, 128 bytes) as the kernels receive it.
struct __align__(64) TmapBytes {
  unsigned char b[128];
};

struct Ctx {
  int qtype, H, I, L, QH, KVH, D, V;
  float eps, attn_scale;
  float fzero;                       // 0.0f, read at run time (an FMA addend the compiler cannot fold)
  int dyn_smem;                      // usable dynamic shared memory of the step kernels (bytes, after alignment)
  const float *embed, *final_norm;
  const LayerW *layers;
  DMat lm_head;
  const float *rope_cos, *rope_sin;  // [rope_max][D/2]
  int rope_max;
  const int *sec_axis;               // [D/2] M-RoPE axis of each frequency
  float *kv_pool;                    // pages of [L][KVH][2 (K, V)][16][D] f32
  const TmapBytes *kv_map;           // 2-D map of the pool: rows of D floats, box 64 floats x 16 rows
  long long page_floats;
  // step work buffers
  float *h, *vbuf, *qkv, *head, *g, *logits;
  float *att_s;                      // long-cache attention scores: per sequence [kv head][head][positions]
  unsigned long long *argkey;        // [B]
  int *tok_out;                      // [B] ids, then the error word
  int max_ctx;
  // step parameters: `sp` is read (inside the step kernels it points to a
  // shared-memory copy made at launch), `sp_w` is the global copy that the
  // device-fed loop advances for the next launch
  const StepParams *sp;
  StepParams *sp_w;
  int pro_cols;                      // widest GEMV input: fixes the stage-ring offset (0: per phase)
  unsigned *lm_count;                // lm_head block arrivals
  int *hist, *hist_pos;              // device-side greedy loop: ids [steps][M], write index
  // persistent-kernel barrier: monotonic arrival counter, error word and the
  // polls a block makes before it gives up (the step then fails with a timeout)
  unsigned *bar_count;
  int *err;
  unsigned long long bar_spins;
  // optional step trace: per phase [start, prologue end, phase end (max over
  // blocks), barrier exit] in %globaltimer ns
  unsigned long long *trace;
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Dynamic shared memory of the kernels that run the phases below, from a
// 1024-byte boundary: TMA tensor copies and tcgen05 operand tiles need
// 128-byte aligned destinations, and where the dynamic area starts depends on
// the kernel's static shared memory (launches reserve kSmemAlignSlack bytes
// for the shift).  The phases derive their pointers from this address inside
// the function, so the compiler knows they point to shared memory and emits
// shared-memory loads (a pointer passed in from the caller is generic).
constexpr int kSmemAlignSlack = 1024;
__device__ __forceinline__ float *dyn_smem() {
  extern __shared__ float4 ocrvl_dyn_smem[];
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(ocrvl_dyn_smem);
  return (float *)((uint8_t *)ocrvl_dyn_smem + ((kSmemAlignSlack - (s & (kSmemAlignSlack - 1))) & (kSmemAlignSlack - 1)));
}

// Trace buffer (OCRVL_TRACE): 256 phase rows of 4 words, then kTraceMarks
// per-block time stamps for each of up to 1024 blocks.
constexpr int kTraceRows = 256;
constexpr int kTraceMarks = 24;
constexpr int kTraceWords = 4 * kTraceRows + kTraceMarks * 1024;
// ---------------------------------------------------------------------------
// Small block-level helpers
// ---------------------------------------------------------------------------
// Block reductions with a single __syncthreads: warp partials go to red[0..7],
// then every thread reduces the eight partials itself.  Callers give each
// reduction its own red slots (no barrier protects them from the next write).
__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; w++) r = fmaxf(r, red[w]);
  return r;
}

__device__ __forceinline__ int block_sum_int(int v, int *red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; w++) r += red[w];
  return r;
}

// sumSquaresF32FMA order (internal/tensor/dot_amd64.s:7395-7455) for n a
// multiple of 128: 64 FMA chains (slot = index mod 64), then
// (Z0+Z1)+(Z2+Z3) and the 16-lane tree.  All threads get the result.
__device__ float ss_rmsnorm(const float *x, int n, float *red) {
  if (threadIdx.x < 64) {
    float a = 0.0f;
#pragma unroll 1
    for (int c = threadIdx.x; c < n; c += 64) a = __fmaf_rn(x[c], x[c], a);
    red[threadIdx.x] = a;
  }
  __syncthreads();
  // every thread folds the 64 slots the same way (no second barrier)
  float r[16];
#pragma unroll
  for (int l = 0; l < 16; l++) r[l] = __fadd_rn(__fadd_rn(red[l], red[16 + l]), __fadd_rn(red[32 + l], red[48 + l]));
  return tree16(r);
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
  // every thread adds the worker partials in worker order (no second barrier)
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
        part = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])), __fadd_rn(r[4], r[5])),
                         __fadd_rn(r[6], r[7]));
        int nb = (e - s) / 8 * 8;
        for (int i = s + nb; i < e; i++) part = __fadd_rn(part, __fmul_rn(v[i], v[i]));
      }
    }
    ss = __fadd_rn(ss, part);
  }
  // the tail terms above read v after the barrier: keep v unchanged until
  // every thread has read it (uniform condition, depends on n only)
  if ((vnni && chunk < 16) || (!vnni && chunk % 8 != 0)) __syncthreads();
  return ss;
}

// ---------------------------------------------------------------------------
// GEMV input prologue.  Every block builds the (normalised, quantised) input
// vectors of all M sequences in shared memory itself, from L2-resident fp32
// sources, so no separate norm / quantise launch is needed.
// ---------------------------------------------------------------------------
enum { PRO_PLAIN = 0, PRO_RMSNORM = 1, PRO_ADDNORM = 2 };

struct XIn {
  // VNNI types: xq (uint8, offset 128) per sequence; Q4 stores even columns
  // then odd columns.  Q8: xf fp32 per sequence.  sx / sumq: per-sequence
  // activation scale and sum of xq (shared memory).
  uint8_t *xq;
  float *xf;
  const float *sx;
  const int *sumq;
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

// x = (x * w) * scale over shared x (mulScaleFMA order); w in shared memory
// (staged by the GEMV phase) or, when w_global, read from global memory.
__device__ __forceinline__ void norm_apply(float *x, const float *w, bool w_global, int n, float scale) {
  constexpr int U = 4;
  const int n4 = n >> 2;
  for (int base = threadIdx.x; base < n4; base += kThreads * U) {
    float4 wv[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      int i = base + u * kThreads;
      if (i < n4) wv[u] = w_global ? __ldg((const float4 *)w + i) : ((const float4 *)w)[i];
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

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory layout of the prologue: [red 320 f32 (sx at 304.., sumq at
// 312..)][tmp n f32][x area].  Out of line: every GEMV phase shares one copy.
// The caller's cp.async copies (row scales, row sums, norm weights) are
// complete and visible after the first barrier here.  Barriers: one after the
// gather, one per reduction, one after the normalisation, one at the end.
__device__ __noinline__ void gemv_prologue(int qt, int M, const float *src, int ld, const StepParams *tok, int n,
                                           int mode, const float *w, bool w_global, float eps, float *smem) {
  float *red = smem;
  float *sxs = smem + 304;
  int *sqs = (int *)(smem + 312);
  float *tmp = smem + 320;
  uint8_t *area = (uint8_t *)(tmp + n);
  const bool vnni = qt != QT_Q8;
#pragma unroll 1
  for (int m = 0; m < M; m++) {
    const float *s = src + (size_t)(tok ? tok->seq[m].tok : m) * ld;
    float *dst = vnni ? tmp : (float *)area + (size_t)m * n;
    g2s_f32(dst, s, n);
    cp_async_wait_all();
    __syncthreads();
    if (mode != PRO_PLAIN) {
      float ss = mode == PRO_RMSNORM ? ss_rmsnorm(dst, n, red) : ss_fused(dst, n, vnni, red);
      float scale = fast_rsqrt(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
      norm_apply(dst, w, w_global, n, scale);
      __syncthreads();
    }
    if (vnni) {
      float mx = 0.0f;
#pragma unroll 1
      for (int i = threadIdx.x; i < n; i += kThreads) mx = fmaxf(mx, fabsf(dst[i]));
      mx = block_max(mx, red + 160);
      float sx = 1.0f, inv = 0.0f;
      if (mx != 0.0f) {
        sx = __fdiv_rn(mx, 127.0f);
        inv = __fdiv_rn(1.0f, sx);
      }
      uint8_t *q = area + (size_t)m * n;
      const int half = qt == QT_Q4 ? n / 2 : 0;
      int acc = 0;
#pragma unroll 1
      for (int i = threadIdx.x; i < n; i += kThreads) {
        float f = __fadd_rn(rintf(__fmul_rn(dst[i], inv)), 128.0f);
        int v = mx != 0.0f ? (int)fminf(fmaxf(f, 0.0f), 255.0f) : 128;
        acc += v;
        q[half ? (i & 1) * half + (i >> 1) : i] = (uint8_t)v;  // Q4: even | odd halves
      }
      acc = block_sum_int(acc, (int *)(red + 176));
      if (threadIdx.x == 0) {
        sxs[m] = sx;
        sqs[m] = acc;
      }
    }
    // tmp / red are rewritten by the next sequence
    __syncthreads();
  }
}

__device__ __forceinline__ XIn gemv_inputs(int n, float *smem) {
  XIn x;
  x.xq = (uint8_t *)(smem + 320 + n);
  x.xf = (float *)x.xq;
  x.sx = smem + 304;
  x.sumq = (const int *)(smem + 312);
  return x;
}

__device__ __forceinline__ size_t gemv_smem_bytes(int qt, int M, int n) {
  size_t area = qt == QT_Q8 ? (size_t)M * n * 4 : (size_t)M * n;
  return (320 + (size_t)n) * 4 + area;
}
// ---------------------------------------------------------------------------
// Bulk copies (TMA, cp.async.bulk) and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Asynchronous global -> shared copies of read-only weights (row scales, row
// sums, norm weights); completed by cp_async_wait_all in the GEMV prologue.
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// global -> shared bulk copy; src and dst 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// 2-D TMA tile copy into this CTA only, of a box at (x elements, y rows); x
// times the element size is a multiple of 16 bytes at every call site.
__device__ __forceinline__ void tma_2d(void *dst, const TmapBytes *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Bounded wait for phase `parity` of an mbarrier: at most kMbarSpins polls
// and kMbarWaitNs of elapsed time (a poll may suspend the thread for a while).
// On timeout the error word is set and false returned.  `bail`: the wait also
// ends once another thread has set the error word (for waits on other
// threads' arrivals; a wait on the block's own copies runs until they land,
// so that no copy is in flight when the block leaves).
constexpr long long kMbarSpins = 1ll << 24;
constexpr unsigned long long kMbarWaitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, bool bail = false) {
  uint32_t done = 0;
  long long spins = 0;
  unsigned long long t0 = 0;
  while (true) {
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    if (done) return true;
    ++spins;
    if ((spins & 255) == 1) {
      const unsigned long long now = gtimer();
      if (spins == 1) t0 = now;
      else if (now - t0 > kMbarWaitNs || (bail && err && *(volatile int *)err)) spins = kMbarSpins + 1;
    }
    if (spins > kMbarSpins) {
      if (err) atomicExch(err, 1);
      return false;
    }
  }
}

// Shared-memory loads as ordinary dereferences: the compiler orders them
// against barriers and the mbarrier waits (asm with a memory clobber) but is
// free to issue them early, ahead of the arithmetic that consumes them.
__device__ __forceinline__ uint4 lds16(const void *p) { return *(const uint4 *)p; }
__device__ __forceinline__ uint32_t lds4(const void *p) { return *(const uint32_t *)p; }

// ---------------------------------------------------------------------------
// Row dot products over a batch of RB rows whose packed weights are staged in
// shared memory (rp[r] = row start).  out[r][m] = finished row value (per-type
// epilogue arithmetic applied), valid on the lane with (lane % lpr) == 0.
// ---------------------------------------------------------------------------

// Q4 (int8-activation mode): per 16-byte chunk, low nibbles hold even columns
// and high nibbles odd columns; dp4a of the unsigned nibbles against the even /
// odd halves of xq gives sum((q+8)*xq), corrected by 8*sum(xq).
template <int M_, int RB>
__device__ __forceinline__ void dot_q4(const DMat &A, const uint8_t *const *rp, const int *rows, int M, const XIn &x,
                                       const float *scl, const int32_t *rsm, int li, int lpr, float (*out)[M_]) {
  const int CH = A.pitch >> 4, n = A.cols;
  uint32_t acc[RB][M_];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++) acc[r][m] = 0;
#pragma unroll 1
  for (int k = li; k < CH; k += lpr) {
    uint4 wv[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) wv[r] = lds16(rp[r] + 16 * k);
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      const uint4 xe = lds16(x.xq + (size_t)m * n + 16 * k);
      const uint4 xo = lds16(x.xq + (size_t)m * n + n / 2 + 16 * k);
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
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      uint32_t a = acc[r][m];
      for (int o = lpr >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      acc[r][m] = a;
    }
  }
  if ((li) != 0) return;
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const int32_t rs = rsm[r];
    const float sw = scl[r];
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      out[r][m] = vnni_finalize((int32_t)acc[r][m] - 8 * x.sumq[m], rs, x.sx[m], sw);
    }
  }
}

// Q6: 48-byte chunks = 64 columns = 16 little-endian 24-bit groups of four
// 6-bit fields; fields widened to bytes for dp4a, corrected by 32*sum(xq).
__device__ __forceinline__ uint32_t q6_spread(uint32_t g) {
  return (g & 0x3Fu) | ((g << 2) & 0x3F00u) | ((g << 4) & 0x3F0000u) | ((g << 6) & 0x3F000000u);
}
template <int M_, int RB>
__device__ __forceinline__ void dot_q6(const DMat &A, const uint8_t *const *rp, const int *rows, int M, const XIn &x,
                                       const float *scl, const int32_t *rsm, int li, int lpr, float (*out)[M_]) {
  const int CH = A.pitch / 48, n = A.cols;
  uint32_t acc[RB][M_];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++) acc[r][m] = 0;
#pragma unroll 1
  for (int k = li; k < CH; k += lpr) {
#pragma unroll
    for (int r = 0; r < RB; r++) {
      const uint4 wa = lds16(rp[r] + 48 * k), wb = lds16(rp[r] + 48 * k + 16), wc = lds16(rp[r] + 48 * k + 32);
      const uint32_t w[12] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w, wc.x, wc.y, wc.z, wc.w};
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const uint32_t w0 = w[3 * t], w1 = w[3 * t + 1], w2 = w[3 * t + 2];
        const uint32_t f0 = q6_spread(w0 & 0xFFFFFFu), f1 = q6_spread(__funnelshift_r(w0, w1, 24) & 0xFFFFFFu);
        const uint32_t f2 = q6_spread(__funnelshift_r(w1, w2, 16) & 0xFFFFFFu), f3 = q6_spread(w2 >> 8);
#pragma unroll
        for (int m = 0; m < M_; m++) {
          if (m >= M) break;
          const uint4 xx = lds16(x.xq + (size_t)m * n + 64 * k + 16 * t);
          acc[r][m] = __dp4a(f0, xx.x, acc[r][m]);
          acc[r][m] = __dp4a(f1, xx.y, acc[r][m]);
          acc[r][m] = __dp4a(f2, xx.z, acc[r][m]);
          acc[r][m] = __dp4a(f3, xx.w, acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; r++) {
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      uint32_t a = acc[r][m];
      for (int o = lpr >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      acc[r][m] = a;
    }
  }
  if (li != 0) return;
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const int32_t rs = rsm[r];
    const float sw = scl[r];
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      out[r][m] = vnni_finalize((int32_t)acc[r][m] - 32 * x.sumq[m], rs, x.sx[m], sw);
    }
  }
}

// Q8 (fp32-activation mode) in dotQ8FMA order (internal/tensor/
// dot_fma_amd64.s:666-799): lane t owns slots 4t..4t+3 of every 128-column
// block (accumulator t/4, ZMM lanes 4(t%4)..+3); the accumulator pairs are
// reduced with xor-4/8/16 shuffles and the 16-lane tree with xor-2/1.
template <int M_, int RB>
__device__ __forceinline__ void dot_q8(const DMat &A, const uint8_t *const *rp, const int *rows, int M, const XIn &x,
                                       const float *scl, int lane, float (*out)[M_]) {
  const int n = A.cols, NB = n >> 7;
  float acc[RB][M_][4];
#pragma unroll
  for (int r = 0; r < RB; r++)
#pragma unroll
    for (int m = 0; m < M_; m++)
#pragma unroll
      for (int i = 0; i < 4; i++) acc[r][m][i] = 0.0f;
#pragma unroll 1
  for (int j = 0; j < NB; j++) {
    uint32_t wv[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) wv[r] = lds4(rp[r] + 128 * j + 4 * lane);
#pragma unroll
    for (int m = 0; m < M_; m++) {
      if (m >= M) break;
      const uint4 xb = lds16(x.xf + (size_t)m * n + 128 * j + 4 * lane);
      const float x0 = __uint_as_float(xb.x), x1 = __uint_as_float(xb.y);
      const float x2 = __uint_as_float(xb.z), x3 = __uint_as_float(xb.w);
#pragma unroll
      for (int r = 0; r < RB; r++) {
        const uint32_t w = wv[r];
        acc[r][m][0] = __fmaf_rn((float)(int8_t)(w & 0xFF), x0, acc[r][m][0]);
        acc[r][m][1] = __fmaf_rn((float)(int8_t)((w >> 8) & 0xFF), x1, acc[r][m][1]);
        acc[r][m][2] = __fmaf_rn((float)(int8_t)((w >> 16) & 0xFF), x2, acc[r][m][2]);
        acc[r][m][3] = __fmaf_rn((float)(int8_t)(w >> 24), x3, acc[r][m][3]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; r++) {
    const float sw = scl[r];
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

// scl[r] / rsm[r]: scale and row sum of row r of the batch (loaded by the
// caller before the dots so their latency overlaps the dot products).
template <int QT, int M_, int RB>
__device__ __forceinline__ void rows_dot(const DMat &A, const uint8_t *const *rp, const int *rows, int M,
                                         const XIn &x, const float *scl, const int32_t *rsm, int lane, int lpr,
                                         float (*out)[M_]) {
  if (QT == QT_Q4)
    dot_q4<M_, RB>(A, rp, rows, M, x, scl, rsm, lane % lpr, lpr, out);
  else if (QT == QT_Q6)
    dot_q6<M_, RB>(A, rp, rows, M, x, scl, rsm, lane % lpr, lpr, out);
  else
    dot_q8<M_, RB>(A, rp, rows, M, x, scl, lane, out);
}

// ---------------------------------------------------------------------------
// GEMV phases
// ---------------------------------------------------------------------------
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };
enum { RESID_ALWAYS = 0, RESID_ATTN = 1, RESID_NEVER = 2, RESID_MASK = 3 };

// Arguments of one GEMV phase; built in shared memory by the caller.
struct GemvArgs {
  DMat A, B;                // B: up matrix for EPI_SWIGLU
  int row_begin, row_end;   // rows of A to compute
  const float *src;         // input vectors [M][ld] (or rows tok[m] when src_tok)
  int ld, src_tok;
  float *copy_src;          // when set, block 0 stores the prologue's input rows here ([M][ld])
  int mode;                 // PRO_*
  const float *norm_w;
  int epi;
  float *out;               // EPI_STORE / EPI_SWIGLU: [M][ldo]
  int ldo;
  float *resid;             // EPI_RESID: residual [M][ldo] (updated when in place)
  float *vout;              // EPI_RESID: v = resid + out, [M][ldo]
  int resid_mode;           // EPI_RESID: RESID_*
  int in_place_mask;        // RESID_MASK: bit m set -> update resid
  unsigned long long *argkey;  // EPI_ARGMAX: [M]
  float *logits;            // EPI_ARGMAX: optional full scores [M][ldo]
  int argmax_finish;        // EPI_ARGMAX: last block turns keys into ids
  int feed;                 // EPI_ARGMAX finish: advance the step parameters
  unsigned long long *tslot;   // optional trace slot of this phase
};

// Contiguous slab of rows [lo, hi) of a GEMV owned by block `b` of `nb`.
__device__ __forceinline__ void gemv_slab(int row_begin, int row_end, int b, int nb, int &lo, int &hi) {
  const unsigned n = (unsigned)(row_end - row_begin);
  if (n < (1u << 23)) {  // n * nb fits 32 bits for any grid of <= 512 blocks
    lo = row_begin + (int)(n * (unsigned)b / (unsigned)nb);
    hi = row_begin + (int)(n * (unsigned)(b + 1) / (unsigned)nb);
  } else {
    lo = row_begin + (int)((unsigned long long)n * b / nb);
    hi = row_begin + (int)((unsigned long long)n * (b + 1) / nb);
  }
}

// Weight staging: each block streams its slab of packed rows through a ring
// of kStages shared-memory stages with TMA bulk copies; the copies of the
// first stages are issued before the input prologue so weight transfer
// overlaps the normalisation / quantisation of the input.
constexpr int kStageBytes = 32768;
constexpr int kStagesM1 = 5;   // stages for the single-sequence form
constexpr int kStagesMB = 2;   // stages for the batched form
// Row scales and row sums of a block's slab (A and B matrices) and the norm
// weights are staged in shared memory with cp.async at the start of the
// phase, when the slab has at most kSlabRowsMax rows and the norm vector at
// most kNormStageMax entries (otherwise they are read from global memory).
constexpr int kSlabRowsMax = 1024;  // A matrix rows
constexpr int kSlabRowsB = 128;     // B matrix (SwiGLU up) rows
constexpr int kNormStageMax = 2048;
// aux layout (floats): A scales | A row sums | B scales | B row sums | norm weights
constexpr int kAuxRsA = kSlabRowsMax, kAuxScB = 2 * kSlabRowsMax, kAuxRsB = kAuxScB + kSlabRowsB;
constexpr int kAuxNw = kAuxRsB + kSlabRowsB;
constexpr size_t kGemvAuxBytes = (size_t)(kAuxNw + kNormStageMax) * 4;

__host__ __device__ __forceinline__ size_t gemv_prologue_bytes(int qt, int nvec, int n) {
  size_t area = qt == QT_Q8 ? (size_t)nvec * n * 4 : (size_t)nvec * n;
  return ((320 + (size_t)n) * 4 + area + 127) / 128 * 128;
}
__host__ __device__ __forceinline__ size_t gemv_smem_total(int qt, int nvec, int n, int stages) {
  return gemv_prologue_bytes(qt, nvec, n) + (size_t)stages * kStageBytes + kGemvAuxBytes;
}

// ---------------------------------------------------------------------------
// Stage ring shared by the GEMV phases of one launch.  One mbarrier per ring
// slot, initialised once per launch; s_ring_par bit i is the parity of slot
// i's next completion and s_ring_busy bit i says a copy into slot i is in
// flight.  A phase's first stages and its cp.async staging (row scales / row
// sums, norm weights) can be issued ahead of the phase ("setup"), in the step
// kernel while the block waits at the grid barrier before it; s_ring_setup
// tells the phase that this was done.
// ---------------------------------------------------------------------------
constexpr int kMaxStages = kStagesM1 > kStagesMB ? kStagesM1 : kStagesMB;
__shared__ __align__(8) uint64_t s_ring_bar[kMaxStages];
__shared__ uint32_t s_ring_par, s_ring_busy;
__shared__ int s_ring_setup;

__device__ __forceinline__ void ring_init() {
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxStages; i++) mbar_init(&s_ring_bar[i], 1);
    mbar_fence_init();
    s_ring_par = 0;
    s_ring_busy = 0;
    s_ring_setup = 0;
  }
  __syncthreads();
}

// Where a GEMV phase keeps its stages and staged values, and how its slab of
// rows splits into stages.  The ring follows the widest prologue the kernel
// can run (Ctx::pro_cols), so its place does not move between phases.
struct GemvGeo {
  int lo, hi, P, srows, nst, kSt;
  int lpr;  // lanes per row of the x-stationary form (Q4/Q6)
  bool two, staged, nw_staged;
  uint8_t *stage;
  float *aux;
};
__shared__ GemvGeo s_geo;  // geometry of the phase that was set up ahead

__device__ __forceinline__ GemvGeo gemv_geo(int qt, const Ctx &c, const GemvArgs &a, int M, float *smem) {
  GemvGeo g;
  gemv_slab(a.row_begin, a.row_end, blockIdx.x, gridDim.x, g.lo, g.hi);
  g.P = a.A.pitch;
  g.two = a.epi == EPI_SWIGLU;
  g.kSt = M <= 1 ? kStagesM1 : kStagesMB;
  g.stage = (uint8_t *)smem + gemv_prologue_bytes(qt, M <= 1 ? 1 : kMaxBatch, c.pro_cols ? c.pro_cols : a.A.cols);
  g.srows = kStageBytes / (g.P * (g.two ? 2 : 1));
  g.nst = (g.hi - g.lo + g.srows - 1) / g.srows;
  g.aux = (float *)(g.stage + (size_t)g.kSt * kStageBytes);
  g.staged = g.hi - g.lo <= kSlabRowsMax && (!g.two || g.hi - g.lo <= kSlabRowsB);
  g.nw_staged = a.mode != PRO_PLAIN && a.A.cols <= kNormStageMax;
  g.lpr = 32;
  if (qt != QT_Q8) {
    const int cb = qt == QT_Q4 ? 16 : 48, xmax = qt == QT_Q4 ? 4 : 2;
    const int ch = g.P / cb;
    int l = 1;
    while (l < 32 && (ch + l - 1) / l > xmax) l <<= 1;
    g.lpr = l;
  }
  return g;
}

// Thread 0: copy of stage `st` of the slab into its ring slot.
__device__ __forceinline__ void gemv_issue(const GemvArgs &a, const GemvGeo &g, int st) {
  const int slot = st % g.kSt;
  const int r0 = g.lo + st * g.srows, nr = min(g.srows, g.hi - r0);
  uint8_t *buf = g.stage + (size_t)slot * kStageBytes;
  const uint32_t bytes = (uint32_t)nr * g.P;
  mbar_expect_tx(&s_ring_bar[slot], g.two ? 2 * bytes : bytes);
  bulk_g2s(buf, a.A.w + (size_t)r0 * g.P, bytes, &s_ring_bar[slot]);
  if (g.two) bulk_g2s(buf + (size_t)g.srows * g.P, a.B.w + (size_t)r0 * g.P, bytes, &s_ring_bar[slot]);
  s_ring_busy |= 1u << slot;
}

// Bounded wait for stage `st`; every thread calls it.
__device__ __forceinline__ bool gemv_wait(const Ctx &c, const GemvGeo &g, int st) {
  const int slot = st % g.kSt;
  return mbar_wait(&s_ring_bar[slot], (s_ring_par >> slot) & 1u, c.err);
}

// After a stage's compute and a block barrier: thread 0 retires the slot and
// refills it with stage st + kSt.
__device__ __forceinline__ void gemv_retire(const GemvArgs &a, const GemvGeo &g, int st) {
  if (threadIdx.x == 0) {
    const int slot = st % g.kSt;
    s_ring_par ^= 1u << slot;
    s_ring_busy &= ~(1u << slot);
    if (st + g.kSt < g.nst) gemv_issue(a, g, st + g.kSt);
  }
}

// Issues the phase's first stages (thread `lead`) and the cp.async staging of
// its row scales / row sums and norm weights (threads lead .. lead+nthr-1).
__device__ void gemv_setup(int qt, const Ctx &c, const GemvArgs &a, int M, float *smem, int lead = 0,
                           int nthr = kThreads) {
  const GemvGeo g = gemv_geo(qt, c, a, M, smem);
  const int tid = (int)threadIdx.x - lead;
  if (tid == 0) {
    s_geo = g;
    for (int st = 0; st < g.nst && st < g.kSt; st++) gemv_issue(a, g, st);
  }
  const bool vnni = qt != QT_Q8;
  if (g.nw_staged) {
    float *nw_s = g.aux + kAuxNw;
    for (int i = tid; i < a.A.cols / 4; i += nthr) cp_async16(nw_s + 4 * i, a.norm_w + 4 * i);
  }
  if (g.staged) {
    const int nrows = g.hi - g.lo;
    for (int i = tid; i < nrows; i += nthr) {
      cp_async4(g.aux + i, a.A.scale + g.lo + i);
      if (vnni) cp_async4(g.aux + kAuxRsA + i, a.A.rowsum + g.lo + i);
      if (g.two) {
        cp_async4(g.aux + kAuxScB + i, a.B.scale + g.lo + i);
        if (vnni) cp_async4(g.aux + kAuxRsB + i, a.B.rowsum + g.lo + i);
      }
    }
  }
}

// Waits for copies the block still has in flight (before leaving the kernel
// early).  Every thread calls it.
__device__ void gemv_drain(const Ctx &c) {
  cp_async_wait_all();
  if (threadIdx.x == 0) {
    for (int slot = 0; slot < kMaxStages; slot++) {
      if ((s_ring_busy >> slot) & 1u) {
        mbar_wait(&s_ring_bar[slot], (s_ring_par >> slot) & 1u, c.err);
        s_ring_par ^= 1u << slot;
      }
    }
    s_ring_busy = 0;
    s_ring_setup = 0;
  }
  __syncthreads();
}

// Last block of the lm_head phase: keys -> ids (ties -> lowest id), key and
// counter reset, and (device-side greedy loop) the next step's parameters:
// tok = argmax, len + 1, position (len, len, len).
__device__ void argmax_finish(const Ctx &c, int M, int feed) {
  const StepParams &sp = *c.sp;
  StepParams &spw = *c.sp_w;
  if (threadIdx.x < M) {
    const int m = threadIdx.x;
    unsigned long long k = __ldcg(c.argkey + m);
    int id = sp.seq[m].need ? argmax_key_row(k) : -1;
    c.tok_out[m] = id;
    c.argkey[m] = 0ull;
    if (feed) {
      // through L2: another block may have advanced it in an earlier step
      // of the same launch (device-fed loop)
      int step = __ldcg(c.hist_pos);
      c.hist[(size_t)step * M + m] = id;
      int len = sp.seq[m].len + 1;
      spw.seq[m].tok = id;
      spw.seq[m].len = len;
      spw.seq[m].pos[0] = spw.seq[m].pos[1] = spw.seq[m].pos[2] = len;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (feed) {
      atomicAdd(c.hist_pos, 1);  // at L2, like the read above
      spw.max_n = sp.max_n + 1;
    }
    *c.lm_count = 0u;
  }
}

template <int QT, int M_, int RB>
__device__ __noinline__ void phase_gemv_t(const Ctx *cp, const GemvArgs *ap, int M, float *smem_arg) {
  float *const smem = dyn_smem();  // == smem_arg (the aligned dynamic base)
  (void)smem_arg;
  const Ctx &c = *cp;
  const GemvArgs &a = *ap;
  const int qt = QT;
  const bool pre = s_ring_setup;
  if (!pre) gemv_setup(qt, c, a, M_ == 1 ? 1 : kMaxBatch, smem);
  const GemvGeo g = pre ? s_geo : gemv_geo(qt, c, a, M_ == 1 ? 1 : kMaxBatch, smem);
  const int P = g.P, lo = g.lo, hi = g.hi, srows = g.srows, nst = g.nst;
  const bool two = g.two;
  float *aux = g.aux;
  const bool staged = g.staged;
  const bool vnni = qt != QT_Q8;
  const float *scl_a = staged ? aux : a.A.scale + lo;
  const int32_t *rsm_a = staged ? (const int32_t *)(aux + kAuxRsA) : a.A.rowsum + lo;
  const float *scl_b = staged ? aux + kAuxScB : a.B.scale + lo;
  const int32_t *rsm_b = staged ? (const int32_t *)(aux + kAuxRsB) : a.B.rowsum + lo;
  const bool nw_staged = g.nw_staged;
  float *nw_s = aux + kAuxNw;
  gemv_prologue(qt, M, a.src, a.ld, a.src_tok ? c.sp : nullptr, a.A.cols, a.mode, nw_staged ? nw_s : a.norm_w,
                !nw_staged, c.eps, smem);
  const XIn x = gemv_inputs(a.A.cols, smem);
  if (a.copy_src && blockIdx.x == 0) {
    // layer 0: the embedding rows the prologue gathered become the residual
    for (int m = 0; m < M; m++) {
      const float4 *s4 = (const float4 *)(a.src + (size_t)c.sp->seq[m].tok * a.ld);
      float4 *d4 = (float4 *)(a.copy_src + (size_t)m * a.ld);
      for (int i = threadIdx.x; i < a.ld / 4; i += kThreads) d4[i] = __ldg(s4 + i);
    }
  }
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
        int len = c.sp->seq[m].len;
        ip = qt == QT_Q8 || (len >= 1 && len + 1 <= 6);
      }
      in_place |= (ip ? 1 : 0) << m;
    }
  }
  unsigned long long best[M_];
#pragma unroll
  for (int m = 0; m < M_; m++) best[m] = 0ull;
  const int per_group = rpw * RB;
  bool ok = true;
#pragma unroll 1
  for (int st = 0; st < nst; st++) {
    const int r0 = lo + st * srows, nr = min(srows, hi - r0);
    const uint8_t *buf = g.stage + (size_t)(st % g.kSt) * kStageBytes;
    if (!gemv_wait(c, g, st)) ok = false;
    const int ngroups = (nr + per_group - 1) / per_group;
#pragma unroll 1
    for (int gi = warp; ok && gi < ngroups; gi += kThreads / 32) {
      int rows[RB];
      const uint8_t *rpa[RB], *rpb[RB];
      bool valid[RB];
#pragma unroll
      for (int r = 0; r < RB; r++) {
        int lr = gi * per_group + r * rpw + sub;
        valid[r] = lr < nr;
        lr = valid[r] ? lr : nr - 1;
        rows[r] = r0 + lr;
        rpa[r] = buf + (size_t)lr * P;
        rpb[r] = buf + (size_t)(srows + lr) * P;
      }
      float sa[RB], sb[RB];
      int32_t ra[RB], rb[RB];
#pragma unroll
      for (int r = 0; r < RB; r++) {
        const int i = rows[r] - lo;
        sa[r] = scl_a[i];
        ra[r] = vnni ? rsm_a[i] : 0;
        sb[r] = two ? scl_b[i] : 0.0f;
        rb[r] = two && vnni ? rsm_b[i] : 0;
      }
      float v[RB][M_], u[RB][M_];
      rows_dot<QT, M_, RB>(a.A, rpa, rows, M, x, sa, ra, lane, lpr, v);
      if (two) rows_dot<QT, M_, RB>(a.B, rpb, rows, M, x, sb, rb, lane, lpr, u);
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
    __syncthreads();  // stage buffer free
    gemv_retire(a, g, st);
  }
  if (threadIdx.x == 0) s_ring_setup = 0;
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
    if (a.argmax_finish) {
      __shared__ int is_last;
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicAdd(c.lm_count, 1u) == gridDim.x - 1;
        if (is_last) __threadfence();
      }
      __syncthreads();
      if (is_last) argmax_finish(c, M, a.feed);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Single-sequence GEMV for the int8-activation types (Q4, Q6): x-stationary.
// A row is split over lpr lanes, each lane owning the same chunk positions
// k = li + lpr*j (j < XMAX) of every row it visits, so the lane keeps those
// chunks of the quantised input in registers for the whole phase and reads
// only weights from the shared-memory stages.  Each thread works on RB rows
// at once with two dp4a chains per row; the int32 sums are exact, so the split
// does not change results.
// ---------------------------------------------------------------------------
// Input prologue of the single-sequence int8-activation GEMV (xs path).
// Every thread loads float4 groups t, t + 256, ... of the input from L2 into
// registers (the norm modes also into shared memory, where the reduction
// chains read them), the chains are reduced in the reference's order and
// combined after a barrier, and every thread quantises the elements it holds:
//   PRO_RMSNORM (sumSquaresF32FMA): thread s < 64 runs slot s's FMA chain over
//     elements s, s+64, ... in order; slots folded as (s[l]+s[l+16]) +
//     (s[l+32]+s[l+48]), then tree16;
//   PRO_ADDNORM (the fused kernels' 8 workers of n/8 rows, VNNI finalize):
//     thread 16 w + l runs worker w's lane l (rows w n/8 + l + 16 k,
//     unfused square-adds), tree16 over the half-warp, workers added in order;
//   PRO_PLAIN: only the largest |x|.
// The largest |normalised value| is fl(max|fl(x*w)| * scale), rounding being
// monotone and sign-symmetric.  Barriers: 3 (norm modes) or 2 (plain).  Writes
// the uint8 activations (Q4: even columns then odd) to the x area and returns
// the activation scale sx (the same value in every thread).
constexpr int kXsMaxPer = 16;  // elements a thread holds (n <= 4096)
__device__ __noinline__ float xs_prologue(int qt, const float *src, int n, int mode, const float *w, bool w_global,
                                          float eps, float *smem, unsigned long long *mk = nullptr) {
  float *red = smem;  // [16..79] slot / worker sums, [96..103] warp maxima
  float *tmp = smem + 320;
  uint8_t *q = (uint8_t *)(tmp + n);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, n4 = n / 4;
  float4 xv[kXsMaxPer / 4];
#pragma unroll
  for (int k = 0; k < kXsMaxPer / 4; k++) {
    const int g = t + kThreads * k;
    xv[k] = g < n4 ? __ldcg((const float4 *)src + g) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float M = 0.0f;
#pragma unroll
  for (int k = 0; k < kXsMaxPer / 4; k++) {
    const int g = t + kThreads * k;
    if (g < n4) {
      const float4 v = xv[k];
      if (mode == PRO_PLAIN) {
        M = fmaxf(M, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      } else {
        ((float4 *)tmp)[g] = v;
        const float4 ww = w_global ? __ldg((const float4 *)w + g) : ((const float4 *)w)[g];
        M = fmaxf(M, fmaxf(fmaxf(fabsf(__fmul_rn(v.x, ww.x)), fabsf(__fmul_rn(v.y, ww.y))),
                           fmaxf(fabsf(__fmul_rn(v.z, ww.z)), fabsf(__fmul_rn(v.w, ww.w)))));
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) red[96 + warp] = M;
  if (mode != PRO_PLAIN) {
    __syncthreads();
    if (mode == PRO_RMSNORM) {
      if (t < 64) {
        float a = 0.0f;
#pragma unroll 4
        for (int c = t; c < n; c += 64) a = __fmaf_rn(tmp[c], tmp[c], a);
        red[16 + t] = a;
      }
    } else {
      const int chunk = n / kFusedWorkers;
      float a = 0.0f;
      if (t < 16 * kFusedWorkers) {
        const float *r = tmp + (t >> 4) * chunk;
#pragma unroll 4
        for (int k = t & 15; k < chunk; k += 16) a = __fadd_rn(a, __fmul_rn(r[k], r[k]));
      }
      // tree16 of each half-warp (one worker)
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 2));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 1));
      if ((t & 15) == 0 && t < 16 * kFusedWorkers) red[16 + (t >> 4)] = a;
    }
  }
  __syncthreads();
  if (mk) mk[17] = clock64();
  M = red[96];
#pragma unroll
  for (int i = 1; i < kThreads / 32; i++) M = fmaxf(M, red[96 + i]);
  float ss = 0.0f;
  if (mode == PRO_RMSNORM) {
    float r[16];
#pragma unroll
    for (int l = 0; l < 16; l++) r[l] = __fadd_rn(__fadd_rn(red[16 + l], red[32 + l]), __fadd_rn(red[48 + l], red[64 + l]));
    ss = tree16(r);
  } else if (mode == PRO_ADDNORM) {
#pragma unroll
    for (int wk = 0; wk < kFusedWorkers; wk++) ss = __fadd_rn(ss, red[16 + wk]);
  }
  float scale = 1.0f, mx = M;
  if (mode != PRO_PLAIN) {
    // ss / n: a power-of-two n divides exactly as a multiply by 1/n
    const float mean = (n & (n - 1)) == 0 ? __fmul_rn(ss, __uint_as_float((uint32_t)(127 - (31 - __clz(n))) << 23))
                                          : __fdiv_rn(ss, (float)n);
    scale = fast_rsqrt(__fadd_rn(mean, eps));
    mx = __fmul_rn(M, scale);
  }
  float sx = 1.0f, inv = 0.0f;
  if (mx != 0.0f) {
    sx = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(1.0f, sx);
  }
  if (mk) mk[18] = clock64();
  const int half = qt == QT_Q4 ? n / 2 : 0;
#pragma unroll
  for (int k = 0; k < kXsMaxPer / 4; k++) {
    const int g = t + kThreads * k;
    if (g < n4) {
      float v4[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      float4 ww = make_float4(1.f, 1.f, 1.f, 1.f);
      if (mode != PRO_PLAIN) ww = w_global ? __ldg((const float4 *)w + g) : ((const float4 *)w)[g];
      const float w4[4] = {ww.x, ww.y, ww.z, ww.w};
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float v = mode != PRO_PLAIN ? __fmul_rn(__fmul_rn(v4[e], w4[e]), scale) : v4[e];
        const float f = __fadd_rn(rintf(__fmul_rn(v, inv)), 128.0f);
        const int b = mx != 0.0f ? (int)fminf(fmaxf(f, 0.0f), 255.0f) : 128;
        packed |= (uint32_t)b << (8 * e);
      }
      const int i = 4 * g;
      if (half) {
        // Q4: even columns to the first half, odd ones to the second
        ((uint16_t *)q)[i >> 2] = (uint16_t)((packed & 0xFFu) | ((packed >> 8) & 0xFF00u));
        ((uint16_t *)(q + half))[i >> 2] = (uint16_t)(((packed >> 8) & 0xFFu) | ((packed >> 16) & 0xFF00u));
      } else {
        *(uint32_t *)(q + i) = packed;
      }
    }
  }
  __syncthreads();
  if (mk) mk[19] = clock64();
  return sx;
}

// Input widths xs_prologue takes (kXsMaxPer elements a thread).
__host__ __device__ __forceinline__ bool xs_prologue_fits(int mode, int n) {
  return mode == PRO_RMSNORM ? n <= 64 * kXsMaxPer : mode == PRO_ADDNORM ? n <= 16 * kFusedWorkers * kXsMaxPer
                                                                         : n <= 4 * kThreads * (kXsMaxPer / 4);
}

template <int QT>
struct XsTraits;
template <>
struct XsTraits<QT_Q4> {
  static constexpr int CB = 16;    // packed bytes per chunk (32 columns)
  static constexpr int XMAX = 4;   // chunks per lane kept in registers
  static constexpr int XW = 2;     // uint4 of activations per chunk (even, odd halves)
  static constexpr int OFF = 8;    // stored nibble = q + 8
};
template <>
struct XsTraits<QT_Q6> {
  static constexpr int CB = 48;    // 64 columns
  static constexpr int XMAX = 2;
  static constexpr int XW = 4;
  static constexpr int OFF = 32;   // stored field = q + 32
};

__host__ __device__ __forceinline__ int xs_lanes_per_row(int chunks, int xmax) {
  int l = 1;
  while (l < 32 && (chunks + l - 1) / l > xmax) l <<= 1;
  return l;
}

// True when the x-stationary path handles a matrix of this pitch.
template <int QT>
__device__ __forceinline__ bool xs_fits(int pitch) {
  const int ch = pitch / XsTraits<QT>::CB;
  return pitch % XsTraits<QT>::CB == 0 && (ch + 31) / 32 <= XsTraits<QT>::XMAX;
}

// Partial dot of one row: the lane's chunks of the row at `w` against its
// register-held activations.
template <int QT>
__device__ __forceinline__ uint32_t xs_row_dot(const uint8_t *w, const uint4 (*xr)[XsTraits<QT>::XW], int li,
                                               int lpr, int CH) {
  using T = XsTraits<QT>;
  uint32_t a0 = 0, a1 = 0;
#pragma unroll
  for (int j = 0; j < T::XMAX; j++) {
    const int k = li + lpr * j;
    if (k >= CH) break;
    if (QT == QT_Q4) {
      const uint4 wv = lds16(w + 16 * k);
      const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t e4[4] = {xr[j][0].x, xr[j][0].y, xr[j][0].z, xr[j][0].w};
      const uint32_t o4[4] = {xr[j][1].x, xr[j][1].y, xr[j][1].z, xr[j][1].w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        a0 = __dp4a(wd[q] & 0x0F0F0F0Fu, e4[q], a0);
        a1 = __dp4a((wd[q] >> 4) & 0x0F0F0F0Fu, o4[q], a1);
      }
    } else {
      const uint4 wa = lds16(w + 48 * k), wb = lds16(w + 48 * k + 16), wc = lds16(w + 48 * k + 32);
      const uint32_t wd[12] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w, wc.x, wc.y, wc.z, wc.w};
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const uint32_t w0 = wd[3 * t], w1 = wd[3 * t + 1], w2 = wd[3 * t + 2];
        const uint32_t f0 = q6_spread(w0 & 0xFFFFFFu), f1 = q6_spread(__funnelshift_r(w0, w1, 24) & 0xFFFFFFu);
        const uint32_t f2 = q6_spread(__funnelshift_r(w1, w2, 16) & 0xFFFFFFu), f3 = q6_spread(w2 >> 8);
        const uint4 xx = xr[j][t];
        a0 = __dp4a(f0, xx.x, a0);
        a1 = __dp4a(f1, xx.y, a1);
        a0 = __dp4a(f2, xx.z, a0);
        a1 = __dp4a(f3, xx.w, a1);
      }
    }
  }
  return a0 + a1;
}

template <int QT, int RB, int EPI>
__device__ __noinline__ void phase_gemv_xs(const Ctx *cp, const GemvArgs *ap, float *smem_arg) {
  float *const smem = dyn_smem();  // == smem_arg (the aligned dynamic base)
  (void)smem_arg;
  using T = XsTraits<QT>;
  const Ctx &c = *cp;
  const GemvArgs &a = *ap;
  const bool pre = s_ring_setup;
  if (!pre) gemv_setup(QT, c, a, 1, smem);
  const GemvGeo g = pre ? s_geo : gemv_geo(QT, c, a, 1, smem);
  const int P = g.P, n = a.A.cols, CH = QT == QT_Q4 ? P >> 4 : P / 48;
  const int lo = g.lo, hi = g.hi, srows = g.srows, nst = g.nst;
  constexpr bool two = EPI == EPI_SWIGLU;
  float *aux = g.aux;
  const bool staged = g.staged;
  const float *scl_a = staged ? aux : a.A.scale + lo;
  const int32_t *rsm_a = staged ? (const int32_t *)(aux + kAuxRsA) : a.A.rowsum + lo;
  const float *scl_b = staged ? aux + kAuxScB : a.B.scale + lo;
  const int32_t *rsm_b = staged ? (const int32_t *)(aux + kAuxRsB) : a.B.rowsum + lo;
  const bool nw_staged = g.nw_staged;
  float *nw_s = aux + kAuxNw;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lpr = g.lpr;
  const int rpw = 32 / lpr, li = lane & (lpr - 1), sub = lane / lpr;
  const int pass = (kThreads / 32) * rpw;  // rows one pass of the block covers per RB slot
  // trace marks 16-23 of the block (QKV phases; the last layer's remain), SM
  // clock cycles: entry, reductions posted, scale formed, input quantised,
  // activations in registers, first stage landed, dots done, exit
  unsigned long long *mk =
      c.trace && EPI == EPI_STORE && threadIdx.x == 0 ? c.trace + 4 * kTraceRows + kTraceMarks * blockIdx.x : nullptr;
  if (mk) mk[16] = clock64();
  // residual values of this lane's rows of a one-stage slab, fetched now so
  // their latency hides behind the prologue
  float rpre[RB];
  const bool rpre_ok = EPI == EPI_RESID && nst == 1 && li == 0;
  if (rpre_ok) {
#pragma unroll
    for (int r = 0; r < RB; r++) {
      const int l = warp * rpw + sub + r * pass;
      rpre[r] = l < hi - lo ? __ldcg(a.resid + lo + l) : 0.0f;
    }
  }
  const float *src = a.src + (a.src_tok ? (size_t)c.sp->seq[0].tok * a.ld : 0);
  const float sx = xs_prologue(QT, src, n, a.mode, nw_staged ? nw_s : a.norm_w, !nw_staged, c.eps, smem, mk);
  const uint8_t *xq = (const uint8_t *)(smem + 320 + n);
  if (a.copy_src && blockIdx.x == 0) {
    // layer 0: the embedding row the prologue gathered becomes the residual
    const float4 *s4 = (const float4 *)src;
    float4 *d4 = (float4 *)a.copy_src;
    for (int i = threadIdx.x; i < a.ld / 4; i += kThreads) d4[i] = __ldg(s4 + i);
  }
  if (a.tslot && blockIdx.x == 0 && threadIdx.x == 0) a.tslot[1] = gtimer();
  // this lane's activation chunks, and the sum of all activations (each warp
  // adds the n bytes itself)
  uint4 xr[T::XMAX][T::XW];
#pragma unroll
  for (int j = 0; j < T::XMAX; j++) {
    const int k = li + lpr * j;
#pragma unroll
    for (int t = 0; t < T::XW; t++) {
      if (k < CH) {
        xr[j][t] = QT == QT_Q4 ? lds16(xq + (size_t)t * (n / 2) + 16 * k) : lds16(xq + 64 * k + 16 * t);
      } else {
        xr[j][t] = make_uint4(0, 0, 0, 0);
      }
    }
  }
  // the sum of all activations: the lpr lanes of a row group hold every
  // chunk once (zero past the row's end)
  uint32_t qsum = 0;
#pragma unroll
  for (int j = 0; j < T::XMAX; j++)
#pragma unroll
    for (int t = 0; t < T::XW; t++) {
      qsum = __dp4a(xr[j][t].x, 0x01010101u, qsum);
      qsum = __dp4a(xr[j][t].y, 0x01010101u, qsum);
      qsum = __dp4a(xr[j][t].z, 0x01010101u, qsum);
      qsum = __dp4a(xr[j][t].w, 0x01010101u, qsum);
    }
  for (int o = lpr >> 1; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
  const int32_t corr = T::OFF * (int32_t)qsum;
  if (mk) mk[20] = clock64();
  bool in_place = false;
  if (EPI == EPI_RESID) {
    if (a.resid_mode == RESID_ALWAYS) {
      in_place = true;
    } else if (a.resid_mode == RESID_MASK) {
      in_place = a.in_place_mask & 1;
    } else if (a.resid_mode == RESID_ATTN) {
      // Q4/Q6 use the in-place form only for caches of 2..6 tokens
      // (matVecOutAddRMSNormCPU), the ...OutOnly form otherwise
      // (model.go:3896-3908, 3975-3992, 4043-4062)
      const int len = c.sp->seq[0].len;
      in_place = len >= 1 && len + 1 <= 6;
    }
  }
  unsigned long long best = 0ull;
  bool ok = true;
#pragma unroll 1
  for (int st = 0; st < nst; st++) {
    const int r0 = lo + st * srows, nr = min(srows, hi - r0);
    const uint8_t *buf = g.stage + (size_t)(st % g.kSt) * kStageBytes;
    if (!gemv_wait(c, g, st)) ok = false;
    if (mk && st == 0) mk[21] = clock64();
#pragma unroll 1
    for (int base = warp * rpw; ok && base < nr; base += pass * RB) {
      int lr[RB];
      bool valid[RB];
      uint32_t da[RB], db[RB];
#pragma unroll
      for (int r = 0; r < RB; r++) {
        const int l = base + sub + r * pass;
        valid[r] = l < nr;
        lr[r] = valid[r] ? l : nr - 1;
        da[r] = xs_row_dot<QT>(buf + (size_t)lr[r] * P, xr, li, lpr, CH);
        if constexpr (two) db[r] = xs_row_dot<QT>(buf + (size_t)(srows + lr[r]) * P, xr, li, lpr, CH);
        else db[r] = 0u;
      }
#pragma unroll
      for (int r = 0; r < RB; r++) {
        for (int o = lpr >> 1; o > 0; o >>= 1) {
          da[r] += __shfl_xor_sync(0xffffffffu, da[r], o);
          if constexpr (two) db[r] += __shfl_xor_sync(0xffffffffu, db[r], o);
        }
      }
      if (li != 0) continue;
#pragma unroll
      for (int r = 0; r < RB; r++) {
        if (!valid[r]) continue;
        const int i = r0 - lo + lr[r];
        const int row = r0 + lr[r];
        const float v = vnni_finalize((int32_t)da[r] - corr, rsm_a[i], sx, scl_a[i]);
        if constexpr (EPI == EPI_STORE) {
          a.out[row] = v;
        } else if constexpr (EPI == EPI_RESID) {
          // rpre holds the rows of the first pass (base == warp * rpw)
          const float t = __fadd_rn(rpre_ok && base == warp * rpw ? rpre[r] : __ldcg(a.resid + row), v);
          a.vout[row] = t;
          if (in_place) a.resid[row] = t;
        } else if constexpr (EPI == EPI_SWIGLU) {
          const float u = vnni_finalize((int32_t)db[r] - corr, rsm_b[i], sx, scl_b[i]);
          a.out[row] = silu_mul(v, u);
        } else {
          if (a.logits) a.logits[row] = v;
          const unsigned long long k = argmax_key(v, row);
          best = k > best ? k : best;
        }
      }
    }
    __syncthreads();  // stage buffer free
    gemv_retire(a, g, st);
  }
  if (mk) mk[22] = clock64();
  if (threadIdx.x == 0) s_ring_setup = 0;
  if constexpr (EPI == EPI_ARGMAX) {
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (lane == 0 && best) atomicMax(a.argkey, best);
    if (a.argmax_finish) {
      __shared__ int is_last;
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicAdd(c.lm_count, 1u) == gridDim.x - 1;
        if (is_last) __threadfence();
      }
      __syncthreads();
      if (is_last) argmax_finish(c, 1, a.feed);
    }
  }
  __syncthreads();
  if (mk) mk[23] = clock64();
}

// Single sequence: the x-stationary path for Q4/Q6 (when the rows are narrow
// enough for its registers), else warp-row batches; one row per batch for the
// batched (M > 1) form.
template <int QT>
__device__ __forceinline__ void phase_gemv_q(const Ctx *c, const GemvArgs *a, int M, float *smem) {
  constexpr int R1 = 2;
  if (M <= 1) {
    if constexpr (QT != QT_Q8) {
      if (xs_fits<QT>(a->A.pitch) && xs_prologue_fits(a->mode, a->A.cols)) {
        // one instance per epilogue keeps each stage loop's code small
        switch (a->epi) {
          case EPI_STORE: phase_gemv_xs<QT, 2, EPI_STORE>(c, a, smem); break;
          case EPI_RESID: phase_gemv_xs<QT, 2, EPI_RESID>(c, a, smem); break;
          case EPI_SWIGLU: phase_gemv_xs<QT, 2, EPI_SWIGLU>(c, a, smem); break;
          default: phase_gemv_xs<QT, 2, EPI_ARGMAX>(c, a, smem); break;
        }
        return;
      }
    }
    phase_gemv_t<QT, 1, R1>(c, a, M, smem);
  } else {
    phase_gemv_t<QT, kMaxBatch, 1>(c, a, M, smem);
  }
}

__device__ __forceinline__ void phase_gemv(const Ctx *c, const GemvArgs *a, int M, float *smem) {
  if (c->qtype == QT_Q4)
    phase_gemv_q<QT_Q4>(c, a, M, smem);
  else if (c->qtype == QT_Q6)
    phase_gemv_q<QT_Q6>(c, a, M, smem);
  else
    phase_gemv_q<QT_Q8>(c, a, M, smem);
}
// ---------------------------------------------------------------------------
// KV cache and RoPE helpers
// ---------------------------------------------------------------------------
// A KV page holds 16 positions of every layer and kv head:
// [layer][kv head][K, V][16 positions][head_dim] floats, so the K and V rows
// of one (layer, kv head) are one contiguous 16 KB block.
__device__ __forceinline__ float *kv_ptr(const Ctx &c, const int *bt, int layer, int kind, int kvh, int t) {
  int page = bt[t / kPageTokens];
  return c.kv_pool + (size_t)page * c.page_floats +
         ((((size_t)layer * c.KVH + kvh) * 2 + kind) * kPageTokens + (t % kPageTokens)) * c.D;
}

// ropeFMA (internal/tensor/dot_amd64.s:5405-5440): a' = a*c - b*s,
// b' = fma(a, s, b*c) over pairs (i, i+D/2) of a head.
__device__ __forceinline__ void rope_pair(float &a, float &b, float cs, float sn) {
  float na = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
  float nb = __fmaf_rn(a, sn, __fmul_rn(b, cs));
  a = na;
  b = nb;
}

__device__ __forceinline__ void rope4(float4 &a, float4 &b, const float *cs, const float *sn) {
  float ax[4] = {a.x, a.y, a.z, a.w}, bx[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 4; j++) rope_pair(ax[j], bx[j], cs[j], sn[j]);
  a = make_float4(ax[0], ax[1], ax[2], ax[3]);
  b = make_float4(bx[0], bx[1], bx[2], bx[3]);
}

// cos/sin of frequencies 4*i4 .. 4*i4+3 for the M-RoPE position triple.
__device__ __forceinline__ void rope_cs4(const Ctx &c, const int *pos, int i4, float *cs, float *sn) {
  const int half = c.D / 2;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int i = i4 * 4 + j;
    int p = pos[c.sec_axis[i]];
    cs[j] = __ldg(c.rope_cos + (size_t)p * half + i);
    sn[j] = __ldg(c.rope_sin + (size_t)p * half + i);
  }
}

// ---------------------------------------------------------------------------
// Softmax of one head over n <= 32 scores, one score per lane (lane t holds
// token t), restating SoftmaxInPlace (ops.go:1199-1363) and the
// cacheAttentionLen2..6 paths (model.go:4797-5081).  Returns lane t's weight.
//   n == 1: weight 1; n == 2: the two-score form; 3..8: FastExpF32 with the
//   fixed sum trees; 9..15: FastExpF32 summed in order; >= 16: exp_fma over
//   the 16-aligned prefix nv summed in 16 lane chains + tree16, tokens at or
//   above nv keep their raw score (dot_amd64.s:6116-6210); all times 1/sum.
// ---------------------------------------------------------------------------
__device__ float warp_softmax_weight(float v, int n) {
  const int lane = threadIdx.x & 31;
  if (n == 1) return 1.0f;
  if (n == 2) {
    const float a = __shfl_sync(0xffffffffu, v, 0), b = __shfl_sync(0xffffffffu, v, 1);
    if (a >= b) {
      const float e = fast_exp(__fsub_rn(b, a));
      const float inv = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
      return lane == 0 ? inv : __fmul_rn(e, inv);
    }
    const float e = fast_exp(__fsub_rn(a, b));
    const float inv = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return lane == 0 ? __fmul_rn(e, inv) : inv;
  }
  float mx = lane < n ? v : -INFINITY;
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (n >= 16) {
    const int nv = n & ~15;
    const float e = lane < nv ? exp_fma(__fsub_rn(v, mx)) : 0.0f;
    const float hi = __shfl_down_sync(0xffffffffu, e, 16);
    float acc = __fadd_rn(0.0f, e);
    if (16 < nv) acc = __fadd_rn(acc, hi);
    float lanes[16];
#pragma unroll
    for (int l = 0; l < 16; l++) lanes[l] = __shfl_sync(0xffffffffu, acc, l);
    const float inv = __fdiv_rn(1.0f, tree16(lanes));
    return lane < nv ? __fmul_rn(e, inv) : __fmul_rn(v, inv);
  }
  const float e = lane < n ? fast_exp(__fsub_rn(v, mx)) : 0.0f;
  float sum;
  if (n <= 8) {
    float e8[8];
#pragma unroll
    for (int t = 0; t < 8; t++) e8[t] = __shfl_sync(0xffffffffu, e, t);
    const float p01 = __fadd_rn(e8[0], e8[1]), p23 = __fadd_rn(e8[2], e8[3]);
    const float p45 = __fadd_rn(e8[4], e8[5]), p67 = __fadd_rn(e8[6], e8[7]);
    const float q4 = __fadd_rn(p01, p23);
    switch (n) {
      case 3: sum = __fadd_rn(p01, e8[2]); break;
      case 4: sum = q4; break;
      case 5: sum = __fadd_rn(q4, e8[4]); break;
      case 6: sum = __fadd_rn(q4, p45); break;
      case 7: sum = __fadd_rn(__fadd_rn(q4, p45), e8[6]); break;
      default: sum = __fadd_rn(__fadd_rn(q4, p45), p67); break;
    }
  } else {
    sum = 0.0f;
#pragma unroll 1
    for (int t = 0; t < n; t++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, e, t));
  }
  return __fmul_rn(e, __fdiv_rn(1.0f, sum));
}

// ---------------------------------------------------------------------------
// Attention phase: RoPE, KV append, scores, softmax and value sums.
//
// Caches of n <= 32 positions form one 32-token item per (sequence m, kv
// head g) that applies the reference softmax exactly (incl. its small-n
// forms) and sums values in token order.  The item serves the G = QH/KVH
// query heads of its kv head (GQA): warp h computes head h's scores, one
// 128-wide dot per token split over the warp in the reference's 16-slot order
// (lane = slot + 16*half, 4 products per lane, xor-16 pair, then the tree16
// pairs by xor 8/4/2/1), so lane t ends holding token t's score.  K/V pages
// arrive by TMA bulk copy into shared memory, issued before the grid barrier
// that precedes the phase when the block's item is known (attn_prefetch);
// the item takes the new token's k and v from the QKV output, rotates k and
// appends both to the page (kvCache.append, model.go:5593-5612).
//
// Longer caches take two phases in the reference's exact order
// (attn_exact.cuh): the scores, run in this phase after the block's
// short-cache items, then the softmax and value sums.
// ---------------------------------------------------------------------------
struct AttnItem {
  int m, g, ch, t0, cnt, n, nch;
  bool exact;
};

// Per-block state of the K/V page loads, kept across phases of one launch.
__shared__ __align__(8) uint64_t s_kv_bar;
__shared__ uint32_t s_kv_parity;
__shared__ int s_kv_item;  // item whose pages are in flight / loaded, -1 none
// cos / sin of every RoPE frequency at each sequence's position of this step
__shared__ float s_rope_cs[kMaxBatch][kHeadDim / 2], s_rope_sn[kMaxBatch][kHeadDim / 2];
__shared__ int s_rope_ready;

}  // namespace ocrvl
#include "attn_exact.cuh"
namespace ocrvl {

// Item `it` of the step (caches of n <= kAttnChunk positions, one item per
// (sequence, kv head), from the launch's list of such sequences); false when
// it is past the last item.
__device__ __forceinline__ bool attn_item(const Ctx &c, const StepParams &sp, int it, AttnItem &I) {
  if (it >= s_ex_n * c.KVH) return false;
  const int m = s_ex_m[it / c.KVH];
  const int n = sp.seq[m].len + 1;
  I.m = m;
  I.g = it % c.KVH;
  I.ch = 0;
  I.t0 = 0;
  I.cnt = n;
  I.n = n;
  I.nch = 1;
  I.exact = true;
  return true;
}

__device__ __forceinline__ int attn_items_total(const Ctx &c, const StepParams &) { return s_ex_n * c.KVH; }

// Shared-memory layout of the attention phase (floats), from the base:
//   q [G][D] | wt [G][32]
// and the K/V page buffers K [32][D] | V [32][D] (32 KB) in the last slot of
// the GEMV stage ring, which the QKV phase before attention leaves unused.
__host__ __device__ __forceinline__ size_t attn_smem_floats() {
  return (size_t)kMaxGroup * kHeadDim + (size_t)kMaxGroup * kAttnChunk;
}
static_assert(2 * kAttnChunk * kHeadDim * 4 <= kStageBytes, "K/V buffers fit one ring slot");

__device__ __forceinline__ float *attn_kv_buf(const Ctx &c, int M, float *smem) {
  const int kSt = M <= 1 ? kStagesM1 : kStagesMB;
  return (float *)((uint8_t *)smem + gemv_prologue_bytes(c.qtype, M <= 1 ? 1 : kMaxBatch, c.pro_cols) +
                   (size_t)(kSt - 1) * kStageBytes);
}

// Called by every thread at the start of a launch that runs attention phases.
__device__ __forceinline__ void attn_block_init(const Ctx &c) {
  if (threadIdx.x == 0) {
    mbar_init(&s_kv_bar, 1);
    mbar_fence_init();
    s_kv_parity = 0;
    s_kv_item = -1;
    s_rope_ready = 0;
  }
  ax_block_init();
  av_block_init();
  ax_launch_init(c);
  __syncthreads();
}

// Named barrier among the threads lead .. kThreads-1 (lead a multiple of 32),
// used by work the block does while thread 0 waits at the grid barrier.
__device__ __forceinline__ void helpers_sync(int lead) {
  asm volatile("bar.sync 1, %0;" ::"r"(kThreads - lead) : "memory");
}

// Fills s_rope_cs / s_rope_sn for the step's sequences (threads lead..; the
// values become visible to the block at its next __syncthreads; positions are
// fixed for the whole launch).
__device__ void attn_rope_tables(const Ctx &c, int lead) {
  const StepParams &sp = *c.sp;
  const int half = c.D / 2;
  for (int p = threadIdx.x - lead; p < sp.M * half; p += kThreads - lead) {
    const int m = p / half, i = p % half;
    const int q = sp.seq[m].pos[c.sec_axis[i]];
    s_rope_cs[m][i] = __ldg(c.rope_cos + (size_t)q * half + i);
    s_rope_sn[m][i] = __ldg(c.rope_sin + (size_t)q * half + i);
  }
  if ((int)threadIdx.x == lead) s_rope_ready = 1;
}

// Thread 0: bulk copies of item I's K and V page(s) into the K/V buffers.
__device__ __forceinline__ void attn_issue_kv(const Ctx &c, int layer, const AttnItem &I, float *kvbuf) {
  float *smem = kvbuf;
  const int *bt = c.sp->seq[I.m].bt;
  const int p0 = I.t0 / kPageTokens;
  const int np = (I.cnt + kPageTokens - 1) / kPageTokens;
  const uint32_t pbytes = (uint32_t)kPageTokens * c.D * 4;
  // the buffers were last touched by ordinary loads/stores of this block
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_expect_tx(&s_kv_bar, 2u * np * pbytes);
  for (int p = 0; p < np; p++) {
    const float *kp = kv_ptr(c, bt, layer, 0, I.g, (p0 + p) * kPageTokens);
    const float *vp = kv_ptr(c, bt, layer, 1, I.g, (p0 + p) * kPageTokens);
    bulk_g2s(smem + (size_t)p * kPageTokens * c.D, kp, pbytes, &s_kv_bar);
    bulk_g2s(smem + (size_t)kAttnChunk * c.D + (size_t)p * kPageTokens * c.D, vp, pbytes, &s_kv_bar);
  }
}

// Issues this block's first attention item's K/V loads ahead of the phase,
// before the QKV phase of the layer, when that phase's stages leave the last
// ring slot free.  Thread 0 acts.
__device__ void attn_prefetch(const Ctx &c, int layer, float *smem, int lead) {
  AttnItem I;
  if ((int)threadIdx.x != lead || s_kv_item >= 0 || !attn_item(c, *c.sp, blockIdx.x, I)) return;
  const int M = c.sp->M;
  const int kSt = M <= 1 ? kStagesM1 : kStagesMB;
  const DMat &A = c.layers[layer].qkv;
  int lo, hi;
  gemv_slab(0, A.rows, blockIdx.x, gridDim.x, lo, hi);
  const int srows = kStageBytes / A.pitch;
  if ((hi - lo + srows - 1) / srows > kSt - 1) return;
  attn_issue_kv(c, layer, I, attn_kv_buf(c, M, smem));
  s_kv_item = blockIdx.x;
}

// Waits for the outstanding K/V load of an n <= kAttnChunk item.
__device__ __forceinline__ void attn_drain_item(const Ctx &c) {
  if (threadIdx.x == 0 && s_kv_item >= 0) {
    mbar_wait(&s_kv_bar, s_kv_parity, c.err);
    s_kv_parity ^= 1u;
    s_kv_item = -1;
  }
}

// Waits for every outstanding K/V load (before the block leaves the kernel).
__device__ void attn_drain(const Ctx &c) {
  attn_drain_item(c);
  if (threadIdx.x == 0) ax_drain(c);
  __syncthreads();
}

// Thread `lead`, ahead of the attention phase of `layer`: the K copies of
// the block's first long-cache chunks (attn_exact.cuh).  during_qkv: before
// the QKV phase, whose weight stages then share the ring (single-sequence
// steps only, two chunk buffers in each ring slot the block's QKV slab leaves
// free at the top).  A block with n <= kAttnChunk items loads those first and
// skips this.
__device__ void attn_range_prefetch(const Ctx &c, int layer, float *smem, int lead, bool during_qkv) {
  const StepParams &sp = *c.sp;
  if ((int)threadIdx.x != lead || attn_items_total(c, sp) > (int)blockIdx.x) return;
  int upto = kAxKBufs;
  if (during_qkv) {
    if (sp.M > 1) return;
    const DMat &A = c.layers[layer].qkv;
    int lo, hi;
    gemv_slab(0, A.rows, blockIdx.x, gridDim.x, lo, hi);
    const int srows = kStageBytes / A.pitch;
    upto = min(upto, 2 * (kStagesM1 - (hi - lo + srows - 1) / srows));
  }
  ax_issue_upto(c, layer, smem, upto);
}

__device__ __noinline__ void phase_attn(const Ctx *cp, int layer, int append_only, int coop, float *smem_arg) {
  float *const smem = dyn_smem();  // == smem_arg (the aligned dynamic base)
  (void)smem_arg;
  const Ctx &c = *cp;
  rg_bmark(c, 0);
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH, D = c.D, D4 = D / 4, H4 = D / 8;
  const int qkvld = (c.QH + 2 * c.KVH) * D;
  float *Ks = attn_kv_buf(c, sp.M, smem);         // [32][D]
  float *Vs = Ks + kAttnChunk * D;                 // [32][D]
  float *qs = smem;                                // [G][D]
  float *wt = qs + kMaxGroup * D;                  // [G][32]
  __shared__ float rcs_l[kHeadDim / 2], rsn_l[kHeadDim / 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int items = attn_items_total(c, sp);
  int tab_m = -1;  // sequence whose RoPE values rcs/rsn hold
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    AttnItem I;
    attn_item(c, sp, it, I);
    const int len = I.n - 1;
    // one K/V copy in flight at a time: a copy started for another item (the
    // one prefetched before the phase, when the block moves past it)
    // completes before the buffers are reused
    if (threadIdx.x == 0 && s_kv_item >= 0 && (s_kv_item != it || append_only)) {
      mbar_wait(&s_kv_bar, s_kv_parity, c.err);
      s_kv_parity ^= 1u;
      s_kv_item = -1;
    }
    const int *pos = sp.seq[I.m].pos;
    const bool has_rope = pos[0] != 0 || pos[1] != 0 || pos[2] != 0;
    const float *qkv = c.qkv + (size_t)I.m * qkvld;
    // ---- K/V pages (unless prefetched for this item), RoPE table of the position
    if (threadIdx.x == 0 && s_kv_item != it && !append_only) {
      attn_issue_kv(c, layer, I, Ks);
      s_kv_item = it;
    }
    const bool rope_pre = s_rope_ready != 0;
    if (!rope_pre && threadIdx.x < D / 2 && I.m != tab_m) {
      const int i = threadIdx.x;
      const int p = pos[c.sec_axis[i]];
      rcs_l[i] = __ldg(c.rope_cos + (size_t)p * (D / 2) + i);
      rsn_l[i] = __ldg(c.rope_sin + (size_t)p * (D / 2) + i);
    }
    __syncthreads();
    tab_m = I.m;
    const float *rcs = rope_pre ? s_rope_cs[I.m] : rcs_l;
    const float *rsn = rope_pre ? s_rope_sn[I.m] : rsn_l;
    // ---- q (rotated) into shared memory; the new token's k (rotated) and v
    // appended to the page and placed into the K/V buffers (after the copy)
    if (!append_only) {
      for (int p = threadIdx.x; p < G * H4; p += kThreads) {
        const int hh = p / H4, i4 = p % H4;
        const float4 *qh = (const float4 *)(qkv + (size_t)(I.g * G + hh) * D);
        float4 ra = __ldcg(qh + i4), rb = __ldcg(qh + i4 + H4);
        if (has_rope) rope4(ra, rb, rcs + 4 * i4, rsn + 4 * i4);
        ((float4 *)(qs + hh * D))[i4] = ra;
        ((float4 *)(qs + hh * D))[i4 + H4] = rb;
      }
    }
    float4 nk_a, nk_b, nv4;
    if (threadIdx.x < D4) {
      if (threadIdx.x < H4) {
        const float4 *kn = (const float4 *)(qkv + (size_t)(c.QH + I.g) * D);
        nk_a = __ldcg(kn + threadIdx.x);
        nk_b = __ldcg(kn + threadIdx.x + H4);
        if (has_rope) rope4(nk_a, nk_b, rcs + 4 * threadIdx.x, rsn + 4 * threadIdx.x);
        float4 *kd = (float4 *)kv_ptr(c, sp.seq[I.m].bt, layer, 0, I.g, len);
        kd[threadIdx.x] = nk_a;
        kd[threadIdx.x + H4] = nk_b;
      }
      nv4 = __ldcg((const float4 *)(qkv + (size_t)(c.QH + c.KVH + I.g) * D) + threadIdx.x);
      ((float4 *)kv_ptr(c, sp.seq[I.m].bt, layer, 1, I.g, len))[threadIdx.x] = nv4;
    }
    if (append_only) {
      __syncthreads();
      continue;
    }
    if (threadIdx.x == 0) {
      mbar_wait(&s_kv_bar, s_kv_parity, c.err);
      s_kv_parity ^= 1u;
      s_kv_item = -1;
    }
    __syncthreads();
    if (threadIdx.x < D4) {
      if (threadIdx.x < H4) {
        ((float4 *)(Ks + (size_t)len * D))[threadIdx.x] = nk_a;
        ((float4 *)(Ks + (size_t)len * D))[threadIdx.x + H4] = nk_b;
      }
      ((float4 *)(Vs + (size_t)len * D))[threadIdx.x] = nv4;
    }
    __syncthreads();
    // ---- scores (warp = head) and the reference softmax
    const int slot = lane & 15, half = lane >> 4;
    if (warp < G) {
      const float *q = qs + warp * D;
      float qv[4];
#pragma unroll
      for (int jj = 0; jj < 4; jj++) qv[jj] = q[16 * (4 * half + (jj ^ half)) + slot];
      float mine = 0.0f;
#pragma unroll 4
      for (int tt = 0; tt < I.cnt; tt++) {
        const float *k = Ks + (size_t)tt * D;
        float pr[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) pr[jj] = __fmul_rn(qv[jj], k[16 * (4 * half + (jj ^ half)) + slot]);
        // products in j order: half 0 read j = 0,1,2,3; half 1 read j = 5,4,7,6
        float s4 = half ? __fadd_rn(__fadd_rn(pr[1], pr[0]), __fadd_rn(pr[3], pr[2]))
                        : __fadd_rn(__fadd_rn(pr[0], pr[1]), __fadd_rn(pr[2], pr[3]));
        float r = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 16));  // slot sum (halves commute)
        r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 8));
        r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
        r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
        r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
        if (lane == tt) mine = __fmul_rn(r, c.attn_scale);
      }
      float w = warp_softmax_weight(mine, I.n);  // every lane takes part in the shuffles
      if (lane >= I.cnt) w = 0.0f;
      wt[warp * kAttnChunk + lane] = w;
    }
    __syncthreads();
    // ---- value sums: thread = (head, 4 dims), token order
    const size_t hbase = (size_t)I.m * c.QH + (size_t)I.g * G;
    for (int p = threadIdx.x; p < G * D4; p += kThreads) {
      const int hh = p / D4, d4 = p % D4;
      const float *w = wt + hh * kAttnChunk;
      const float4 v0 = ((const float4 *)Vs)[d4];
      float4 acc = make_float4(__fmul_rn(w[0], v0.x), __fmul_rn(w[0], v0.y), __fmul_rn(w[0], v0.z), __fmul_rn(w[0], v0.w));
#pragma unroll 4
      for (int t = 1; t < I.cnt; t++) {
        const float4 v = ((const float4 *)(Vs + (size_t)t * D))[d4];
        const float wv = w[t];
        acc.x = __fmaf_rn(wv, v.x, acc.x);
        acc.y = __fmaf_rn(wv, v.y, acc.y);
        acc.z = __fmaf_rn(wv, v.z, acc.z);
        acc.w = __fmaf_rn(wv, v.w, acc.w);
      }
      ((float4 *)(c.head + (hbase + hh) * D))[d4] = acc;
    }
    __syncthreads();
  }
  attn_drain_item(c);
  __syncthreads();
  (void)coop;
  // ---- caches of more than kAttnChunk positions: their scores (the
  // softmax and value sums follow in phase_attn_values after a grid barrier)
  if (append_only) {
    if (threadIdx.x == 0) ax_drain(c);
    phase_append_long(c, layer);
    __syncthreads();
  } else {
    phase_attn_scores(cp, layer, smem);
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

}  // namespace ocrvl
