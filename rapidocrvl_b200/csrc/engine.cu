// Host engine and C ABI (include/ocrvl_cuda.h) of the B200 decode path.
//
// A decode step runs as ONE persistent cooperative kernel (k_step): every
// block walks the phases of decoder.cuh for all layers, separated by a grid
// barrier whose waits are bounded (a timed-out wait sets an error word and
// every block returns).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>

#include "../../include/ocrvl_cuda.h"
#include "decoder.cuh"
#include "batched.cuh"
#include "sample.cuh"

using namespace ocrvl;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}

#define CK(call)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess) return fail(OCRVL_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

int packed_row_bytes(int type, int cols) {
  switch (type) {
    case OCRVL_Q8_ROW: return cols;
    case OCRVL_Q4_ROW: return (cols + 1) / 2;
    case OCRVL_Q6_ROW: return (cols * 6 + 7) / 8;
  }
  return -1;
}

}  // namespace

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
namespace ocrvl {

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier of the cooperative step kernel: every block adds 1 to a
// monotonic counter with a non-returning release reduction and polls it with
// acquire loads until it reaches `target` (the host tracks the counter's value
// across launches).  Waits are bounded: after kBarrierSpins polls the block
// records an error and leaves; waiting blocks also leave once any block has
// recorded one.  Returns false on error.
constexpr unsigned long long kBarrierSpins = 1ull << 22;  // default poll limit (Ctx::bar_spins)
__shared__ int s_grid_ok;
// Arrival half: after the block's phase work (all threads), thread 0 adds 1.
__device__ __forceinline__ void grid_arrive(const Ctx &c) {
  __syncthreads();
  if (threadIdx.x == 0) red_add_release(c.bar_count, 1u);
}
// Waiting half: thread 0 polls until the counter reaches `target`; the block
// may do work that does not depend on other blocks between the two halves.
__device__ bool grid_wait(const Ctx &c, unsigned target) {
  if (threadIdx.x == 0) {
    int ok = 1;
    unsigned long long spins = 0;
    while ((int)(ld_acquire(c.bar_count) - target) < 0) {
      ++spins;
      if (spins > c.bar_spins || ((spins & 1023) == 0 && *(volatile int *)c.err)) {
        atomicExch(c.err, 1);
        ok = 0;
        break;
      }
    }
    s_grid_ok = ok;
  }
  __syncthreads();
  return s_grid_ok != 0;
}
__device__ bool grid_sync(const Ctx &c, unsigned target) {
  grid_arrive(c);
  return grid_wait(c, target);
}

// qkv, attention (short caches; long caches' scores), long caches' softmax
// and values, o, gate/up, down
constexpr int kLayerPhases = 6;
constexpr int kPhaseLM = 6;      // lm_head argmax (after the last layer)

__host__ __device__ __forceinline__ unsigned barriers_per_step(int L, int any_logits) {
  return any_logits ? (unsigned)(kLayerPhases * L) : (unsigned)(kLayerPhases * (L - 1) + 1);
}

// GEMV arguments of a phase, built by thread 0 in shared memory.
__shared__ GemvArgs s_args;

__device__ void build_args(const Ctx &c, int phase, int layer, int any_logits, int do_embed, int feed, int tidx) {
  GemvArgs &sa = s_args;
  const LayerW &L = c.layers[layer < c.L ? layer : c.L - 1];
  const bool last = layer == c.L - 1;
  memset(&sa, 0, sizeof(sa));
  sa.tslot = c.trace ? c.trace + 4 * tidx : nullptr;
    switch (phase) {
      case 0:  // QKV with the input RMSNorm (layer 0: embedding gather) as prologue
        sa.A = L.qkv;
        sa.row_begin = (last && !any_logits) ? c.QH * c.D : 0;
        sa.row_end = L.qkv.rows;
        sa.ld = c.H;
        if (layer == 0 && do_embed) {
          sa.src = c.embed;
          sa.src_tok = 1;
          sa.copy_src = c.h;
        } else {
          sa.src = c.h;
        }
        sa.mode = PRO_RMSNORM;
        sa.norm_w = L.ln1;
        sa.epi = EPI_STORE;
        sa.out = c.qkv;
        sa.ldo = (c.QH + 2 * c.KVH) * c.D;
        break;
      case 3:  // o projection + residual
        sa.A = L.o;
        sa.row_end = L.o.rows;
        sa.src = c.head;
        sa.ld = c.QH * c.D;
        sa.mode = PRO_PLAIN;
        sa.epi = EPI_RESID;
        sa.ldo = c.H;
        sa.resid = c.h;
        sa.vout = c.vbuf;
        sa.resid_mode = RESID_ATTN;
        break;
      case 4:  // gate/up with the post-attention AddRMSNorm as prologue
        sa.A = L.gate;
        sa.B = L.up;
        sa.row_end = L.gate.rows;
        sa.src = c.vbuf;
        sa.ld = c.H;
        sa.mode = PRO_ADDNORM;
        sa.norm_w = L.ln2;
        sa.epi = EPI_SWIGLU;
        sa.out = c.g;
        sa.ldo = c.I;
        break;
      case 5:  // down projection + residual (last layer: out-only)
        sa.A = L.down;
        sa.row_end = L.down.rows;
        sa.src = c.g;
        sa.ld = c.I;
        sa.mode = PRO_PLAIN;
        sa.epi = EPI_RESID;
        sa.ldo = c.H;
        sa.resid = c.h;
        sa.vout = c.vbuf;
        sa.resid_mode = last ? RESID_NEVER : RESID_ALWAYS;
        break;
      default:  // lm_head argmax with the final AddRMSNorm as prologue
        sa.A = c.lm_head;
        sa.row_end = c.lm_head.rows;
        sa.src = c.vbuf;
        sa.ld = c.H;
        sa.mode = PRO_ADDNORM;
        sa.norm_w = c.final_norm;
        sa.epi = EPI_ARGMAX;
        sa.ldo = c.V;
        sa.argkey = c.argkey;
        sa.logits = c.sp->store_logits ? c.logits : nullptr;
        sa.argmax_finish = 1;
        sa.feed = feed;
        break;
    }
}

__device__ __forceinline__ bool is_gemv_phase(int phase) { return phase != 1 && phase != 2; }

// Work for phase (phase, layer) that needs nothing from other blocks, done by
// threads kHelper.. while thread 0 waits at the grid barrier before it: the
// GEMV arguments, the first weight stages and the staged scales / norm
// weights; before a QKV phase also the K/V pages of the block's first
// short-cache item or (single-sequence steps) of its first long-cache chunks,
// and before the attention phase the remaining first chunks.  The block's
// next __syncthreads publishes the results.
constexpr int kHelper = 32;
template <int QT>
__device__ void prepare_phase(const Ctx &c, int phase, int layer, int M, int any_logits, int do_embed, int feed,
                              float *smem, int tidx) {
  const bool kv_only = layer == c.L - 1 && !any_logits;
  if (!is_gemv_phase(phase)) {
    if (phase == 1 && !kv_only) attn_range_prefetch(c, layer, smem, kHelper, false);
    return;
  }
  if (threadIdx.x == kHelper) build_args(c, phase, layer, any_logits, do_embed, feed, tidx);
  helpers_sync(kHelper);
  gemv_setup(QT, c, s_args, M, smem, kHelper, kThreads - kHelper);
  if (phase == 0) {
    attn_prefetch(c, layer, smem, kHelper);
    if (!kv_only) attn_range_prefetch(c, layer, smem, kHelper, true);
  }
  if (threadIdx.x == kHelper) s_ring_setup = 1;
}

// One phase of layer `layer`; `prepared`: prepare_phase ran for it.
template <int QT>
__device__ void run_phase(const Ctx &c, int phase, int layer, int M, int any_logits, int do_embed, int feed,
                          float *smem, int tidx, int coop, bool prepared) {
  unsigned long long *tslot = c.trace ? c.trace + 4 * tidx : nullptr;
  if (tslot && blockIdx.x == 0 && threadIdx.x == 0) tslot[0] = gtimer();
  const bool last = layer == c.L - 1;
  if (phase == 1) {
    phase_attn(&c, layer, last && !any_logits, coop, smem);
  } else if (phase == 2) {
    phase_attn_values(&c, layer, smem);
  } else {
    if (!prepared) {
      if (threadIdx.x == 0) build_args(c, phase, layer, any_logits, do_embed, feed, tidx);
      __syncthreads();
    }
    phase_gemv_q<QT>(&c, &s_args, M, smem);
  }
  if (tslot && threadIdx.x == 0) atomicMax(tslot + 2, gtimer());
}

// Ctx is copied into shared memory once per launch, and with it the step
// parameters and (up to kSmemLayers layers) the layer descriptors, so phases
// start without global-memory round trips for their arguments.
constexpr int kSmemLayers = 32;
__shared__ StepParams s_step_params;
__shared__ LayerW s_layer_desc[kSmemLayers];

__device__ __forceinline__ void copy_words(void *dst, const void *src, int bytes) {
  for (int i = threadIdx.x; i < bytes / 4; i += kThreads) ((int *)dst)[i] = ((const int *)src)[i];
}

__device__ __forceinline__ float *align_dyn_smem(void *) { return dyn_smem(); }

#define OCRVL_CTX_TO_SMEM(cv)                                                        \
  __shared__ Ctx sctx;                                                               \
  if (threadIdx.x == 0) sctx = cv;                                                   \
  if (cv.sp) copy_words(&s_step_params, cv.sp, (int)sizeof(StepParams));             \
  if (cv.layers && cv.L <= kSmemLayers)                                              \
    copy_words(s_layer_desc, cv.layers, (int)sizeof(LayerW) * cv.L);                 \
  __syncthreads();                                                                   \
  if (threadIdx.x == 0) {                                                            \
    if (cv.sp) sctx.sp = &s_step_params;                                             \
    if (cv.layers && cv.L <= kSmemLayers) sctx.layers = s_layer_desc;                \
  }                                                                                  \
  __syncthreads();                                                                   \
  const Ctx &c = sctx;

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    k_step(Ctx cv, int M, int any_logits, int do_embed, int feed, unsigned bar_base, int nsteps) {
  extern __shared__ float4 smem4[];
  float *smem = align_dyn_smem(smem4);
  OCRVL_CTX_TO_SMEM(cv);
  if (nsteps > 1) {  // the trace holds one step
    Ctx &cm = sctx;
    if (threadIdx.x == 0) cm.trace = nullptr;
    __syncthreads();
  }
  attn_block_init(c);
  ring_init();
  unsigned k = 0;
  for (int st = 0; st < nsteps; st++) {
    if (st > 0) {
      // the next device-fed step: the previous step's lm_head phase (its last
      // block) wrote the step parameters; every block reloads them (from L2)
      // and the per-launch attention geometry
      grid_arrive(c);
      if (!grid_wait(c, bar_base + (++k) * gridDim.x)) {
        attn_drain(c);
        gemv_drain(c);
        return;
      }
      for (int i = threadIdx.x; i < (int)sizeof(StepParams) / 4; i += kThreads)
        ((int *)&s_step_params)[i] = __ldcg((const int *)cv.sp + i);
      if (threadIdx.x == 0) s_rope_ready = 0;
      __syncthreads();
      ax_launch_init(c);
      __syncthreads();
    }
    int t = 0;
    if (threadIdx.x >= kHelper) prepare_phase<QT>(c, 0, 0, M, any_logits, do_embed, feed, smem, 0);
    __syncthreads();
    for (int l = 0; l < c.L; l++) {
      const bool kv_only = l == c.L - 1 && !any_logits;
      for (int ph = 0; ph < kLayerPhases; ph++, t++) {
        run_phase<QT>(c, ph, l, M, any_logits, do_embed, feed, smem, t, 1, is_gemv_phase(ph));
        if (kv_only && ph == 1) return;
        grid_arrive(c);
        // while thread 0 waits for the other blocks, the helper threads set up
        // the next phase and (once per step) the RoPE values of this step
        if (threadIdx.x >= kHelper) {
          const bool more = ph + 1 < kLayerPhases || l + 1 < c.L || any_logits;
          if (more) {
            const int nph = ph + 1 < kLayerPhases ? ph + 1 : (l + 1 < c.L ? 0 : kPhaseLM);
            const int nl = ph + 1 < kLayerPhases ? l : l + 1;
            if (!(nl == c.L - 1 && !any_logits && nph > 1))
              prepare_phase<QT>(c, nph, nl, M, any_logits, do_embed, feed, smem, t + 1);
          }
          if (l == 0 && ph == 0) attn_rope_tables(c, kHelper);
        }
        if (!grid_wait(c, bar_base + (++k) * gridDim.x)) {
          attn_drain(c);
          gemv_drain(c);
          return;
        }
        if (c.trace && blockIdx.x == 0 && threadIdx.x == 0) c.trace[4 * t + 3] = gtimer();
      }
    }
    if (any_logits) run_phase<QT>(c, kPhaseLM, c.L, M, any_logits, do_embed, feed, smem, t, 1, true);
  }
}

template <int QT>
__global__ void __launch_bounds__(kThreads) k_gemv(Ctx cv, GemvArgs av, int M) {
  extern __shared__ float4 smem4[];
  OCRVL_CTX_TO_SMEM(cv);
  ring_init();
  __shared__ GemvArgs sa;
  if (threadIdx.x == 0) sa = av;
  __syncthreads();
  phase_gemv_q<QT>(&c, &sa, M, dyn_smem());
}

__global__ void __launch_bounds__(kThreads) k_addnorm_out(Ctx c, const float *v, int n, int M, const float *w,
                                                          float *out) {
  extern __shared__ float4 smem4[];
  phase_addnorm_out(c, v, n, M, w, out, (float *)smem4);
}

__global__ void __launch_bounds__(kThreads) k_rmsnorm_out(Ctx c, const float *x, int n, int M, const float *w,
                                                          float *out) {
  extern __shared__ float4 smem4[];
  phase_rmsnorm_out(c, x, n, M, w, out, (float *)smem4);
}

__global__ void k_argmax_ids(const unsigned long long *keys, int M, int *ids) {
  int m = threadIdx.x;
  if (m < M) ids[m] = argmax_key_row(keys[m]);
}

// ---------------------------------------------------------------------------
// Batched step kernel (kMaxBatch < M <= kMaxSeqs, Q4 / Q6): per layer the
// input quantisation and tcgen05 int8 GEMM for QKV, o, gate/up and down, the
// attention phase between QKV and o; grid barrier after each phase.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int gemm_nt(int rows, int grid) {
  const int per = (rows + grid - 1) / grid;
  const int nt = (per + 15) & ~15;
  return nt < 256 ? nt : 256;  // kMaxNT
}
__host__ __device__ __forceinline__ unsigned barriers_per_step_b(int L, int any_logits) {
  // per layer: 4 quantisation phases, 4 GEMMs, the two attention phases, the
  // o and down projections' split-K finalize; then the final norm (and
  // lm_head)
  return any_logits ? (unsigned)(12 * L + 1) : (unsigned)(12 * (L - 1) + 2);
}

template <int QT>
__device__ void step_b_body(const Ctx &c, const BatchedW *bw, uint32_t tmem, int any_logits, int do_embed, int feed,
                            unsigned bar_base, float *smem) {
  __shared__ GemmArgs sg;
  unsigned k = 0;
  // trace (OCRVL_TRACE): per phase [start, 0, last block's end, barrier exit]
  int t = 0;
  if (c.trace && blockIdx.x == 0 && threadIdx.x == 0) c.trace[0] = gtimer();
  auto sync = [&]() {
    if (c.trace && threadIdx.x == 0 && t < 256) atomicMax(c.trace + 4 * t + 2, gtimer());
    const bool ok = grid_sync(c, bar_base + (++k) * gridDim.x);
    if (c.trace && blockIdx.x == 0 && threadIdx.x == 0 && t + 1 < 256) {
      const unsigned long long now = gtimer();
      c.trace[4 * t + 3] = now;
      c.trace[4 * (t + 1)] = now;
    }
    t++;
    return ok;
  };
  auto gemm = [&](const GemmArgs &g) {
    if (threadIdx.x == 0) sg = g;
    __syncthreads();
    phase_gemm_b<QT>(&c, bw, &sg, tmem, smem);
  };
  const int qkvld = (c.QH + 2 * c.KVH) * c.D;
  for (int l = 0; l < c.L; l++) {
    const LayerW &L = c.layers[l];
    const bool last = l == c.L - 1, kv_only = last && !any_logits, emb = l == 0 && do_embed;
    phase_quant_b(&c, bw, emb ? c.embed : c.h, c.H, emb, c.H, PRO_RMSNORM, L.ln1, emb ? c.h : nullptr, smem);
    if (!sync()) return;
    {
      GemmArgs g{};
      g.mapA = bw_map(*bw, l, 0);
      g.A = L.qkv;
      g.row_begin = kv_only ? c.QH * c.D : 0;
      g.row_end = L.qkv.rows;
      g.K = c.H;
      g.nt = gemm_nt(L.qkv.rows, gridDim.x);
      g.u = gemm_u(QT, g.nt);
      g.epi = EPI_STORE;
      g.out = c.qkv;
      g.ldo = qkvld;
      gemm(g);
    }
    if (!sync()) return;
    phase_attn(&c, l, kv_only, 1, smem);
    if (kv_only) return;
    if (!sync()) return;
    phase_attn_values(&c, l, smem);
    if (!sync()) return;
    phase_quant_b(&c, bw, c.head, c.QH * c.D, 0, c.QH * c.D, PRO_PLAIN, nullptr, nullptr, smem);
    if (!sync()) return;
    {
      GemmArgs g{};
      g.mapA = bw_map(*bw, l, 1);
      g.A = L.o;
      g.row_end = L.o.rows;
      g.K = c.QH * c.D;
      g.ks = down_splits(L.o.cols);
      g.nt = gemm_nt(L.o.rows, gridDim.x / g.ks);
      g.u = gemm_u(QT, g.nt);
      g.epi = EPI_RESID;
      g.ldo = c.H;
      g.part = bw->part;
      gemm(g);
    }
    if (!sync()) return;
    phase_splitk_resid(&c, bw, &L.o, down_splits(L.o.cols), c.H, c.h, c.vbuf, RESID_ATTN);
    if (!sync()) return;
    phase_quant_b(&c, bw, c.vbuf, c.H, 0, c.H, PRO_ADDNORM, L.ln2, nullptr, smem);
    if (!sync()) return;
    {
      GemmArgs g{};
      g.mapA = bw_map(*bw, l, 2);
      g.mapB = bw_map(*bw, l, 3);
      g.A = L.gate;
      g.B = L.up;
      g.row_end = L.gate.rows;
      g.K = c.H;
      g.nt = gemm_nt(L.gate.rows, gridDim.x);
      g.u = gemm_u(QT, g.nt);
      g.epi = EPI_SWIGLU;
      g.out = c.g;
      g.ldo = c.I;
      gemm(g);
    }
    if (!sync()) return;
    phase_quant_b(&c, bw, c.g, c.I, 0, c.I, PRO_PLAIN, nullptr, nullptr, smem);
    if (!sync()) return;
    {
      GemmArgs g{};
      g.mapA = bw_map(*bw, l, 4);
      g.A = L.down;
      g.row_end = L.down.rows;
      g.K = c.I;
      g.ks = down_splits(L.down.cols);
      g.nt = gemm_nt(L.down.rows, gridDim.x / g.ks);
      g.u = gemm_u(QT, g.nt);
      g.epi = EPI_RESID;
      g.ldo = c.H;
      g.part = bw->part;
      gemm(g);
    }
    if (!sync()) return;
    phase_splitk_resid(&c, bw, &L.down, down_splits(L.down.cols), c.H, c.h, c.vbuf, last ? RESID_NEVER : RESID_ALWAYS);
    if (!sync()) return;
  }
  phase_quant_b(&c, bw, c.vbuf, c.H, 0, c.H, PRO_ADDNORM, c.final_norm, nullptr, smem);
  if (!sync()) return;
  GemmArgs g{};
  g.mapA = bw_map(*bw, c.L, 0);
  g.A = c.lm_head;
  g.row_end = c.lm_head.rows;
  g.K = c.H;
  g.nt = gemm_nt(c.lm_head.rows, gridDim.x);
  g.u = gemm_u(QT, g.nt);
  g.epi = EPI_ARGMAX;
  g.ldo = c.V;
  g.argkey = c.argkey;
  g.logits = c.sp->store_logits ? c.logits : nullptr;
  g.argmax_finish = 1;
  g.feed = feed;
  gemm(g);
  if (c.trace && threadIdx.x == 0 && t < 256) atomicMax(c.trace + 4 * t + 2, gtimer());
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    k_step_b(Ctx cv, BatchedW bwv, int any_logits, int do_embed, int feed, unsigned bar_base) {
  extern __shared__ float4 smem4[];
  float *smem = align_dyn_smem(smem4);
  OCRVL_CTX_TO_SMEM(cv);
  __shared__ BatchedW sbw;
  __shared__ uint32_t s_tmem;
  if (threadIdx.x == 0) sbw = bwv;
  attn_block_init(c);
  ring_init();
  if (threadIdx.x < 32) tmem_alloc(&s_tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  step_b_body<QT>(c, &sbw, s_tmem, any_logits, do_embed, feed, bar_base, smem);
  // every exit path: no TMEM held when the block leaves
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(s_tmem, kTmemCols);
}

// Seeded pseudo-random K/V for positions [0, n) of the pages listed in
// `pages` (np of them): K uniform in [-0.5, 0.5), V in [-1, 1), a hash of
// (seed, position, layer, kv head, K|V, dim).  Grid-stride over float4s of
// the pages.
__global__ void k_fill_kv(float *pool, long long page_floats, const int *pages, int np, int n, int L, int KVH, int D,
                          unsigned long long seed) {
  const long long per4 = page_floats / 4, total = per4 * np;
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(q / per4);
    const long long r = (q - (long long)p * per4) * 4;  // float offset within the page
    const int d = (int)(r % D), row = (int)((r / D) % kPageTokens);
    const long long blk = r / ((long long)D * kPageTokens);  // (layer, kv head, K|V)
    const int kind = (int)(blk & 1);
    const int pos = p * kPageTokens + row;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (pos < n) {
      float e[4];
      for (int j = 0; j < 4; j++) {
        unsigned long long h = seed ^ ((unsigned long long)pos << 32) ^ ((unsigned long long)blk << 12) ^ (d + j);
        h ^= h >> 33;
        h *= 0xff51afd7ed558ccdull;
        h ^= h >> 33;
        h *= 0xc4ceb9fe1a85ec53ull;
        h ^= h >> 33;
        const float u = (float)(h >> 40) * (1.0f / 16777216.0f);  // [0, 1)
        e[j] = kind ? 2.0f * u - 1.0f : u - 0.5f;
      }
      v = make_float4(e[0], e[1], e[2], e[3]);
    }
    ((float4 *)(pool + (size_t)pages[p] * page_floats))[r / 4] = v;
  }
  (void)L;
  (void)KVH;
}

// Per-row sum of unpacked int8 weights; one warp per row.
__global__ void k_rowsum(int type, const uint8_t *w, int rows, int cols, int pitch, int32_t *out) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const uint8_t *r = w + (size_t)warp * pitch;
  int s = 0;
  for (int cidx = lane; cidx < cols; cidx += 32) {
    int v;
    if (type == QT_Q8) {
      v = (int8_t)r[cidx];
    } else if (type == QT_Q4) {
      uint8_t b = r[cidx >> 1];
      v = ((cidx & 1) ? (b >> 4) : (b & 0x0F)) - 8;
    } else {
      int bit = cidx * 6, idx = bit >> 3, sh = bit & 7;
      uint32_t x = r[idx];
      if (idx + 1 < pitch) x |= (uint32_t)r[idx + 1] << 8;
      v = (int)((x >> sh) & 0x3F) - 32;
    }
    s += v;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[warp] = s;
}

}  // namespace ocrvl

// ---------------------------------------------------------------------------
// Host state
// ---------------------------------------------------------------------------
struct ocrvl_model {
  int device = 0;
  ocrvl_model_desc desc{};
  int qtype = 0;
  bool finalized = false;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::vector<void *> allocs;
  // weights
  float *embed = nullptr, *final_norm = nullptr;
  DMat lm_head{};
  std::vector<LayerW> layers;
  LayerW *layers_d = nullptr;
  std::vector<uint32_t> have;  // bitmask of loaded tensors per layer (+ globals at index L)
  // rope
  float *rope_cos = nullptr, *rope_sin = nullptr;
  int *sec_axis = nullptr;
  // kv
  float *kv_pool = nullptr;
  long long page_floats = 0;
  int num_pages = 0;
  std::vector<int> free_pages;
  // work
  Ctx ctx{};
  StepParams *sp_h = nullptr, *sp_d = nullptr;
  int *out_h = nullptr;  // [kMaxSeqs tokens][err]
  int *bt_stage = nullptr;
  int grid = 0;
  size_t smem = 0;
  unsigned bar_base = 0;  // value of the barrier counter before the next launch
  int sms = 0;
  // device-fed decode loop: id history and pinned staging for block-table
  // updates, grown on demand and kept (no allocation in the steady state)
  int *hist_d = nullptr;
  size_t hist_cap = 0;
  int *pin_pages = nullptr;
  size_t pin_cap = 0;
  // batched step (Q4 / Q6, more than kMaxBatch sequences): weight tensor maps
  // and the activation image
  bool batched = false;
  BatchedW bw{};
  // sampling: per-sequence fastRNG states (device + pinned staging) and the
  // full-vocabulary cumulative-sum scratch (allocated on first use)
  unsigned long long *rng_d = nullptr, *rng_h = nullptr;
  float *samp_work = nullptr;

  template <typename T>
  T *dalloc(size_t n) {
    void *p = nullptr;
    if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
    allocs.push_back(p);
    return (T *)p;
  }
};

struct ocrvl_seq {
  ocrvl_model *m = nullptr;
  int max_tokens = 0, len = 0;
  std::vector<int> pages;
  int *bt_d = nullptr;
};

namespace {

enum {
  T_LN1 = 0, T_LN2, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_NLAYER,
  G_EMBED = 0, G_NORM, G_LM, G_N
};

int set_device(ocrvl_model *m) {
  CK(cudaSetDevice(m->device));
  return OCRVL_OK;
}

bool parse_layer(const std::string &name, int &layer, std::string &suffix) {
  const std::string pre = "model.layers.";
  if (name.compare(0, pre.size(), pre) != 0) return false;
  size_t dot = name.find('.', pre.size());
  if (dot == std::string::npos) return false;
  std::string num = name.substr(pre.size(), dot - pre.size());
  if (num.empty() || num.size() > 6) return false;
  for (char ch : num)
    if (ch < '0' || ch > '9') return false;
  layer = std::atoi(num.c_str());
  suffix = name.substr(dot + 1);
  return true;
}

int upload_matrix(ocrvl_model *m, DMat &dst, int type, int64_t rows, int64_t cols, const float *scales,
                  const void *data, int row_offset, int total_rows) {
  int pb = packed_row_bytes(type, (int)cols);
  if (!dst.w) {
    uint8_t *w = m->dalloc<uint8_t>((size_t)total_rows * pb);
    float *s = m->dalloc<float>((size_t)total_rows);
    int32_t *rs = m->dalloc<int32_t>((size_t)total_rows);
    if (!w || !s || !rs) return fail(OCRVL_E_NOMEM, "cudaMalloc failed for weights");
    dst.w = w;
    dst.scale = s;
    dst.rowsum = rs;
    dst.rows = total_rows;
    dst.cols = (int)cols;
    dst.pitch = pb;
  }
  CK(cudaMemcpy((void *)(dst.w + (size_t)row_offset * pb), data, (size_t)rows * pb, cudaMemcpyHostToDevice));
  CK(cudaMemcpy((void *)(dst.scale + row_offset), scales, (size_t)rows * 4, cudaMemcpyHostToDevice));
  k_rowsum<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, m->stream>>>(
      type, dst.w + (size_t)row_offset * pb, (int)rows, (int)cols, pb, (int32_t *)dst.rowsum + row_offset);
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(m->stream));
  return OCRVL_OK;
}

int upload_f32(ocrvl_model *m, float *&dst, int64_t n, const void *data) {
  if (!dst) dst = m->dalloc<float>((size_t)n);
  if (!dst) return fail(OCRVL_E_NOMEM, "cudaMalloc failed");
  CK(cudaMemcpy(dst, data, (size_t)n * 4, cudaMemcpyHostToDevice));
  return OCRVL_OK;
}

size_t smem_bytes(const ocrvl_model_desc &d, int qtype) {
  int nmax = std::max(std::max(d.hidden_size, d.intermediate_size), d.num_heads * d.head_dim);
  size_t g1 = gemv_smem_total(qtype, 1, nmax, kStagesM1);
  size_t gb = gemv_smem_total(qtype, kMaxBatch, nmax, kStagesMB);
  size_t attn = std::max(attn_smem_floats() * 4, ax_smem_bytes_multi());
  size_t bgemm = qtype == QT_Q8 ? 0 : gemm_b_smem_bytes();
  return std::max(std::max(std::max(g1, gb), attn), bgemm) + 64 + kSmemAlignSlack;
}

typedef CUresult (*PfnEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D TMA map of a packed weight matrix: rows of `pitch` bytes; box =
// gemm_u K tiles of packed bytes x gemm_nt(rows, grid) rows (rows and
// columns past the end read 0).
bool make_weight_map(PfnEncodeTiled enc, const DMat &A, int qtype, int grid, TmapBytes *out) {
  const int KP = qtype == QT_Q4 ? kKT / 2 : kKT * 3 / 4;
  const int nt = gemm_nt(A.rows, grid);
  cuuint64_t dims[2] = {(cuuint64_t)A.pitch, (cuuint64_t)A.rows};
  cuuint64_t strides[1] = {(cuuint64_t)A.pitch};
  cuuint32_t box[2] = {(cuuint32_t)(gemm_u(qtype, nt) * KP), (cuuint32_t)nt};
  cuuint32_t es[2] = {1, 1};
  memset(out, 0, sizeof(*out));
  return enc((CUtensorMap *)out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)A.w, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D TMA map of the KV pool for the attention value phase: rows of head_dim
// floats (every (page, layer, kv head, K|V, position) is one row), boxes of
// 64 floats x 16 rows (half a head's dims over one page).
int make_kv_map(ocrvl_model *m) {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return fail(OCRVL_E_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old for the attention path)");
  }
  PfnEncodeTiled enc = (PfnEncodeTiled)fn;
  const ocrvl_model_desc &d = m->desc;
  const long long rows = (long long)m->num_pages * d.num_layers * d.num_kv_heads * 2 * kPageTokens;
  if (rows >= (1ll << 31)) return fail(OCRVL_E_INVALID, "kv_pool_bytes too large for the attention map");
  cuuint64_t dims[2] = {(cuuint64_t)d.head_dim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)d.head_dim * 4};
  cuuint32_t box[2] = {64, (cuuint32_t)kPageTokens};
  cuuint32_t es[2] = {1, 1};
  TmapBytes map;
  memset(&map, 0, sizeof(map));
  if (enc((CUtensorMap *)&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)m->kv_pool, dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return fail(OCRVL_E_CUDA, "cuTensorMapEncodeTiled failed for the KV pool");
  TmapBytes *dmap = m->dalloc<TmapBytes>(1);
  if (!dmap) return fail(OCRVL_E_NOMEM, "KV map");
  CK(cudaMemcpy(dmap, &map, sizeof(map), cudaMemcpyHostToDevice));
  m->ctx.kv_map = dmap;
  return OCRVL_OK;
}

// Sets up the batched step for Q4 / Q6 models: weight maps, activation image,
// kernel attributes.  Leaves m->batched false (steps of more than kMaxBatch
// sequences then run as groups) when any part is unavailable.
template <int QT>
void setup_batched(ocrvl_model *m) {
  static_assert(sizeof(TmapBytes) == sizeof(CUtensorMap), "tensor map size");
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return;
  }
  PfnEncodeTiled enc = (PfnEncodeTiled)fn;
  // the quantisation phases hold each thread's inputs in registers
  const ocrvl_model_desc &dd = m->desc;
  if (!xs_prologue_fits(PRO_RMSNORM, dd.hidden_size) ||
      !xs_prologue_fits(PRO_PLAIN, std::max(dd.num_heads * dd.head_dim, dd.intermediate_size)))
    return;
  const int L = m->desc.num_layers;
  std::vector<TmapBytes> maps((size_t)L * 5 + 1);
  for (int l = 0; l < L; l++) {
    const LayerW &w = m->layers[l];
    const DMat *mats[5] = {&w.qkv, &w.o, &w.gate, &w.up, &w.down};
    // the o and down projections' maps: N tiles of their split-K slabs
    for (int i = 0; i < 5; i++)
      if (!make_weight_map(enc, *mats[i], QT, i == 1 || i == 4 ? m->grid / down_splits(mats[i]->cols) : m->grid,
                           &maps[(size_t)l * 5 + i]))
        return;
  }
  if (!make_weight_map(enc, m->lm_head, QT, m->grid, &maps[(size_t)L * 5])) return;
  TmapBytes *dmaps = m->dalloc<TmapBytes>(maps.size());
  const int kcols = (m->ctx.pro_cols + kKT - 1) / kKT * kKT;
  uint8_t *act = m->dalloc<uint8_t>((size_t)kMmaM * kcols);
  float *act_sx = m->dalloc<float>(kMaxSeqs);
  int32_t *part = m->dalloc<int32_t>((size_t)kDownSplits * kMmaM * m->desc.hidden_size);
  if (!dmaps || !act || !act_sx || !part) return;
  if (cudaMemcpy(dmaps, maps.data(), maps.size() * sizeof(TmapBytes), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(act, 0, (size_t)kMmaM * kcols) != cudaSuccess ||
      cudaFuncSetAttribute(k_step_b<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step_b<QT>, kThreads, m->smem) != cudaSuccess ||
      per_sm * m->sms < m->grid) {
    cudaGetLastError();
    return;
  }
  m->bw.tm = dmaps;
  m->bw.act = act;
  m->bw.act_sx = act_sx;
  m->bw.part = part;
  m->bw.smem_avail = (int)(m->smem - kSmemAlignSlack);
  m->batched = true;
}

template <int QT>
int launch_step_q(ocrvl_model *m, int M, int any_logits, int do_embed, int feed, int nsteps = 1) {
  Ctx c = m->ctx;
  unsigned base = m->bar_base;
  void *args[] = {&c, &M, &any_logits, &do_embed, &feed, &base, &nsteps};
  CK(cudaLaunchCooperativeKernel((void *)k_step<QT>, dim3(m->grid), dim3(kThreads), args, m->smem, m->stream));
  // each step's barriers, and one between consecutive steps
  m->bar_base += ((unsigned)nsteps * barriers_per_step(m->desc.num_layers, any_logits) + (unsigned)(nsteps - 1)) *
                 (unsigned)m->grid;
  return OCRVL_OK;
}

template <int QT>
int launch_step_b(ocrvl_model *m, int any_logits, int do_embed, int feed) {
  Ctx c = m->ctx;
  BatchedW bw = m->bw;
  unsigned base = m->bar_base;
  void *args[] = {&c, &bw, &any_logits, &do_embed, &feed, &base};
  CK(cudaLaunchCooperativeKernel((void *)k_step_b<QT>, dim3(m->grid), dim3(kThreads), args, m->smem, m->stream));
  m->bar_base += barriers_per_step_b(m->desc.num_layers, any_logits) * (unsigned)m->grid;
  return OCRVL_OK;
}

int launch_step(ocrvl_model *m, int M, int any_logits, int do_embed, int feed = 0) {
  if (M > kMaxBatch) {
    if (!m->batched) return fail(OCRVL_E_INVALID, "batched step needs Q4 or Q6 weights");
    if (m->qtype == QT_Q4) return launch_step_b<QT_Q4>(m, any_logits, do_embed, feed);
    return launch_step_b<QT_Q6>(m, any_logits, do_embed, feed);
  }
  if (m->qtype == QT_Q4) return launch_step_q<QT_Q4>(m, M, any_logits, do_embed, feed);
  if (m->qtype == QT_Q6) return launch_step_q<QT_Q6>(m, M, any_logits, do_embed, feed);
  return launch_step_q<QT_Q8>(m, M, any_logits, do_embed, feed);
}

template <int QT>
int set_kernel_attrs(ocrvl_model *m) {
  CK(cudaFuncSetAttribute(k_step<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem));
  int per_sm = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step<QT>, kThreads, m->smem));
  if (per_sm <= 0) return fail(OCRVL_E_CUDA, "step kernel does not fit on an SM");
  m->grid = m->sms;  // one block per SM (the kernel holds ~200 KB of shared memory)
  return OCRVL_OK;
}

// Clears the barrier counter and error word after a timed-out step.
void reset_after_timeout(ocrvl_model *m) {
  int zero = 0;
  cudaMemcpy(m->ctx.err, &zero, 4, cudaMemcpyHostToDevice);
  cudaMemset(m->ctx.bar_count, 0, 4);
  cudaMemset(m->ctx.lm_count, 0, 4);
  cudaMemset(m->ctx.argkey, 0, kMaxSeqs * 8);
  m->bar_base = 0;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char *ocrvl_last_error(void) { return g_err.c_str(); }

int ocrvl_device_count(void) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return fail(OCRVL_E_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  return n;
}

int ocrvl_init(int device, const ocrvl_model_desc *desc, ocrvl_model **out) {
  if (!desc || !out) return fail(OCRVL_E_INVALID, "null argument");
  const ocrvl_model_desc &d = *desc;
  if (d.num_layers <= 0 || d.hidden_size <= 0 || d.vocab_size <= 0 || d.num_heads <= 0 || d.num_kv_heads <= 0 ||
      d.intermediate_size <= 0)
    return fail(OCRVL_E_INVALID, "model dimensions must be positive");
  if (d.head_dim != kHeadDim) return fail(OCRVL_E_INVALID, "head_dim must be 128");
  if (d.num_heads % d.num_kv_heads != 0 || d.num_heads / d.num_kv_heads > 8)
    return fail(OCRVL_E_INVALID, "num_heads must be 1..8 x num_kv_heads");
  if (d.num_kv_heads > 16) return fail(OCRVL_E_INVALID, "num_kv_heads must be at most 16");
  int qrows = d.num_heads * d.head_dim;
  if (d.hidden_size % 128 || d.intermediate_size % 128 || qrows % 128)
    return fail(OCRVL_E_INVALID, "hidden, intermediate and heads*head_dim must be multiples of 128");
  // The fused AddRMSNorm sums split hidden_size rows over 8 workers; the
  // reference's vector finalize needs each chunk < 16 rows or a multiple of 16.
  int chunk = (d.hidden_size + kFusedWorkers - 1) / kFusedWorkers;
  if (chunk >= 16 && chunk % 16) return fail(OCRVL_E_INVALID, "hidden_size/8 must be a multiple of 16");
  int secsum = d.mrope_section[0] + d.mrope_section[1] + d.mrope_section[2];
  if (secsum <= 0) return fail(OCRVL_E_INVALID, "mrope_section must be positive");
  ocrvl_model *m = new ocrvl_model();
  m->device = device;
  m->desc = d;
  if (m->desc.max_position <= 0) m->desc.max_position = 32768;
  if (m->desc.kv_pool_bytes <= 0) m->desc.kv_pool_bytes = 4ll << 30;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete m;
    return fail(OCRVL_E_CUDA, std::string("device init: ") + cudaGetErrorString(e));
  }
  m->layers.assign(d.num_layers, LayerW{});
  m->have.assign(d.num_layers + 1, 0);
  *out = m;
  return OCRVL_OK;
}

int ocrvl_load_tensor(ocrvl_model *m, const char *cname, int type, int64_t rows, int64_t cols,
                      const float *scales, const void *data) {
  if (!m || !cname || !data) return fail(OCRVL_E_INVALID, "null argument");
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->finalized) return fail(OCRVL_E_INVALID, "model already finalized");
  if (int rc = set_device(m)) return rc;
  const ocrvl_model_desc &d = m->desc;
  std::string name(cname);
  int H = d.hidden_size, I = d.intermediate_size, qr = d.num_heads * d.head_dim, kvr = d.num_kv_heads * d.head_dim;
  auto want_q = [&](int64_t r, int64_t c) -> int {
    if (type != OCRVL_Q8_ROW && type != OCRVL_Q4_ROW && type != OCRVL_Q6_ROW)
      return fail(OCRVL_E_INVALID, name + ": expected a row-quantized tensor (1000/1001/1002)");
    if (!scales) return fail(OCRVL_E_INVALID, name + ": missing scales");
    if (rows != r || cols != c) return fail(OCRVL_E_INVALID, name + ": unexpected shape");
    if (m->qtype == 0) m->qtype = type;
    if (m->qtype != type) return fail(OCRVL_E_INVALID, name + ": mixed quantization types");
    return OCRVL_OK;
  };
  auto want_f32 = [&](int64_t n) -> int {
    if (type != OCRVL_F32) return fail(OCRVL_E_INVALID, name + ": expected F32");
    if (rows * std::max<int64_t>(cols, 1) != n) return fail(OCRVL_E_INVALID, name + ": unexpected shape");
    return OCRVL_OK;
  };
  int rc;
  if (name == "model.embed_tokens.weight") {
    if ((rc = want_f32((int64_t)d.vocab_size * H))) return rc;
    if ((rc = upload_f32(m, m->embed, (int64_t)d.vocab_size * H, data))) return rc;
    m->have[d.num_layers] |= 1u << G_EMBED;
    return OCRVL_OK;
  }
  if (name == "model.norm.weight") {
    if ((rc = want_f32(H))) return rc;
    if ((rc = upload_f32(m, m->final_norm, H, data))) return rc;
    m->have[d.num_layers] |= 1u << G_NORM;
    return OCRVL_OK;
  }
  if (name == "lm_head.weight") {
    if ((rc = want_q(d.vocab_size, H))) return rc;
    if ((rc = upload_matrix(m, m->lm_head, type, rows, cols, scales, data, 0, (int)rows))) return rc;
    m->have[d.num_layers] |= 1u << G_LM;
    return OCRVL_OK;
  }
  int layer;
  std::string suf;
  if (!parse_layer(name, layer, suf) || layer >= d.num_layers) return OCRVL_OK;  // not a decoder tensor
  LayerW &L = m->layers[layer];
  uint32_t &have = m->have[layer];
  float *tmp = nullptr;
  if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight") {
    if ((rc = want_f32(H))) return rc;
    bool first = suf[0] == 'i';
    tmp = first ? (float *)L.ln1 : (float *)L.ln2;
    if ((rc = upload_f32(m, tmp, H, data))) return rc;
    if (first) { L.ln1 = tmp; have |= 1u << T_LN1; } else { L.ln2 = tmp; have |= 1u << T_LN2; }
    return OCRVL_OK;
  }
  struct Slot { const char *s; int bit; int rows, cols, off, total; DMat *dst; };
  Slot slots[] = {
      {"self_attn.q_proj.weight", T_Q, qr, H, 0, qr + 2 * kvr, &L.qkv},
      {"self_attn.k_proj.weight", T_K, kvr, H, qr, qr + 2 * kvr, &L.qkv},
      {"self_attn.v_proj.weight", T_V, kvr, H, qr + kvr, qr + 2 * kvr, &L.qkv},
      {"self_attn.o_proj.weight", T_O, H, qr, 0, H, &L.o},
      {"mlp.gate_proj.weight", T_GATE, I, H, 0, I, &L.gate},
      {"mlp.up_proj.weight", T_UP, I, H, 0, I, &L.up},
      {"mlp.down_proj.weight", T_DOWN, H, I, 0, H, &L.down},
  };
  for (auto &s : slots) {
    if (suf != s.s) continue;
    if ((rc = want_q(s.rows, s.cols))) return rc;
    if ((rc = upload_matrix(m, *s.dst, type, rows, cols, scales, data, s.off, s.total))) return rc;
    have |= 1u << s.bit;
    return OCRVL_OK;
  }
  return OCRVL_OK;
}

int ocrvl_finalize(ocrvl_model *m) {
  if (!m) return fail(OCRVL_E_INVALID, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->finalized) return OCRVL_OK;
  if (int rc = set_device(m)) return rc;
  const ocrvl_model_desc &d = m->desc;
  if (m->have[d.num_layers] != (1u << G_N) - 1) return fail(OCRVL_E_INVALID, "missing embed/norm/lm_head tensor");
  for (int l = 0; l < d.num_layers; l++)
    if (m->have[l] != (1u << T_NLAYER) - 1)
      return fail(OCRVL_E_INVALID, "missing tensor(s) of layer " + std::to_string(l));
  int half = d.head_dim / 2;
  // RoPE tables (initTextRoPE + buildMRoPETable, model.go:877-902, 7318-7357):
  // freq in float64, angle p*freq in float64, cos/sin rounded to f32.
  {
    std::vector<double> freq(half);
    std::vector<int> axis(half);
    int sec[3] = {d.mrope_section[0], d.mrope_section[1], d.mrope_section[2]};
    int end = sec[0], ax = 0;
    for (int i = 0; i < half; i++) {
      while (ax + 1 < 3 && i >= end) { ax++; end += sec[ax]; }
      axis[i] = std::min(ax, 2);
      freq[i] = std::pow(d.rope_theta, -(double)(2 * i) / (double)d.head_dim);
    }
    size_t n = (size_t)d.max_position * half;
    std::vector<float> cs(n), sn(n);
    for (int p = 0; p < d.max_position; p++)
      for (int i = 0; i < half; i++) {
        double ang = (double)p * freq[i];
        cs[(size_t)p * half + i] = (float)std::cos(ang);
        sn[(size_t)p * half + i] = (float)std::sin(ang);
      }
    m->rope_cos = m->dalloc<float>(n);
    m->rope_sin = m->dalloc<float>(n);
    m->sec_axis = m->dalloc<int>(half);
    if (!m->rope_cos || !m->rope_sin || !m->sec_axis) return fail(OCRVL_E_NOMEM, "rope tables");
    CK(cudaMemcpy(m->rope_cos, cs.data(), n * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->rope_sin, sn.data(), n * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->sec_axis, axis.data(), half * 4, cudaMemcpyHostToDevice));
  }
  // layers
  m->layers_d = m->dalloc<LayerW>(d.num_layers);
  if (!m->layers_d) return fail(OCRVL_E_NOMEM, "layers");
  CK(cudaMemcpy(m->layers_d, m->layers.data(), sizeof(LayerW) * d.num_layers, cudaMemcpyHostToDevice));
  // KV pool
  m->page_floats = (long long)d.num_layers * 2 * d.num_kv_heads * kPageTokens * d.head_dim;
  m->num_pages = (int)std::min<long long>(d.kv_pool_bytes / (m->page_floats * 4), 1 << 24);
  if (m->num_pages <= 0) return fail(OCRVL_E_INVALID, "kv_pool_bytes too small for one page");
  m->kv_pool = m->dalloc<float>((size_t)m->num_pages * m->page_floats);
  if (!m->kv_pool) return fail(OCRVL_E_NOMEM, "kv pool allocation failed");
  m->free_pages.resize(m->num_pages);
  for (int i = 0; i < m->num_pages; i++) m->free_pages[i] = m->num_pages - 1 - i;
  // work buffers
  Ctx &c = m->ctx;
  c.qtype = m->qtype;
  c.H = d.hidden_size;
  c.I = d.intermediate_size;
  c.L = d.num_layers;
  c.QH = d.num_heads;
  c.KVH = d.num_kv_heads;
  c.D = d.head_dim;
  c.V = d.vocab_size;
  c.eps = d.rms_norm_eps;
  c.attn_scale = (float)(1.0 / std::sqrt((double)d.head_dim));
  c.fzero = 0.0f;
  c.bar_spins = kBarrierSpins;
  c.embed = m->embed;
  c.final_norm = m->final_norm;
  c.layers = m->layers_d;
  c.lm_head = m->lm_head;
  c.rope_cos = m->rope_cos;
  c.rope_sin = m->rope_sin;
  c.rope_max = d.max_position;
  c.sec_axis = m->sec_axis;
  c.kv_pool = m->kv_pool;
  c.page_floats = m->page_floats;
  if (int rc = make_kv_map(m)) return rc;
  c.max_ctx = d.max_position;
  int qkvld = (c.QH + 2 * c.KVH) * c.D;
  size_t B = kMaxSeqs;
  c.h = m->dalloc<float>(B * c.H);
  c.vbuf = m->dalloc<float>(B * c.H);
  c.qkv = m->dalloc<float>(B * qkvld);
  c.head = m->dalloc<float>(B * c.QH * c.D);
  c.g = m->dalloc<float>(B * c.I);
  // long-cache attention scores: every position of a step's caches lies in a
  // page of the pool (the new position's page is taken before the step)
  // (rows padded to 4 floats: at most 3 more per (sequence, head))
  c.att_s = m->dalloc<float>(((size_t)m->num_pages * kPageTokens + 4 * kMaxSeqs) * c.QH);
  c.logits = m->dalloc<float>(B * (size_t)c.V);
  c.argkey = m->dalloc<unsigned long long>(B);
  c.tok_out = m->dalloc<int>(B + 1);
  c.bar_count = m->dalloc<unsigned>(2);
  c.lm_count = c.bar_count + 1;
  c.hist_pos = m->dalloc<int>(1);
  if (!c.hist_pos) return fail(OCRVL_E_NOMEM, "history counter");
  StepParams *spd = m->dalloc<StepParams>(1);
  if (!c.h || !c.vbuf || !c.qkv || !c.head || !c.g || !c.att_s || !c.logits || !c.argkey ||
      !c.tok_out || !c.bar_count || !spd)
    return fail(OCRVL_E_NOMEM, "work buffer allocation failed");
  c.err = c.tok_out + B;
  c.sp = spd;
  c.sp_w = spd;
  m->sp_d = spd;
  c.pro_cols = std::max(std::max(d.hidden_size, d.intermediate_size), d.num_heads * d.head_dim);
  CK(cudaMemset(c.argkey, 0, B * 8));
  CK(cudaMemset(c.tok_out, 0, (B + 1) * 4));
  CK(cudaMemset(c.bar_count, 0, 2 * 4));
  CK(cudaHostAlloc((void **)&m->sp_h, sizeof(StepParams), cudaHostAllocDefault));
  CK(cudaHostAlloc((void **)&m->out_h, (B + 1) * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc((void **)&m->bt_stage, B * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc((void **)&m->rng_h, B * 8, cudaHostAllocDefault));
  m->rng_d = m->dalloc<unsigned long long>(B);
  if (!m->rng_d) return fail(OCRVL_E_NOMEM, "sampler state");
  // launch geometry
  m->smem = smem_bytes(d, m->qtype);
  c.dyn_smem = (int)(m->smem - kSmemAlignSlack - 64);
  CK(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, m->device));
  {
    int rc = m->qtype == QT_Q4 ? set_kernel_attrs<QT_Q4>(m)
             : m->qtype == QT_Q6 ? set_kernel_attrs<QT_Q6>(m) : set_kernel_attrs<QT_Q8>(m);
    if (rc) return rc;
  }
  if (m->qtype == QT_Q4) setup_batched<QT_Q4>(m);
  if (m->qtype == QT_Q6) setup_batched<QT_Q6>(m);
  if (getenv("OCRVL_TRACE")) {
    c.trace = m->dalloc<unsigned long long>(kTraceWords);
    if (!c.trace) return fail(OCRVL_E_NOMEM, "trace buffer");
    CK(cudaMemset(c.trace, 0, kTraceWords * 8));
  }
  CK(cudaStreamSynchronize(m->stream));
  m->finalized = true;
  return OCRVL_OK;
}

int ocrvl_quant_type(const ocrvl_model *m) { return m ? m->qtype : OCRVL_E_INVALID; }

int ocrvl_trace_read(ocrvl_model *m, uint64_t *out, int cap) {
  if (!m || !out) return fail(OCRVL_E_INVALID, "null argument");
  if (!m->ctx.trace) return 0;
  std::lock_guard<std::mutex> lk(m->mu);
  if (int rc = set_device(m)) return rc;
  int n = std::min(cap, kTraceWords);
  CK(cudaStreamSynchronize(m->stream));
  CK(cudaMemcpy(out, m->ctx.trace, (size_t)n * 8, cudaMemcpyDeviceToHost));
  CK(cudaMemset(m->ctx.trace, 0, kTraceWords * 8));
  return n;
}

int ocrvl_set_wait_limit(ocrvl_model *m, int64_t barrier_polls) {
  if (!m || barrier_polls < 0) return fail(OCRVL_E_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->finalized) return fail(OCRVL_E_INVALID, "model not finalized");
  m->ctx.bar_spins = barrier_polls == 0 ? kBarrierSpins : (unsigned long long)barrier_polls;
  return OCRVL_OK;
}

int ocrvl_debug_read(ocrvl_model *m, int which, float *out, int64_t count) {
  if (!m || !out || count < 0) return fail(OCRVL_E_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->finalized) return fail(OCRVL_E_INVALID, "model not finalized");
  if (int rc = set_device(m)) return rc;
  const Ctx &c = m->ctx;
  const float *src = nullptr;
  int64_t n = 0;
  switch (which) {
    case 0: src = c.h; n = (int64_t)kMaxSeqs * c.H; break;
    case 1: src = c.vbuf; n = (int64_t)kMaxSeqs * c.H; break;
    case 2: src = c.qkv; n = (int64_t)kMaxSeqs * (c.QH + 2 * c.KVH) * c.D; break;
    case 3: src = c.head; n = (int64_t)kMaxSeqs * c.QH * c.D; break;
    case 4: src = c.g; n = (int64_t)kMaxSeqs * c.I; break;
    case 5: src = c.att_s; n = ((int64_t)m->num_pages * kPageTokens + 4 * kMaxSeqs) * c.QH; break;
    default: return fail(OCRVL_E_INVALID, "which must be 0..5");
  }
  n = std::min(n, count);
  CK(cudaStreamSynchronize(m->stream));
  CK(cudaMemcpy(out, src, (size_t)n * 4, cudaMemcpyDeviceToHost));
  return (int)n;
}

void ocrvl_free(ocrvl_model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (void *p : m->allocs) cudaFree(p);
  if (m->sp_h) cudaFreeHost(m->sp_h);
  if (m->out_h) cudaFreeHost(m->out_h);
  if (m->bt_stage) cudaFreeHost(m->bt_stage);
  if (m->rng_h) cudaFreeHost(m->rng_h);
  if (m->hist_d) cudaFree(m->hist_d);
  if (m->pin_pages) cudaFreeHost(m->pin_pages);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int ocrvl_seq_create(ocrvl_model *m, int max_tokens, ocrvl_seq **out) {
  if (!m || !out || max_tokens <= 0) return fail(OCRVL_E_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->finalized) return fail(OCRVL_E_INVALID, "model not finalized");
  if (max_tokens > m->desc.max_position) return fail(OCRVL_E_INVALID, "max_tokens exceeds max_position");
  if (int rc = set_device(m)) return rc;
  ocrvl_seq *s = new ocrvl_seq();
  s->m = m;
  s->max_tokens = max_tokens;
  int np = (max_tokens + kPageTokens - 1) / kPageTokens;
  if (cudaMalloc(&s->bt_d, (size_t)np * 4) != cudaSuccess) {
    delete s;
    return fail(OCRVL_E_NOMEM, "block table allocation failed");
  }
  cudaMemset(s->bt_d, 0, (size_t)np * 4);
  *out = s;
  return OCRVL_OK;
}

int ocrvl_seq_reset(ocrvl_seq *s) {
  if (!s) return fail(OCRVL_E_INVALID, "null seq");
  std::lock_guard<std::mutex> lk(s->m->mu);
  for (int p : s->pages) s->m->free_pages.push_back(p);
  s->pages.clear();
  s->len = 0;
  return OCRVL_OK;
}

void ocrvl_seq_free(ocrvl_seq *s) {
  if (!s) return;
  ocrvl_seq_reset(s);
  cudaSetDevice(s->m->device);
  cudaFree(s->bt_d);
  delete s;
}

int ocrvl_seq_len(const ocrvl_seq *s) { return s ? s->len : OCRVL_E_INVALID; }

int ocrvl_seq_import_kv(ocrvl_seq *s, int n, const float *k, const float *v) {
  if (!s) return fail(OCRVL_E_INVALID, "null seq");
  if (n < 0 || n > s->max_tokens) return fail(OCRVL_E_INVALID, "n outside 0..max_tokens");
  if (n > 0 && (!k || !v)) return fail(OCRVL_E_INVALID, "null K/V");
  if (int rc = ocrvl_seq_reset(s)) return rc;
  ocrvl_model *m = s->m;
  std::lock_guard<std::mutex> lk(m->mu);
  const ocrvl_model_desc &d = m->desc;
  const int np = (n + kPageTokens - 1) / kPageTokens;
  if ((size_t)np > m->free_pages.size()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
  if (int rc = set_device(m)) return rc;
  CK(cudaStreamSynchronize(m->stream));
  const int kvd = d.num_kv_heads * d.head_dim;
  // one page at a time in the pool layout [layer][kv head][K, V][16][head_dim]
  std::vector<float> page((size_t)m->page_floats);
  std::vector<int> ids(np);
  for (int p = 0; p < np; p++) {
    ids[p] = m->free_pages.back();
    m->free_pages.pop_back();
    s->pages.push_back(ids[p]);
    std::fill(page.begin(), page.end(), 0.0f);
    for (int l = 0; l < d.num_layers; l++)
      for (int g = 0; g < d.num_kv_heads; g++)
        for (int kind = 0; kind < 2; kind++)
          for (int r = 0; r < kPageTokens && p * kPageTokens + r < n; r++) {
            const float *src = (kind ? v : k) + ((size_t)l * n + (size_t)p * kPageTokens + r) * kvd + (size_t)g * d.head_dim;
            float *dst = page.data() + ((((size_t)l * d.num_kv_heads + g) * 2 + kind) * kPageTokens + r) * d.head_dim;
            std::copy(src, src + d.head_dim, dst);
          }
    cudaError_t e = cudaMemcpy(m->kv_pool + (size_t)ids[p] * m->page_floats, page.data(), page.size() * 4,
                               cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      for (int q : s->pages) m->free_pages.push_back(q);
      s->pages.clear();
      return fail(OCRVL_E_CUDA, std::string("cudaMemcpy: ") + cudaGetErrorString(e));
    }
  }
  if (np > 0) {
    cudaError_t e = cudaMemcpy(s->bt_d, ids.data(), (size_t)np * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      for (int q : s->pages) m->free_pages.push_back(q);
      s->pages.clear();
      return fail(OCRVL_E_CUDA, std::string("cudaMemcpy: ") + cudaGetErrorString(e));
    }
  }
  s->len = n;
  return OCRVL_OK;
}

int ocrvl_seq_fill_synthetic(ocrvl_seq *s, int n, uint64_t seed) {
  if (!s) return fail(OCRVL_E_INVALID, "null seq");
  if (n < 0 || n > s->max_tokens) return fail(OCRVL_E_INVALID, "n outside 0..max_tokens");
  if (int rc = ocrvl_seq_reset(s)) return rc;
  ocrvl_model *m = s->m;
  std::lock_guard<std::mutex> lk(m->mu);
  const ocrvl_model_desc &d = m->desc;
  const int np = (n + kPageTokens - 1) / kPageTokens;
  if ((size_t)np > m->free_pages.size()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
  if (int rc = set_device(m)) return rc;
  if (np == 0) {
    s->len = 0;
    return OCRVL_OK;
  }
  CK(cudaStreamSynchronize(m->stream));  // the pinned staging may feed an earlier copy
  std::vector<int> ids(np);
  for (int p = 0; p < np; p++) {
    ids[p] = m->free_pages.back();
    m->free_pages.pop_back();
    s->pages.push_back(ids[p]);
  }
  auto undo = [&](cudaError_t e) {
    for (int q : s->pages) m->free_pages.push_back(q);
    s->pages.clear();
    return fail(OCRVL_E_CUDA, std::string("fill: ") + cudaGetErrorString(e));
  };
  cudaError_t e = cudaMemcpy(s->bt_d, ids.data(), (size_t)np * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return undo(e);
  const long long total4 = m->page_floats / 4 * np;
  const int blocks = (int)std::min<long long>((total4 + 255) / 256, (long long)m->sms * 16);
  k_fill_kv<<<blocks, 256, 0, m->stream>>>(m->kv_pool, m->page_floats, s->bt_d, np, n, d.num_layers, d.num_kv_heads,
                                           d.head_dim, (unsigned long long)seed);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return undo(e);
  s->len = n;
  return OCRVL_OK;
}

int ocrvl_seq_read_kv(ocrvl_seq *s, int layer, float *k, float *v) {
  if (!s || !k || !v) return fail(OCRVL_E_INVALID, "null argument");
  ocrvl_model *m = s->m;
  std::lock_guard<std::mutex> lk(m->mu);
  const ocrvl_model_desc &d = m->desc;
  if (layer < 0 || layer >= d.num_layers) return fail(OCRVL_E_INVALID, "layer out of range");
  if (int rc = set_device(m)) return rc;
  CK(cudaStreamSynchronize(m->stream));
  int kvd = d.num_kv_heads * d.head_dim;
  for (int t = 0; t < s->len; t++) {
    int page = s->pages[t / kPageTokens];
    for (int kind = 0; kind < 2; kind++)
      for (int g = 0; g < d.num_kv_heads; g++) {
        size_t off = (size_t)page * m->page_floats +
                     ((((size_t)layer * d.num_kv_heads + g) * 2 + kind) * kPageTokens + t % kPageTokens) * d.head_dim;
        float *dst = (kind == 0 ? k : v) + (size_t)t * kvd + (size_t)g * d.head_dim;
        CK(cudaMemcpy(dst, m->kv_pool + off, d.head_dim * 4, cudaMemcpyDeviceToHost));
      }
  }
  return s->len;
}

}  // extern "C"

namespace {

// The generation loop's choice of sampler for GenerateOptions
// (internal/model/model.go:1536-1544, 1854-1868, 3611-3642, 7202-7205).
struct SamplePlan {
  int mode = SAMPLE_ARGMAX, k = 0, temp1 = 0;
  float inv = 1.0f;
};

int plan_sampling(double temperature, int top_k, int vocab, SamplePlan *p) {
  if (std::isnan(temperature) || std::isinf(temperature)) return fail(OCRVL_E_INVALID, "temperature must be finite");
  if (top_k < 0) return fail(OCRVL_E_INVALID, "top_k must be >= 0");
  *p = SamplePlan{};
  if (temperature <= 0 || top_k == 1) return OCRVL_OK;
  if (top_k > 1 && top_k < vocab) {
    if (top_k > kSampleMaxTopK) return fail(OCRVL_E_INVALID, "top_k above 4096 is not supported by the device sampler");
    p->mode = SAMPLE_TOPK;
    p->k = top_k;
    p->temp1 = temperature == 1.0 ? 1 : 0;
    p->inv = (float)(1.0 / temperature);
    return OCRVL_OK;
  }
  // expScaledVecFMA leaves the last vocab % 16 weights unset, so the full
  // path is restated for whole 16-float blocks only
  if (vocab < 16 || vocab % 16 != 0)
    return fail(OCRVL_E_INVALID, "full-vocabulary sampling needs vocab_size to be a multiple of 16");
  if (vocab > kFullMaxVocab)
    return fail(OCRVL_E_INVALID, "full-vocabulary sampling supports vocab_size up to 262144");
  p->mode = SAMPLE_FULL;
  const float t = (float)temperature;
  p->inv = t == 1.0f ? 1.0f : 1.0f / t;
  return OCRVL_OK;
}

int launch_sample(const SamplePlan &p, int rows, int vocab, const float *logits, long long ld,
                  unsigned long long *rng, int *out, int *cand_ids, float *cand_scores, float *work,
                  cudaStream_t stream) {
  SampleArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.V = vocab;
  a.mode = p.mode;
  a.k = p.k;
  a.temp1 = p.temp1;
  a.inv = p.inv;
  a.rng = rng;
  a.out = out;
  a.cand_ids = cand_ids;
  a.cand_scores = cand_scores;
  a.work = work;
  const size_t smem = p.mode == SAMPLE_TOPK ? sample_smem_topk(p.k) : p.mode == SAMPLE_FULL ? sample_smem_full(vocab) : 0;
  if (smem > 48 * 1024) {
    // more than the default dynamic shared memory: opt in once per device
    static std::atomic<unsigned long long> opted{0};
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(OCRVL_E_INVALID, "device index out of range");
    if (!(opted.load() & (1ull << dev))) {
      CK(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sample_smem_max()));
      opted.fetch_or(1ull << dev);
    }
  }
  k_sample<<<rows, kSampleThreads, smem, stream>>>(a);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

// One launch of the step kernel for n <= kMaxBatch sequences that ocrvl_step
// has validated (model lock held): page allocation, parameter upload,
// launch, results.
int step_group(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
               const int32_t *pos_thw, int need_logits, int32_t *out_ids, float *out_logits,
               const SamplePlan *smp = nullptr, uint64_t *rng_state = nullptr) {
  const ocrvl_model_desc &d = m->desc;
  const bool draw = need_logits && smp && smp->mode != SAMPLE_ARGMAX;
  StepParams &sp = *m->sp_h;
  sp.M = n;
  sp.any_logits = need_logits ? 1 : 0;
  sp.store_logits = need_logits && (out_logits || draw) ? 1 : 0;
  int max_n = 0;
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    int p[3] = {s->len, s->len, s->len};
    if (pos_thw)
      for (int a = 0; a < 3; a++) p[a] = pos_thw[3 * i + a];
    sp.seq[i].tok = ids ? ids[i] : 0;
    sp.seq[i].len = s->len;
    for (int a = 0; a < 3; a++) sp.seq[i].pos[a] = p[a];
    sp.seq[i].need = need_logits ? 1 : 0;
    sp.seq[i].bt = s->bt_d;
    max_n = std::max(max_n, s->len + 1);
  }
  sp.max_n = max_n;
  // pages for the positions appended this step
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    if (s->len % kPageTokens == 0 && (int)s->pages.size() <= s->len / kPageTokens) {
      if (m->free_pages.empty()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
      int pg = m->free_pages.back();
      m->free_pages.pop_back();
      s->pages.push_back(pg);
      m->bt_stage[i] = pg;
      CK(cudaMemcpyAsync(s->bt_d + s->len / kPageTokens, &m->bt_stage[i], 4, cudaMemcpyHostToDevice, m->stream));
    }
  }
  CK(cudaMemcpyAsync(m->sp_d, &sp, step_params_bytes(n), cudaMemcpyHostToDevice, m->stream));
  if (embeds) CK(cudaMemcpyAsync(m->ctx.h, embeds, (size_t)n * d.hidden_size * 4, cudaMemcpyHostToDevice, m->stream));
  if (draw) {
    memcpy(m->rng_h, rng_state, (size_t)n * 8);
    CK(cudaMemcpyAsync(m->rng_d, m->rng_h, (size_t)n * 8, cudaMemcpyHostToDevice, m->stream));
  }
  if (int rc = launch_step(m, n, sp.any_logits, embeds ? 0 : 1)) return rc;
  if (draw) {
    // the draw replaces the greedy ids in tok_out (same stream, after the step)
    if (int rc = launch_sample(*smp, n, d.vocab_size, m->ctx.logits, d.vocab_size, m->rng_d, m->ctx.tok_out, nullptr,
                               nullptr, m->samp_work, m->stream))
      return rc;
    CK(cudaMemcpyAsync(m->rng_h, m->rng_d, (size_t)n * 8, cudaMemcpyDeviceToHost, m->stream));
  }
  CK(cudaMemcpyAsync(m->out_h, m->ctx.tok_out, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaMemcpyAsync(m->out_h + kMaxSeqs, m->ctx.err, 4, cudaMemcpyDeviceToHost, m->stream));
  if (out_logits && need_logits)
    CK(cudaMemcpyAsync(out_logits, m->ctx.logits, (size_t)n * d.vocab_size * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if (m->out_h[kMaxSeqs]) {
    reset_after_timeout(m);
    return fail(OCRVL_E_TIMEOUT, "device grid barrier timed out");
  }
  if (draw) {
    for (int i = 0; i < n; i++)
      if (m->out_h[i] < 0) return fail(OCRVL_E_CUDA, "device sampler: internal failure (candidate count or bounded wait)");
    memcpy(rng_state, m->rng_h, (size_t)n * 8);
  }
  for (int i = 0; i < n; i++) {
    seqs[i]->len++;
    if (out_ids) out_ids[i] = need_logits ? m->out_h[i] : -1;
  }
  return OCRVL_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// ocrvl_step / ocrvl_step_sample: validation of every sequence, then one
// step_group per launch.
int step_impl(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
              const int32_t *pos_thw, int need_logits, int32_t *out_ids, float *out_logits, const SamplePlan *smp,
              uint64_t *rng_state) {
  if (!m || !seqs) return fail(OCRVL_E_INVALID, "null argument");
  if (n < 1 || n > kMaxSeqs) return fail(OCRVL_E_INVALID, "batch must be 1..64 sequences");
  if (!ids && !embeds) return fail(OCRVL_E_INVALID, "ids or embeds required");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->finalized) return fail(OCRVL_E_INVALID, "model not finalized");
  if (int rc = set_device(m)) return rc;
  const ocrvl_model_desc &d = m->desc;
  // validate every sequence before any state changes
  size_t new_pages = 0;
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    if (!s || s->m != m) return fail(OCRVL_E_INVALID, "sequence belongs to another model");
    for (int j = 0; j < i; j++)
      if (seqs[j] == s) return fail(OCRVL_E_INVALID, "sequence repeated in one step");
    if (s->len >= s->max_tokens) return fail(OCRVL_E_INVALID, "sequence is full (max_tokens reached)");
    if (ids && (ids[i] < 0 || ids[i] >= d.vocab_size))
      return fail(OCRVL_E_INVALID, "token id " + std::to_string(ids ? ids[i] : 0) + " outside vocab");
    if (pos_thw)
      for (int a = 0; a < 3; a++)
        if (pos_thw[3 * i + a] < 0 || pos_thw[3 * i + a] >= d.max_position)
          return fail(OCRVL_E_INVALID, "position outside RoPE table");
    if (!pos_thw && s->len >= d.max_position) return fail(OCRVL_E_INVALID, "position outside RoPE table");
    if (s->len % kPageTokens == 0 && (int)s->pages.size() <= s->len / kPageTokens) new_pages++;
  }
  if (new_pages > m->free_pages.size()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
  if (smp && smp->mode == SAMPLE_FULL && !m->samp_work) {
    m->samp_work = m->dalloc<float>((size_t)kMaxSeqs * d.vocab_size);
    if (!m->samp_work) return fail(OCRVL_E_NOMEM, "sampler scratch");
  }
  if (n > kMaxBatch && m->batched)
    return step_group(m, seqs, n, ids, embeds, pos_thw, need_logits, out_ids, out_logits, smp, rng_state);
  // groups of kMaxBatch sequences, one launch each
  for (int g0 = 0; g0 < n; g0 += kMaxBatch) {
    const int gn = std::min(kMaxBatch, n - g0);
    int rc = step_group(m, seqs + g0, gn, ids ? ids + g0 : nullptr, embeds ? embeds + (size_t)g0 * d.hidden_size : nullptr,
                        pos_thw ? pos_thw + 3 * g0 : nullptr, need_logits, out_ids ? out_ids + g0 : nullptr,
                        out_logits ? out_logits + (size_t)g0 * d.vocab_size : nullptr, smp,
                        rng_state ? rng_state + g0 : nullptr);
    if (rc) return rc;
  }
  return OCRVL_OK;
}

}  // namespace

extern "C" {

int ocrvl_step(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
               const int32_t *pos_thw, int need_logits, int32_t *out_ids, float *out_logits) {
  return step_impl(m, seqs, n, ids, embeds, pos_thw, need_logits, out_ids, out_logits, nullptr, nullptr);
}

int ocrvl_step_sample(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
                      const int32_t *pos_thw, double temperature, int top_k, uint64_t *rng_state, int32_t *out_ids) {
  if (!m || !out_ids) return fail(OCRVL_E_INVALID, "null argument");
  SamplePlan p;
  if (int rc = plan_sampling(temperature, top_k, m->desc.vocab_size, &p)) return rc;
  if (p.mode != SAMPLE_ARGMAX && !rng_state) return fail(OCRVL_E_INVALID, "rng_state required when sampling");
  return step_impl(m, seqs, n, ids, embeds, pos_thw, 1, out_ids, nullptr, &p, rng_state);
}

void *ocrvl_model_stream(ocrvl_model *m) { return m ? (void *)m->stream : nullptr; }

int ocrvl_step_io_bytes(const ocrvl_model *m, int n, int64_t *h2d, int64_t *d2h) {
  if (!m || !h2d || !d2h || n < 1 || n > kMaxSeqs) return fail(OCRVL_E_INVALID, "bad arguments");
  const int groups = m->batched ? 1 : (n + kMaxBatch - 1) / kMaxBatch;
  *h2d = groups == 1 ? (int64_t)step_params_bytes(n)
                     : (int64_t)(step_params_bytes(kMaxBatch) * (groups - 1) + step_params_bytes(n - (groups - 1) * kMaxBatch));
  *d2h = (int64_t)n * 4 + 4 * groups;  // ids + error word per launch
  return OCRVL_OK;
}

}  // extern "C"

namespace {

// The device-fed loop for n <= kMaxBatch sequences (model lock held).
int decode_group(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *first_ids, int steps,
                 int32_t *out_ids) {
  const ocrvl_model_desc &d = m->desc;
  StepParams &sp = *m->sp_h;
  sp.M = n;
  sp.store_logits = 0;
  sp.any_logits = 1;
  int max_n = 0;
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    if (!s || s->m != m) return fail(OCRVL_E_INVALID, "sequence belongs to another model");
    for (int j = 0; j < i; j++)
      if (seqs[j] == s) return fail(OCRVL_E_INVALID, "sequence repeated in one step");
    if (s->len + steps > s->max_tokens) return fail(OCRVL_E_INVALID, "steps exceed the sequence's max_tokens");
    if (s->len + steps > d.max_position) return fail(OCRVL_E_INVALID, "positions exceed the RoPE table");
    if (first_ids[i] < 0 || first_ids[i] >= d.vocab_size) return fail(OCRVL_E_INVALID, "token id outside vocab");
    sp.seq[i].tok = first_ids[i];
    sp.seq[i].len = s->len;
    sp.seq[i].pos[0] = sp.seq[i].pos[1] = sp.seq[i].pos[2] = s->len;
    sp.seq[i].need = 1;
    sp.seq[i].bt = s->bt_d;
    max_n = std::max(max_n, s->len + 1);
  }
  sp.max_n = max_n;
  // buffers sized for this call (grown once, then reused): the id history and
  // pinned staging for the new block-table entries
  size_t new_pages = 0;
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    int need_pages = (s->len + steps + kPageTokens - 1) / kPageTokens;
    new_pages += (size_t)std::max(0, need_pages - (int)s->pages.size());
  }
  if (new_pages > m->free_pages.size()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
  if ((size_t)steps * n > m->hist_cap) {
    CK(cudaStreamSynchronize(m->stream));
    if (m->hist_d) cudaFree(m->hist_d);
    m->hist_d = nullptr;
    m->hist_cap = 0;
    size_t cap = std::max<size_t>((size_t)steps * n, 4096);
    if (cudaMalloc(&m->hist_d, cap * 4) != cudaSuccess) return fail(OCRVL_E_NOMEM, "id history allocation failed");
    m->hist_cap = cap;
  }
  if (new_pages > m->pin_cap) {
    CK(cudaStreamSynchronize(m->stream));
    if (m->pin_pages) cudaFreeHost(m->pin_pages);
    m->pin_pages = nullptr;
    m->pin_cap = 0;
    size_t cap = std::max<size_t>(new_pages, 1024);
    CK(cudaHostAlloc((void **)&m->pin_pages, cap * 4, cudaHostAllocDefault));
    m->pin_cap = cap;
  } else if (new_pages) {
    CK(cudaStreamSynchronize(m->stream));  // the staging buffer may still feed an earlier copy
  }
  // every page the loop will touch is allocated up front
  size_t off = 0;
  for (int i = 0; i < n; i++) {
    ocrvl_seq *s = seqs[i];
    int need_pages = (s->len + steps + kPageTokens - 1) / kPageTokens;
    int first_new = (int)s->pages.size();
    while ((int)s->pages.size() < need_pages) {
      int pg = m->free_pages.back();
      m->free_pages.pop_back();
      s->pages.push_back(pg);
      m->pin_pages[off + s->pages.size() - 1 - first_new] = pg;
    }
    if (need_pages > first_new) {
      CK(cudaMemcpyAsync(s->bt_d + first_new, m->pin_pages + off, (size_t)(need_pages - first_new) * 4,
                         cudaMemcpyHostToDevice, m->stream));
      off += (size_t)(need_pages - first_new);
    }
  }
  int *hist = m->hist_d;
  m->ctx.hist = hist;
  CK(cudaMemsetAsync(m->ctx.hist_pos, 0, 4, m->stream));
  CK(cudaMemcpyAsync(m->sp_d, &sp, step_params_bytes(n), cudaMemcpyHostToDevice, m->stream));
  int rc = OCRVL_OK;
  if (n <= kMaxBatch) {
    // every step in one persistent launch (the token feedback stays on the
    // device; no launch between steps)
    rc = m->qtype == QT_Q4   ? launch_step_q<QT_Q4>(m, n, 1, 1, 1, steps)
         : m->qtype == QT_Q6 ? launch_step_q<QT_Q6>(m, n, 1, 1, 1, steps)
                             : launch_step_q<QT_Q8>(m, n, 1, 1, 1, steps);
  } else {
    for (int st = 0; st < steps && rc == OCRVL_OK; st++) rc = launch_step(m, n, 1, 1, 1);
  }
  m->ctx.hist = nullptr;
  if (rc == OCRVL_OK) {
    cudaError_t e1 = cudaMemcpyAsync(out_ids, hist, (size_t)steps * n * 4, cudaMemcpyDeviceToHost, m->stream);
    cudaError_t e2 = cudaMemcpyAsync(m->out_h + kMaxSeqs, m->ctx.err, 4, cudaMemcpyDeviceToHost, m->stream);
    if (e1 != cudaSuccess || e2 != cudaSuccess) rc = fail(OCRVL_E_CUDA, "copy of decoded ids failed");
  }
  CK(cudaStreamSynchronize(m->stream));
  if (rc) return rc;
  if (m->out_h[kMaxSeqs]) {
    reset_after_timeout(m);
    return fail(OCRVL_E_TIMEOUT, "device grid barrier timed out");
  }
  for (int i = 0; i < n; i++) seqs[i]->len += steps;
  return OCRVL_OK;
}

}  // namespace

extern "C" {

int ocrvl_decode_greedy_device(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *first_ids, int steps,
                               int32_t *out_ids) {
  if (!m || !seqs || !first_ids || !out_ids) return fail(OCRVL_E_INVALID, "null argument");
  if (n < 1 || n > kMaxSeqs || steps < 1) return fail(OCRVL_E_INVALID, "batch must be 1..64, steps >= 1");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->finalized) return fail(OCRVL_E_INVALID, "model not finalized");
  if (int rc = set_device(m)) return rc;
  if (n <= kMaxBatch || m->batched) return decode_group(m, seqs, n, first_ids, steps, out_ids);
  // groups of kMaxBatch sequences run one after another; pages for all of
  // them are checked first so that no group starts when a later one cannot
  size_t new_pages = 0;
  for (int i = 0; i < n; i++) {
    const ocrvl_seq *s = seqs[i];
    if (!s || s->m != m) return fail(OCRVL_E_INVALID, "sequence belongs to another model");
    for (int j = 0; j < i; j++)
      if (seqs[j] == s) return fail(OCRVL_E_INVALID, "sequence repeated in one step");
    int need_pages = (s->len + steps + kPageTokens - 1) / kPageTokens;
    new_pages += (size_t)std::max(0, need_pages - (int)s->pages.size());
  }
  if (new_pages > m->free_pages.size()) return fail(OCRVL_E_NOMEM, "KV page pool exhausted");
  std::vector<int32_t> part((size_t)steps * kMaxBatch);
  for (int g0 = 0; g0 < n; g0 += kMaxBatch) {
    const int gn = std::min(kMaxBatch, n - g0);
    if (int rc = decode_group(m, seqs + g0, gn, first_ids + g0, steps, part.data())) return rc;
    for (int st = 0; st < steps; st++)
      for (int i = 0; i < gn; i++) out_ids[(size_t)st * n + g0 + i] = part[(size_t)st * gn + i];
  }
  return OCRVL_OK;
}

int ocrvl_generate_greedy(ocrvl_model *m, const int32_t *ids, int n_ids, int max_new, const int32_t *eos,
                          int n_eos, int32_t *out, int out_cap, int *n_out) {
  if (!m || !out || !n_out || (n_ids > 0 && !ids)) return fail(OCRVL_E_INVALID, "null argument");
  if (max_new < 0) return fail(OCRVL_E_INVALID, "max_new_tokens must be >= 0");
  for (int i = 0; i < n_ids; i++)
    if (ids[i] < 0) return fail(OCRVL_E_INVALID, "input tokens must not contain negative ids");
  if (max_new > 0 && n_ids == 0) return fail(OCRVL_E_INVALID, "input tokens must not be empty when max_new_tokens > 0");
  if (out_cap < n_ids + max_new) return fail(OCRVL_E_INVALID, "output buffer too small");
  static const int32_t kDefaultEOS[1] = {2};
  if (!eos) { eos = kDefaultEOS; n_eos = 1; }
  for (int i = 0; i < n_ids; i++) out[i] = ids[i];
  *n_out = n_ids;
  if (max_new == 0) return OCRVL_OK;
  ocrvl_seq *s = nullptr;
  int rc = ocrvl_seq_create(m, n_ids + max_new, &s);
  if (rc) return rc;
  int32_t tok = -1;
  for (int p = 0; p < n_ids && rc == 0; p++) rc = ocrvl_step(m, &s, 1, &ids[p], nullptr, nullptr, p == n_ids - 1, &tok, nullptr);
  int n = n_ids;
  for (int i = 0; rc == 0 && i < max_new; i++) {
    out[n++] = tok;
    bool stop = false;
    for (int j = 0; j < n_eos; j++) stop |= tok == eos[j];
    if (stop || i + 1 >= max_new) break;
    int32_t cur = tok;
    rc = ocrvl_step(m, &s, 1, &cur, nullptr, nullptr, 1, &tok, nullptr);
  }
  ocrvl_seq_free(s);
  *n_out = n;
  return rc;
}

int ocrvl_generate(ocrvl_model *m, const int32_t *ids, int n_ids, int max_new, const int32_t *eos, int n_eos,
                   double temperature, int top_k, int64_t seed, int32_t *out, int out_cap, int *n_out) {
  if (!m || !out || !n_out || (n_ids > 0 && !ids)) return fail(OCRVL_E_INVALID, "null argument");
  SamplePlan p;
  if (int rc = plan_sampling(temperature, top_k, m->desc.vocab_size, &p)) return rc;
  if (p.mode == SAMPLE_ARGMAX) return ocrvl_generate_greedy(m, ids, n_ids, max_new, eos, n_eos, out, out_cap, n_out);
  if (max_new < 0) return fail(OCRVL_E_INVALID, "max_new_tokens must be >= 0");
  for (int i = 0; i < n_ids; i++)
    if (ids[i] < 0) return fail(OCRVL_E_INVALID, "input tokens must not contain negative ids");
  if (max_new > 0 && n_ids == 0) return fail(OCRVL_E_INVALID, "input tokens must not be empty when max_new_tokens > 0");
  if (out_cap < n_ids + max_new) return fail(OCRVL_E_INVALID, "output buffer too small");
  static const int32_t kDefaultEOS[1] = {2};
  if (!eos) { eos = kDefaultEOS; n_eos = 1; }
  for (int i = 0; i < n_ids; i++) out[i] = ids[i];
  *n_out = n_ids;
  if (max_new == 0) return OCRVL_OK;
  ocrvl_seq *s = nullptr;
  int rc = ocrvl_seq_create(m, n_ids + max_new, &s);
  if (rc) return rc;
  uint64_t rng = (uint64_t)seed;  // samplingRNGInto (model.go:1846-1852)
  int32_t tok = -1;
  for (int q = 0; q + 1 < n_ids && rc == 0; q++) rc = ocrvl_step(m, &s, 1, &ids[q], nullptr, nullptr, 0, &tok, nullptr);
  if (rc == 0) rc = ocrvl_step_sample(m, &s, 1, &ids[n_ids - 1], nullptr, nullptr, temperature, top_k, &rng, &tok);
  int n = n_ids;
  for (int i = 0; rc == 0 && i < max_new; i++) {
    out[n++] = tok;
    bool stop = false;
    for (int j = 0; j < n_eos; j++) stop |= tok == eos[j];
    if (stop || i + 1 >= max_new) break;
    int32_t cur = tok;
    rc = ocrvl_step_sample(m, &s, 1, &cur, nullptr, nullptr, temperature, top_k, &rng, &tok);
  }
  ocrvl_seq_free(s);
  *n_out = n;
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// GGUF file loading (gguf.Open, internal/gguf/gguf.go:111-251, and the row
// loaders 313-569): header parsed here, tensor bytes handed to
// ocrvl_load_tensor straight from a read-only mapping of the file.
// ---------------------------------------------------------------------------
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace {

struct Reader {
  const uint8_t *p;
  size_t n, pos = 0;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (pos + sizeof(T) > n) { ok = false; return v; }
    memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t len = get<uint64_t>();
    if (!ok || len > (16u << 20) || pos + len > n) { ok = false; return ""; }
    std::string s((const char *)p + pos, len);
    pos += len;
    return s;
  }
};

}  // namespace

extern "C" int ocrvl_load_gguf(ocrvl_model *m, const char *path) {
  if (!m || !path) return fail(OCRVL_E_INVALID, "null argument");
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(OCRVL_E_INVALID, std::string("cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return fail(OCRVL_E_INVALID, "bad GGUF file");
  }
  size_t size = (size_t)st.st_size;
  void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return fail(OCRVL_E_INVALID, "mmap failed");
  struct Unmap { void *p; size_t n; ~Unmap() { munmap(p, n); } } um{map, size};
  Reader r{(const uint8_t *)map, size};
  uint32_t magic = r.get<uint32_t>();
  if (magic != 0x46554747u) return fail(OCRVL_E_INVALID, "bad GGUF magic");
  if (r.get<uint32_t>() != 3u) return fail(OCRVL_E_INVALID, "unsupported GGUF version");
  uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
  if (nt > (1u << 20) || nkv > (1u << 20)) return fail(OCRVL_E_INVALID, "GGUF counts too large");
  for (uint64_t i = 0; i < nkv && r.ok; i++) {
    r.str();
    uint32_t t = r.get<uint32_t>();
    if (t == 4) r.get<uint32_t>();
    else if (t == 10) r.get<uint64_t>();
    else if (t == 8) r.str();
    else return fail(OCRVL_E_INVALID, "unsupported GGUF metadata type");
  }
  struct TI { std::string name; std::vector<uint64_t> shape; uint32_t type; uint64_t off; };
  std::vector<TI> infos;
  for (uint64_t i = 0; i < nt && r.ok; i++) {
    TI t;
    t.name = r.str();
    uint32_t nd = r.get<uint32_t>();
    if (nd > 8) return fail(OCRVL_E_INVALID, "GGUF tensor has too many dimensions");
    for (uint32_t j = 0; j < nd; j++) t.shape.push_back(r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    t.off = r.get<uint64_t>();
    infos.push_back(t);
  }
  if (!r.ok) return fail(OCRVL_E_INVALID, "truncated GGUF header");
  size_t data_start = (r.pos + 31) / 32 * 32;
  for (auto &t : infos) {
    int64_t rows = t.shape.empty() ? 1 : (int64_t)t.shape[0];
    int64_t cols = t.shape.size() >= 2 ? (int64_t)t.shape[1] : 1;
    size_t bytes;
    if (t.type == OCRVL_F32) {
      bytes = 4;
      for (auto dsz : t.shape) bytes *= dsz;
    } else {
      int pb = packed_row_bytes((int)t.type, (int)cols);
      if (pb < 0 || t.shape.size() != 2) return fail(OCRVL_E_INVALID, "unsupported GGUF tensor " + t.name);
      bytes = (size_t)rows * (4 + pb);
    }
    if (data_start + t.off + bytes > size) return fail(OCRVL_E_INVALID, "GGUF tensor " + t.name + " exceeds file size");
    const uint8_t *base = (const uint8_t *)map + data_start + t.off;
    int rc;
    if (t.type == OCRVL_F32)
      rc = ocrvl_load_tensor(m, t.name.c_str(), 0, rows, t.shape.size() >= 2 ? cols : 1, nullptr, base);
    else
      rc = ocrvl_load_tensor(m, t.name.c_str(), (int)t.type, rows, cols, (const float *)base, base + rows * 4);
    if (rc) return rc;
  }
  return OCRVL_OK;
}

// ---------------------------------------------------------------------------
// Op-level entry points (device pointers)
// ---------------------------------------------------------------------------
namespace {

Ctx op_ctx(int type, float eps) {
  Ctx c;
  memset(&c, 0, sizeof(c));
  c.qtype = type;
  c.eps = eps;
  return c;
}

DMat op_mat(int type, int rows, int cols, const void *w, const float *scale, const int32_t *rowsum) {
  DMat a;
  a.w = (const uint8_t *)w;
  a.scale = scale;
  a.rowsum = rowsum;
  a.rows = rows;
  a.cols = cols;
  a.pitch = packed_row_bytes(type, cols);
  return a;
}

int op_check(int type, int rows, int cols, int m) {
  if (type != OCRVL_Q8_ROW && type != OCRVL_Q4_ROW && type != OCRVL_Q6_ROW)
    return fail(OCRVL_E_INVALID, "type must be 1000, 1001 or 1002");
  if (rows <= 0 || cols <= 0 || cols % 128) return fail(OCRVL_E_INVALID, "cols must be a positive multiple of 128");
  if (m < 1 || m > kMaxBatch) return fail(OCRVL_E_INVALID, "m must be 1..8");
  return OCRVL_OK;
}

int op_grid(int rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return std::max(1, std::min(sms * 2, (rows + 7) / 8));
}

template <int QT>
int op_gemv_q(const Ctx &c, const GemvArgs &a, int m, cudaStream_t st) {
  // the batched form (m > 1) keeps kMaxBatch input vectors in shared memory
  size_t smem = (m > 1 ? gemv_smem_total(QT, kMaxBatch, a.A.cols, kStagesMB)
                       : gemv_smem_total(QT, 1, a.A.cols, kStagesM1)) + 64 + kSmemAlignSlack;
  CK(cudaFuncSetAttribute(k_gemv<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_gemv<QT><<<op_grid(a.A.rows), kThreads, smem, st>>>(c, a, m);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

int op_gemv(const Ctx &c, const GemvArgs &a, int m, cudaStream_t st) {
  if (c.qtype == QT_Q4) return op_gemv_q<QT_Q4>(c, a, m, st);
  if (c.qtype == QT_Q6) return op_gemv_q<QT_Q6>(c, a, m, st);
  return op_gemv_q<QT_Q8>(c, a, m, st);
}

std::mutex g_scratch_mu;
unsigned long long *g_keys[64];

}  // namespace

extern "C" {

int ocrvl_op_rowsum(int type, int rows, int cols, const void *w, int32_t *rowsum, void *stream) {
  if (int rc = op_check(type, rows, cols, 1)) return rc;
  k_rowsum<<<(unsigned)(((int64_t)rows * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      type, (const uint8_t *)w, rows, cols, packed_row_bytes(type, cols), rowsum);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

int ocrvl_op_matvec(int type, int rows, int cols, const void *w, const float *scale, const int32_t *rowsum, int m,
                    const float *x, const float *norm_w, float eps, float *out, void *stream) {
  if (int rc = op_check(type, rows, cols, m)) return rc;
  Ctx c = op_ctx(type, eps);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.A = op_mat(type, rows, cols, w, scale, rowsum);
  a.row_end = rows;
  a.src = x;
  a.ld = cols;
  a.mode = norm_w ? PRO_RMSNORM : PRO_PLAIN;
  a.norm_w = norm_w;
  a.epi = EPI_STORE;
  a.out = out;
  a.ldo = rows;
  return op_gemv(c, a, m, (cudaStream_t)stream);
}

int ocrvl_op_matvec_add_rmsnorm(int type, int rows, int cols, const void *w, const float *scale,
                                const int32_t *rowsum, int m, const float *x, float *residual, int in_place,
                                const float *norm_w, float eps, float *v_out, float *norm_out, void *stream) {
  if (int rc = op_check(type, rows, cols, m)) return rc;
  int chunk = (rows + kFusedWorkers - 1) / kFusedWorkers;
  if (type != OCRVL_Q8_ROW && chunk >= 16 && chunk % 16)
    return fail(OCRVL_E_INVALID, "rows/8 must be < 16 or a multiple of 16");
  Ctx c = op_ctx(type, eps);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.A = op_mat(type, rows, cols, w, scale, rowsum);
  a.row_end = rows;
  a.src = x;
  a.ld = cols;
  a.mode = PRO_PLAIN;
  a.epi = EPI_RESID;
  a.ldo = rows;
  a.resid = residual;
  a.vout = v_out;
  a.resid_mode = RESID_MASK;
  a.in_place_mask = in_place ? 0xFF : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = op_gemv(c, a, m, st)) return rc;
  size_t smem = (320 + (size_t)rows) * 4 + 64;
  CK(cudaFuncSetAttribute(k_addnorm_out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_addnorm_out<<<m, kThreads, smem, st>>>(c, v_out, rows, m, norm_w, norm_out);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

int ocrvl_op_swiglu(int type, int rows, int cols, const void *wg, const float *sg, const int32_t *rsg,
                    const void *wu, const float *su, const int32_t *rsu, int m, const float *x, float *out,
                    void *stream) {
  if (int rc = op_check(type, rows, cols, m)) return rc;
  Ctx c = op_ctx(type, 0.0f);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.A = op_mat(type, rows, cols, wg, sg, rsg);
  a.B = op_mat(type, rows, cols, wu, su, rsu);
  a.row_end = rows;
  a.src = x;
  a.ld = cols;
  a.mode = PRO_PLAIN;
  a.epi = EPI_SWIGLU;
  a.out = out;
  a.ldo = rows;
  return op_gemv(c, a, m, (cudaStream_t)stream);
}

int ocrvl_op_argmax(int type, int rows, int cols, const void *w, const float *scale, const int32_t *rowsum, int m,
                    const float *x, int32_t *ids, void *stream) {
  if (int rc = op_check(type, rows, cols, m)) return rc;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(OCRVL_E_INVALID, "device index out of range");
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long *keys;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_keys[dev]) CK(cudaMalloc(&g_keys[dev], kMaxBatch * 8));
    keys = g_keys[dev];
  }
  CK(cudaMemsetAsync(keys, 0, kMaxBatch * 8, st));
  Ctx c = op_ctx(type, 0.0f);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.A = op_mat(type, rows, cols, w, scale, rowsum);
  a.row_end = rows;
  a.src = x;
  a.ld = cols;
  a.mode = PRO_PLAIN;
  a.epi = EPI_ARGMAX;
  a.ldo = rows;
  a.argkey = keys;
  if (int rc = op_gemv(c, a, m, st)) return rc;
  k_argmax_ids<<<1, 32, 0, st>>>(keys, m, ids);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

int ocrvl_op_rmsnorm(int n, int m, const float *x, const float *w, float eps, float *out, void *stream) {
  if (n <= 0 || n % 128 || m < 1) return fail(OCRVL_E_INVALID, "n must be a positive multiple of 128, m >= 1");
  Ctx c = op_ctx(OCRVL_Q8_ROW, eps);
  size_t smem = (320 + (size_t)n) * 4 + 64;
  CK(cudaFuncSetAttribute(k_rmsnorm_out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_rmsnorm_out<<<std::min(m, 1024), kThreads, smem, (cudaStream_t)stream>>>(c, x, n, m, w, out);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free argmax (ocrvl_op_argmax_noalloc)
//
// ocrvl_op_argmax keeps its per-vector argmax keys in device memory that it
// cudaMalloc's on first use.  Some callers must not allocate device memory at
// all: a server that reserves the GPU's memory for its own pools at start-up
// (a cudaMalloc from inside a request can then fail), or a latency-critical
// loop where cudaMalloc may synchronize the device and stall other streams.
// This variant keeps the keys in a fixed file-scope device array instead.
//
// Limit: kNoAllocArgmaxKeys keys (one 64-bit key per input vector, i.e. at
// most 8 vectors per call; 64 bytes that every GPU loading this library holds
// until the process exits).  The host obtains the array's device address with
// cudaGetSymbolAddress once per device, on the first call made with that
// device current; make that first call before any stream capture.  All calls
// share the one array: the keys are cleared at the start of every call, and
// calls whose kernels overlap on the GPU (different streams, or different
// host threads on one device) race on it and must be ordered by the caller.
// ---------------------------------------------------------------------------
namespace {

constexpr int kNoAllocArgmaxKeys = kMaxBatch;
static __device__ __align__(256) unsigned long long g_noalloc_argmax_keys[kNoAllocArgmaxKeys];

std::mutex g_noalloc_mu;
unsigned long long *g_noalloc_keys_dev[64];  // device address of the array, per device

}  // namespace

extern "C" {

int ocrvl_op_argmax_noalloc(int type, int rows, int cols, const void *w, const float *scale, const int32_t *rowsum,
                            int m, const float *x, int32_t *ids, void *stream) {
  if (m > kNoAllocArgmaxKeys)
    return fail(OCRVL_E_INVALID, "m = " + std::to_string(m) + " exceeds the " + std::to_string(kNoAllocArgmaxKeys) +
                                     " vectors the static argmax scratch holds");
  if (int rc = op_check(type, rows, cols, m)) return rc;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(OCRVL_E_INVALID, "device index out of range");
  unsigned long long *keys = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_keys_dev[dev]) {
      // the device address of the file-scope array on the current device (the
      // host-side name g_noalloc_argmax_keys is not a device pointer)
      void *p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_argmax_keys);
      if (e != cudaSuccess) return fail(OCRVL_E_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      g_noalloc_keys_dev[dev] = (unsigned long long *)p;
    }
    keys = g_noalloc_keys_dev[dev];
  }
  cudaStream_t st = (cudaStream_t)stream;
  // the array keeps the previous call's keys: clear the ones this call uses
  CK(cudaMemsetAsync(keys, 0, (size_t)m * sizeof(unsigned long long), st));
  Ctx c = op_ctx(type, 0.0f);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.A = op_mat(type, rows, cols, w, scale, rowsum);
  a.row_end = rows;
  a.src = x;
  a.ld = cols;
  a.mode = PRO_PLAIN;
  a.epi = EPI_ARGMAX;
  a.ldo = rows;
  a.argkey = keys;
  if (int rc = op_gemv(c, a, m, st)) return rc;
  k_argmax_ids<<<1, 32, 0, st>>>(keys, m, ids);
  CK(cudaGetLastError());
  return OCRVL_OK;
}

int ocrvl_op_sample(int m, int vocab, const float *logits, double temperature, int top_k, uint64_t *rng_state,
                    int32_t *out_ids, int32_t *cand_ids, float *cand_scores, float *work, void *stream) {
  if (m < 1 || m > 65535) return fail(OCRVL_E_INVALID, "m must be 1..65535 rows");
  if (vocab < 2) return fail(OCRVL_E_INVALID, "vocab must be >= 2");
  if (!logits || !out_ids) return fail(OCRVL_E_INVALID, "null argument");
  SamplePlan p;
  if (int rc = plan_sampling(temperature, top_k, vocab, &p)) return rc;
  if (p.mode != SAMPLE_ARGMAX && !rng_state) return fail(OCRVL_E_INVALID, "rng_state required when sampling");
  if (p.mode == SAMPLE_FULL && !work) return fail(OCRVL_E_INVALID, "work (m * vocab floats) required for full-vocabulary sampling");
  if (p.mode == SAMPLE_FULL && ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(work)) & 15))
    return fail(OCRVL_E_INVALID, "logits and work must be 16-byte aligned for full-vocabulary sampling");
  if (p.mode != SAMPLE_TOPK && (cand_ids || cand_scores))
    return fail(OCRVL_E_INVALID, "candidates are only produced by top-k sampling");
  return launch_sample(p, m, vocab, logits, vocab, (unsigned long long *)rng_state, out_ids, cand_ids, cand_scores,
                       work, (cudaStream_t)stream);
}

}  // extern "C"
