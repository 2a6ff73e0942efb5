// Attention over long caches (more than kAttnChunk positions) in the
// reference's exact arithmetic, as two phases separated by a grid barrier.
// Included by decoder.cuh after the KV, RoPE, mbarrier and stage-ring
// helpers.
//
// The reference (cacheAttentionScores, SoftmaxInPlace, weightedCacheValueSum;
// internal/model/model.go:4623-4795, 5201-5591, internal/tensor/ops.go:
// 1199-1363) computes, per query head h over the n cached positions:
//   s_t = dotF32(q_h, k_t) * 1/sqrt(D)      (16-slot order + tree16)
//   M   = max_t s_t
//   e_t = exp_fma(s_t - M) for t < nv = 16 floor(n / 16); the positions at or
//         above nv keep their raw score (expF32VecFMA leaves the tail,
//         internal/tensor/dot_amd64.s:6131-6168)
//   sum = tree16 of 16 lane chains, lane l adding e_l, e_{l+16}, ... in order
//   w_t = e_t * (1 / sum)                    (the tail: s_t * (1 / sum))
//   o   = w_0 v_0, then o = fma(w_t, v_t, o) for t = 1 .. n-1
// Both phases restate these steps in the same order, so the head outputs
// are bit-identical to the reference's.
//
// Phase 1 (scores).  The long caches' positions split into chunks of 32
// (two KV pages) per (sequence m, kv head g); the step's chunks, in (m, g,
// chunk) order, go to the blocks in contiguous ranges of equal count.  A
// block streams its chunks' K rows (one 8 KB bulk copy per page) through a
// ring of K buffers, the first ones issued before the phase, and writes the
// G scores of every position to the score scratch (c.att_s, per sequence
// [kv head][head][n rounded up to 4]).  Chunk descriptors (sequence, kv head,
// first position, pool pages) come from a per-launch table, and two chunks of
// one pair are scored per iteration (independent work for the warps between
// block barriers); refills are issued from two warps (one thread issues bulk
// copies at about 24 GB/s).  The chunk holding the new position scores it
// with the new key (rotated) and appends the new K and V rows to the cache.
//
// Phase 2 (softmax and values).  One item per (m, g, half of the head dims):
// warp h reads head h's scores, takes M, the lane chains and 1/sum (every
// item of a pair recomputes them: 8 n exponentials), then lane i of warp h
// runs the value chains of dims (64 half + 2 i, +1) over all n positions in
// order, with V rows staged through shared memory 32 positions at a time.
namespace ocrvl {

constexpr int kAxTok = 32;                            // positions per score chunk (two pages)
constexpr int kAxKBufs = 8;                           // K chunk buffers per block (M > 1)
constexpr int kAxKBufsM1 = 4;                         // K chunk buffers per block (M <= 1: GEMV ring slots)
constexpr int kAxKBytes = kAxTok * kHeadDim * 4;      // K rows of one chunk: 16 KB
constexpr int kAxVRing = 8;                           // value-step buffers in flight
constexpr int kAxVTok = 32;                           // positions per value step
constexpr int kAxVBytes = kAxVTok * (kHeadDim / 2) * 4;  // half-dim V rows of one step: 8 KB
constexpr int kAxVRingBytes = kAxVRing * kAxVBytes;
static_assert(2 * kAxKBytes == kStageBytes, "two K chunks per ring slot");
static_assert(kMaxGroup == 8 && kHeadDim == 128, "score layout: 8 heads x 2 tokens per half-warp");

__host__ __device__ __forceinline__ int ax_nbufs(int M) { return M <= 1 ? kAxKBufsM1 : kAxKBufs; }

// Small arrays of the score phase (floats from their base): rotated q by lane
// [half-warp grp][head][2][slot][4] (dims (16 (j ^ grp) + slot, +64)), the
// new key (rotated) and value, cos / sin of the sequence's position.
constexpr int kAxQs = 0;
constexpr int kAxKnew = kAxQs + 2 * 8 * 128;  // [128] rotated new k, [128] new v
constexpr int kAxCos = kAxKnew + 256;         // [64] cos, [64] sin
constexpr int kAxSmallFloats = kAxCos + 128;
static_assert(kAxSmallFloats * 4 <= kStageBytes, "small arrays fit one ring slot");

// Shared memory the attention phases need when M > 1 (their buffers start at
// the base of the dynamic shared memory; for M <= 1 the K buffers use ring
// slots kStagesM1-1 and kStagesM1-2 and the small arrays ring slot 0; the
// value phase uses the base of the shared memory for every M).
__host__ __device__ __forceinline__ size_t ax_smem_bytes_multi() {
  return (size_t)kAxKBufs * kAxKBytes + (size_t)kAxSmallFloats * 4;
}

__device__ __forceinline__ float *ax_kbuf(const Ctx &c, int M, float *smem, int j) {
  if (M <= 1)
    return (float *)((uint8_t *)smem + gemv_prologue_bytes(c.qtype, 1, c.pro_cols) +
                     (size_t)(kStagesM1 - 1 - j / 2) * kStageBytes + (size_t)(j & 1) * kAxKBytes);
  return (float *)((uint8_t *)smem + (size_t)j * kAxKBytes);
}
__device__ __forceinline__ float *ax_small(const Ctx &c, int M, float *smem) {
  if (M <= 1) return (float *)((uint8_t *)smem + gemv_prologue_bytes(c.qtype, 1, c.pro_cols));
  return (float *)((uint8_t *)smem + (size_t)kAxKBufs * kAxKBytes);
}
// Geometry of the step's caches, fixed for a launch and computed at its start
// (ax_launch_init): per sequence its positions n (0 for a cache of at most
// kAttnChunk positions, handled by the short path), the prefix of its chunks
// over (sequence, kv head) and of its scores; the long caches (longest
// first) and the short ones (in order); this block's chunk range.
__shared__ int s_ax_n[kMaxSeqs], s_ax_cb[kMaxSeqs + 1], s_ax_sb[kMaxSeqs];
__shared__ int s_ax_nl, s_ax_long[kMaxSeqs];
__shared__ int s_ax_hg;  // head groups per value item (the longest cache's scores of G / hg heads fit shared memory;
                         // more groups when there are few long caches)
__shared__ int s_ex_n, s_ex_m[kMaxSeqs];
__shared__ int s_ax_lo, s_ax_hi;
// Descriptors of the block's first kAxTabCap chunks: x = m | g << 8, y = first
// position, z / w = pool pages (w = -1 when the chunk has one page), so that
// neither a chunk's scoring nor its refill searches the chunk list.
constexpr int kAxTabCap = 256;
__shared__ int4 s_ax_tab[kAxTabCap];

// Per-block state of the K chunk loads, kept across the phases of a launch:
// s_ax_full[j] completes when buffer j's copies land, s_ax_par bit j is the
// parity of its next completion, s_ax_issued counts the chunks of the coming
// (or running) score phase issued so far (chunk lo + i into buffer i %
// nbufs).
__shared__ __align__(8) uint64_t s_ax_full[kAxKBufs];
__shared__ uint32_t s_ax_par;
__shared__ int s_ax_issued;

__device__ __forceinline__ void ax_block_init() {
  if (threadIdx.x == 0) {
    for (int j = 0; j < kAxKBufs; j++) mbar_init(&s_ax_full[j], 1);
    mbar_fence_init();
    s_ax_par = 0;
    s_ax_issued = 0;
  }
}

// Row stride of a head's scores: n rounded up to 4 floats, so every row starts
// on a 16-byte boundary (bulk and cp.async copies of whole rows).
__host__ __device__ __forceinline__ int ax_stride(int n) { return (n + 3) & ~3; }

__device__ __forceinline__ int ax_bound(int P, int b, int nb) { return (int)(((long long)P * b + nb - 1) / nb); }

// Chunk ci of the step: its sequence, kv head and first position.
struct AxChunk {
  int m, g, t0;
};
__device__ __forceinline__ AxChunk ax_chunk(const Ctx &c, const StepParams &sp, int ci) {
  int lo = 0, hi = sp.M - 1;  // last sequence with s_ax_cb <= ci
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_ax_cb[mid] <= ci) lo = mid;
    else hi = mid - 1;
  }
  const int nch = (s_ax_n[lo] + kAxTok - 1) / kAxTok;
  const int r = ci - s_ax_cb[lo];
  AxChunk k;
  k.m = lo;
  k.g = r / nch;
  k.t0 = (r - k.g * nch) * kAxTok;
  return k;
}

// All threads, once per launch (after the step parameters are in shared
// memory and ax_block_init).
__device__ void ax_launch_init(const Ctx &c) {
  const StepParams &sp = *c.sp;
  if (threadIdx.x == 0) {
    int cb = 0, sb = 0, ne = 0, nl = 0;
    for (int m = 0; m < sp.M; m++) {
      const int n = sp.seq[m].len + 1;
      const bool lng = n > kAttnChunk;
      s_ax_n[m] = lng ? n : 0;
      s_ax_cb[m] = cb;
      s_ax_sb[m] = sb;
      if (lng) {
        cb += c.KVH * ((n + kAxTok - 1) / kAxTok);
        sb += c.QH * ax_stride(n);
        s_ax_long[nl++] = m;
      } else {
        s_ex_m[ne++] = m;
      }
    }
    s_ax_cb[sp.M] = cb;
    s_ex_n = ne;
    s_ax_nl = nl;
    // value items go to the blocks longest cache first (stable insertion sort)
    for (int i = 1; i < nl; i++) {
      const int m = s_ax_long[i];
      int j = i - 1;
      while (j >= 0 && s_ax_n[s_ax_long[j]] < s_ax_n[m]) {
        s_ax_long[j + 1] = s_ax_long[j];
        j--;
      }
      s_ax_long[j + 1] = m;
    }
    s_ax_lo = ax_bound(cb, blockIdx.x, gridDim.x);
    s_ax_hi = ax_bound(cb, blockIdx.x + 1, gridDim.x);
    const int G = c.QH / c.KVH;
    int hg = 1;
    if (nl > 0)
      while (hg < G && (size_t)(G / hg) * ax_stride(s_ax_n[s_ax_long[0]]) * 4 + kAxVRingBytes > (size_t)c.dyn_smem)
        hg *= 2;
    // few long caches (single-sequence steps): more, smaller items (fewer
    // heads each) spread over the blocks
    while (hg < G && nl * c.KVH * 2 * hg * 2 <= (int)gridDim.x) hg *= 2;
    s_ax_hg = hg;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < s_ax_hi - s_ax_lo && i < kAxTabCap; i += kThreads) {
    const AxChunk k = ax_chunk(c, sp, s_ax_lo + i);
    const int *bt = sp.seq[k.m].bt;
    s_ax_tab[i] = make_int4(k.m | (k.g << 8), k.t0, __ldg(bt + k.t0 / kPageTokens),
                            k.t0 + kPageTokens < s_ax_n[k.m] ? __ldg(bt + k.t0 / kPageTokens + 1) : -1);
  }
}

// Descriptor of the block's chunk lo + i (from the table, or computed for the
// chunks past its end).
__device__ __forceinline__ int4 ax_desc(const Ctx &c, const StepParams &sp, int i) {
  if (i < kAxTabCap) return s_ax_tab[i];
  const AxChunk k = ax_chunk(c, sp, s_ax_lo + i);
  const int *bt = sp.seq[k.m].bt;
  return make_int4(k.m | (k.g << 8), k.t0, __ldg(bt + k.t0 / kPageTokens),
                   k.t0 + kPageTokens < s_ax_n[k.m] ? __ldg(bt + k.t0 / kPageTokens + 1) : -1);
}

// K rows of (layer, kv head g) in pool page `page`: 8 KB (the V rows follow).
__device__ __forceinline__ const float *ax_page_k(const Ctx &c, int page, int layer, int g) {
  return c.kv_pool + (size_t)page * c.page_floats + ((size_t)layer * c.KVH + g) * 2 * kPageTokens * c.D;
}

// One thread: the K copies of the block's chunk lo + i into buffer i % nbufs.
__device__ __forceinline__ void ax_issue(const Ctx &c, int layer, float *smem, int i) {
  const StepParams &sp = *c.sp;
  const int4 d = ax_desc(c, sp, i);
  const int g = d.x >> 8;
  constexpr uint32_t pb = kPageTokens * kHeadDim * 4;
  const int b = i % ax_nbufs(sp.M);
  float *buf = ax_kbuf(c, sp.M, smem, b);
  uint64_t *bar = &s_ax_full[b];
  mbar_expect_tx(bar, (d.w >= 0 ? 2u : 1u) * pb);
  bulk_g2s(buf, ax_page_k(c, d.z, layer, g), pb, bar);
  if (d.w >= 0) bulk_g2s(buf + kPageTokens * kHeadDim, ax_page_k(c, d.w, layer, g), pb, bar);
}

// One thread: issues the block's chunks while fewer than `upto` (at most
// nbufs) are in flight or done for the coming phase.
__device__ void ax_issue_upto(const Ctx &c, int layer, float *smem, int upto) {
  int i = s_ax_issued;
  const int nch = s_ax_hi - s_ax_lo;
  const int nb = ax_nbufs(c.sp->M);
  if (upto > nb) upto = nb;
  if (i >= upto || i >= nch) return;
  // the buffers were last written by ordinary stores (or read) in earlier
  // phases: order those before the async copies
  if (i == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  for (; i < upto && i < nch; i++) ax_issue(c, layer, smem, i);
  s_ax_issued = i;
}

// Waits for chunk copies issued ahead of a score phase that did not run
// (thread 0).
__device__ __forceinline__ void ax_drain(const Ctx &c) {
  for (int j = 0; j < s_ax_issued && j < ax_nbufs(c.sp->M); j++) {
    mbar_wait(&s_ax_full[j], (s_ax_par >> j) & 1u, c.err);
    s_ax_par ^= 1u << j;
  }
  s_ax_issued = 0;
}

// Per-block time stamp i (thread 0; the last layer's values remain).
__device__ __forceinline__ void rg_bmark(const Ctx &c, int i) {
  if (c.trace && threadIdx.x == 0) c.trace[4 * kTraceRows + kTraceMarks * blockIdx.x + i] = gtimer();
}

// Pairs of floats in one 64-bit register pair and the sm_100 packed FP32
// operations on them (each half rounded to nearest even, as the scalar
// __fmul_rn / __fadd_rn / __fmaf_rn).  A packed multiply whose result feeds a
// packed add is contracted into an FMA by ptxas (measured on B200 even with
// the explicit .rn), so no exact path uses that pair.
typedef unsigned long long f2x;
__device__ __forceinline__ f2x f2_pack(float a, float b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float f2_lo(f2x r) { return __uint_as_float((uint32_t)(r & 0xFFFFFFFFull)); }
__device__ __forceinline__ float f2_hi(f2x r) { return __uint_as_float((uint32_t)(r >> 32)); }
__device__ __forceinline__ f2x f2_mul(f2x a, f2x b) {
  f2x d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2x f2_add(f2x a, f2x b) {
  f2x d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2x f2_fma(f2x a, f2x b, f2x c) {
  f2x d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// All threads: rotated q of pair (m, g) into the lane layout, the new key
// (rotated) and value.
__device__ void ax_load_q(const Ctx &c, const StepParams &sp, int m, int g, float *sm) {
  const int G = c.QH / c.KVH;
  const size_t qkvld = (size_t)(c.QH + 2 * c.KVH) * kHeadDim;
  const float *row = c.qkv + (size_t)m * qkvld;
  float *qs = sm + kAxQs, *knew = sm + kAxKnew;
  const int *pos = sp.seq[m].pos;
  const bool has_rope = pos[0] != 0 || pos[1] != 0 || pos[2] != 0;
  const bool tab = s_rope_ready && m < kMaxBatch;  // the launch's RoPE tables hold sequence m
  float *cs = sm + kAxCos;
  if (!tab && threadIdx.x < kHeadDim) {
    const int i = threadIdx.x & 63;
    const int p = pos[c.sec_axis[i]];
    cs[threadIdx.x] = __ldg((threadIdx.x < 64 ? c.rope_cos : c.rope_sin) + (size_t)p * (kHeadDim / 2) + i);
  }
  __syncthreads();
  const float *rc = tab ? s_rope_cs[m] : cs, *rs = tab ? s_rope_sn[m] : cs + 64;
  for (int p = threadIdx.x; p < G * 16 + 48; p += kThreads) {
    if (p < G * 16) {
      const int hh = p >> 4, i4 = p & 15;
      const float *qh = row + (size_t)(g * G + hh) * kHeadDim;
      float4 a = __ldcg((const float4 *)qh + i4), b = __ldcg((const float4 *)(qh + 64) + i4);
      if (has_rope) rope4(a, b, rc + 4 * i4, rs + 4 * i4);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int d = 4 * i4 + e, jd = d >> 4, sd = d & 15;  // dims d and d + 64
#pragma unroll
        for (int gg = 0; gg < 2; gg++) {
          const int jp = jd ^ gg;
          *(float2 *)(qs + (((gg * 8 + hh) * 2 + (jp >> 1)) * 16 + sd) * 4 + (jp & 1) * 2) = make_float2(av[e], bv[e]);
        }
      }
    } else if (p < G * 16 + 16) {
      const int i4 = p - G * 16;
      const float *kn = row + (size_t)(c.QH + g) * kHeadDim;
      float4 a = __ldcg((const float4 *)kn + i4), b = __ldcg((const float4 *)(kn + 64) + i4);
      if (has_rope) rope4(a, b, rc + 4 * i4, rs + 4 * i4);
      ((float4 *)knew)[i4] = a;
      ((float4 *)knew)[i4 + 16] = b;
    } else {
      const int i4 = p - G * 16 - 16;
      ((float4 *)(knew + 128))[i4] = __ldcg((const float4 *)(row + (size_t)(c.QH + c.KVH + g) * kHeadDim) + i4);
    }
  }
  __syncthreads();
}

// Scores of the warp's tokens 4 warp .. 4 warp + 3 of NC chunks of one pair
// (K rows in Kb[k], first positions t0[k]; the new position len takes the
// rotated key knew): half grp takes tokens 4 warp + 2 grp + {0, 1}; lane slot
// s multiplies dims s + 16 j (j = 0..7) and sums them as
// ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)) (packed in pairs (p_j, p_j+4)); the
// reduce-scatter over the 16 slots (xor 8, 4, 2, 1: the reference's tree16)
// leaves (token lane >> 3, head lane & 7) on each lane, returned in out[k]
// times the attention scale.
template <int NC>
__device__ __forceinline__ void ax_score_chunks(const Ctx &c, const float *sm, const float *const *Kb, const int *t0,
                                                int len, int G, float *out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = lane & 15, grp = lane >> 4;
  const ulonglong2 *qlane = (const ulonglong2 *)(sm + kAxQs) + (grp * 8 * 2) * 16 + slot;
  const float *knew = sm + kAxKnew;
  float v[NC][16];
  f2x kp[NC][2][4];
#pragma unroll
  for (int k = 0; k < NC; k++) {
#pragma unroll
    for (int tl = 0; tl < 2; tl++) {
      const int tok = 4 * warp + 2 * grp + tl;
      const float *kr = t0[k] + tok == len ? knew : Kb[k] + (size_t)tok * kHeadDim;
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        const int idx = 16 * (jj ^ grp) + slot;
        kp[k][tl][jj] = f2_pack(kr[idx], kr[idx + 64]);
      }
    }
  }
  // products as the reference forms them, fmaf(q, k, +0) (its slot
  // accumulators start at zero): a packed FMA whose zero addend is read at
  // run time.  ptxas contracts a packed multiply followed by a packed add
  // into an FMA even with explicit .rn, and folds a constant zero addend,
  // either of which changes the sums' rounding.
  const f2x z0 = f2_pack(c.fzero, c.fzero);
#pragma unroll
  for (int h = 0; h < 8; h++) {
    const ulonglong2 qa = qlane[(2 * h) * 16], qb = qlane[(2 * h + 1) * 16];
#pragma unroll
    for (int k = 0; k < NC; k++) {
#pragma unroll
      for (int tl = 0; tl < 2; tl++) {
        const f2x z = f2_add(f2_add(f2_fma(qa.x, kp[k][tl][0], z0), f2_fma(qa.y, kp[k][tl][1], z0)),
                             f2_add(f2_fma(qb.x, kp[k][tl][2], z0), f2_fma(qb.y, kp[k][tl][3], z0)));
        v[k][tl * 8 + h] = h < G ? __fadd_rn(f2_lo(z), f2_hi(z)) : 0.0f;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NC; k++) {
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const bool up = lane & 8;
      const float send = up ? v[k][q] : v[k][8 + q];
      v[k][q] = __fadd_rn(up ? v[k][8 + q] : v[k][q], __shfl_xor_sync(0xffffffffu, send, 8));
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const bool up = lane & 4;
      const float send = up ? v[k][q] : v[k][4 + q];
      v[k][q] = __fadd_rn(up ? v[k][4 + q] : v[k][q], __shfl_xor_sync(0xffffffffu, send, 4));
    }
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const bool up = lane & 2;
      const float send = up ? v[k][q] : v[k][2 + q];
      v[k][q] = __fadd_rn(up ? v[k][2 + q] : v[k][q], __shfl_xor_sync(0xffffffffu, send, 2));
    }
    const bool up = lane & 1;
    const float send = up ? v[k][0] : v[k][1];
    out[k] = __fmul_rn(__fadd_rn(up ? v[k][1] : v[k][0], __shfl_xor_sync(0xffffffffu, send, 1)), c.attn_scale);
  }
}

// Phase 1: scores of the block's chunks (see the top of this file).
__device__ __noinline__ void phase_attn_scores(const Ctx *cp, int layer, float *smem_arg) {
  float *const smem = dyn_smem();  // == smem_arg (the aligned dynamic base)
  (void)smem_arg;
  const Ctx &c = *cp;
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = s_ax_hi - s_ax_lo;
  if (nch <= 0) return;
  const int M = sp.M, nb = ax_nbufs(M);
  rg_bmark(c, 1);
  float *sm = ax_small(c, M, smem);
  if (threadIdx.x == 0) ax_issue_upto(c, layer, smem, nb);
  const uint32_t par0 = s_ax_par;  // parity of each buffer's next completion
  int qpair = -1;
#pragma unroll 1
  for (int i = 0; i < nch;) {
    const int4 d0 = ax_desc(c, sp, i);
    const int4 d1 = i + 1 < nch ? ax_desc(c, sp, i + 1) : make_int4(-1, 0, 0, 0);
    const int nc = d1.x == d0.x ? 2 : 1;  // two chunks of one pair
    const int m = d0.x & 255, g = d0.x >> 8;
    const int n = s_ax_n[m], len = n - 1;
    if (d0.x != qpair) {
      ax_load_q(c, sp, m, g, sm);
      qpair = d0.x;
    }
    const float *Kb[2];
    const int t0[2] = {d0.y, d1.y};
    for (int k = 0; k < nc; k++) {
      const int b = (i + k) % nb;
      Kb[k] = ax_kbuf(c, M, smem, b);
      mbar_wait(&s_ax_full[b], ((par0 >> b) ^ (uint32_t)((i + k) / nb)) & 1u, c.err);
    }
    if (i == 0) rg_bmark(c, 2);
    float sc[2];
    if (nc == 2) {
      ax_score_chunks<2>(c, sm, Kb, t0, len, G, sc);
    } else {
      Kb[1] = Kb[0];
      ax_score_chunks<1>(c, sm, Kb, t0, len, G, sc);
    }
    const int ld = ax_stride(n), h = lane & 7;
    float *srow = c.att_s + s_ax_sb[m] + (size_t)g * G * ld;
    for (int k = 0; k < nc; k++) {
      const int t = t0[k] + 4 * warp + (lane >> 3);
      if (t < n && h < G) __stcg(srow + (size_t)h * ld + t, sc[k]);
      if (t0[k] <= len && len < t0[k] + kAxTok && ((len - t0[k]) >> 2) == warp) {
        // the new position: appended to the cache (kvCache.append,
        // internal/model/model.go:5593-5612)
        const float *knew = sm + kAxKnew;
        ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, 0, g, len))[lane] = ((const float4 *)knew)[lane];
        ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, 1, g, len))[lane] = ((const float4 *)(knew + kHeadDim))[lane];
      }
    }
    // every warp is done with the chunks' buffers (and, at a pair change,
    // with q); the refills go out from two warps
    __syncthreads();
    if (lane == 0 && warp < nc && i + warp + nb < nch) ax_issue(c, layer, smem, i + warp + nb);
    i += nc;
  }
  if (threadIdx.x == 0) {
    // chunk i completed a phase of buffer i % nb
    for (int b = 0; b < nb; b++)
      if (nch > b && (((nch - 1 - b) / nb) & 1) == 0) s_ax_par ^= 1u << b;
    s_ax_issued = 0;
  }
  rg_bmark(c, 3);
  __syncthreads();
}

// Value phase shared memory, from the base of the dynamic shared memory (the
// phase runs alone: no copies of other phases are in flight during it): a
// ring of kAxVRing value-step buffers (V rows of 32 positions, half the head
// dims: 8 KB each; per page one 2-D TMA box of 64 dims x 16 rows from the
// pool map), then the item's scores (G / hg heads x stride floats, one bulk
// copy), which the item turns into exponentials and then weights in place.
// An item whose whole V half (all its pages) and scores fit shared memory
// loads all pages at once instead ("whole" items: the boxes are requested from
// every warp against one barrier, and the chains then run without a block
// barrier per step).
__shared__ __align__(8) uint64_t s_av_bar[kAxVRing + 2];  // value steps, the scores, an item's whole V
__shared__ __align__(8) uint64_t s_av_free[kAxVRing];     // value step buffers released by every warp
__shared__ uint32_t s_av_par;                             // parity of each barrier's next completion
constexpr int kAvPgCap = 576;                             // pages of an item held in shared memory (9,216 positions)
__shared__ int s_av_pg[kAvPgCap];

__device__ __forceinline__ float *ax_vbuf(float *smem, int j) { return (float *)((uint8_t *)smem + (size_t)j * kAxVBytes); }

__device__ __forceinline__ void av_block_init() {
  if (threadIdx.x == 0) {
    for (int j = 0; j <= kAxVRing + 1; j++) mbar_init(&s_av_bar[j], 1);
    for (int j = 0; j < kAxVRing; j++) mbar_init(&s_av_free[j], kThreads / 32);
    mbar_fence_init();
    s_av_par = 0;
  }
}

// One thread: the copies of value step st (positions 32 st .. +31, dims
// 64 half .. +63) of pair (m, g) into ring buffer st % kAxVRing.
__device__ __forceinline__ void av_issue(const Ctx &c, const int *bt, int layer, int g, int half, int st, int n,
                                         float *smem) {
  const int t0 = st * kAxVTok;
  if (t0 >= n) return;
  const int b = st % kAxVRing;
  float *vb = ax_vbuf(smem, b);
  const int np = t0 + kPageTokens < n ? 2 : 1;
  mbar_expect_tx(&s_av_bar[b], (uint32_t)np * kPageTokens * 64 * 4);
  for (int p = 0; p < np; p++) {
    // pool row of (page, layer, kv head g, V, position 0 of the page)
    const int pi = t0 / kPageTokens + p;
    const int page = pi < kAvPgCap ? s_av_pg[pi] : __ldg(bt + pi);
    const int row = (((page * c.L + layer) * c.KVH + g) * 2 + 1) * kPageTokens;
    tma_2d(vb + p * kPageTokens * 64, c.kv_map, 64 * half, row, &s_av_bar[b]);
  }
}

__device__ __forceinline__ float4 lds_f4(const float *p) { return *(const float4 *)p; }
__device__ __forceinline__ f2x lds_f2x(const float *p) { return *(const f2x *)p; }
__device__ __forceinline__ float lds_f1(const float *p) { return *p; }

// Phase 2: softmax and value chains of the step's long caches.  Items are
// (sequence, kv head, half of the dims, group of G / hg heads), longest cache
// first.
__device__ __noinline__ void phase_attn_values(const Ctx *cp, int layer, float *smem_arg) {
  float *const smem = dyn_smem();  // == smem_arg (the aligned dynamic base)
  (void)smem_arg;
  const Ctx &c = *cp;
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH, hg = s_ax_hg, Gs = G / hg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_pair = 2 * hg;
  const int items = s_ax_nl * c.KVH * per_pair;
  float *ssc = (float *)((uint8_t *)smem + kAxVRingBytes);  // the item's scores
  if ((int)blockIdx.x >= items) return;
  // trace marks 4-15 of the block's first item (SM clock cycles): entry,
  // scores landed, weights formed, then (landed, chain done) of steps 0, 1,
  // 8 and the last, exit
  unsigned long long *mk = c.trace && threadIdx.x == 0 ? c.trace + 4 * kTraceRows + kTraceMarks * blockIdx.x : nullptr;
  if (mk) mk[4] = clock64();
  if (lane == 0) {
    // the ring's buffers were last written by ordinary stores in earlier
    // phases; the scores and the new V rows were written by other blocks'
    // ordinary stores (ordered by the grid barrier) and are read by the
    // async proxy (every warp's lane 0 issues copies)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  // items in rows of gridDim.x, longest first; even rows left to right over
  // the blocks, odd rows right to left, so a block's items balance
#pragma unroll 1
  for (int row = 0; row * (int)gridDim.x < items; row++) {
    const int it = row * gridDim.x + ((row & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
    if (it >= items) continue;
    const int pair = it / per_pair, sub = it % per_pair;
    const int m = s_ax_long[pair / c.KVH], g = pair % c.KVH, half = sub & 1, h0 = (sub >> 1) * Gs;
    const int n = s_ax_n[m], nv = n & ~15, ld = ax_stride(n);
    const int *bt = sp.seq[m].bt;
    const float *Sg = c.att_s + s_ax_sb[m] + ((size_t)g * G + h0) * ld;
    const int nst = (n + kAxVTok - 1) / kAxVTok;
    const int npg = (n + kPageTokens - 1) / kPageTokens;
    const bool whole = npg <= kAvPgCap && (size_t)npg * kPageTokens * 256 + (size_t)Gs * ld * 4 <= (size_t)c.dyn_smem;
    float *ssc_i = whole ? smem + (size_t)npg * kPageTokens * 64 : ssc;
    const uint32_t par = s_av_par;
    for (int i = threadIdx.x; i < (n + kPageTokens - 1) / kPageTokens && i < kAvPgCap; i += kThreads)
      s_av_pg[i] = __ldg(bt + i);
    __syncthreads();
    // the scores by one bulk copy; the V steps from every warp (one thread
    // issues bulk copies at about 24 GB/s): step st from warp st % 8
    // (the previous item wrote its weights over its scores with ordinary
    // stores; the copies below reuse that memory)
    if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x == 0) {
      mbar_expect_tx(&s_av_bar[kAxVRing], (uint32_t)(Gs * ld * 4));
      bulk_g2s(ssc_i, Sg, (uint32_t)(Gs * ld * 4), &s_av_bar[kAxVRing]);
      if (whole) mbar_expect_tx(&s_av_bar[kAxVRing + 1], (uint32_t)npg * kPageTokens * 64 * 4);
    }
    if (whole) {
      __syncthreads();  // the expected bytes are registered before any box lands
      if (lane == 0)
        for (int p = warp; p < npg; p += kThreads / 32) {
          const int row = (((s_av_pg[p] * c.L + layer) * c.KVH + g) * 2 + 1) * kPageTokens;
          tma_2d(smem + (size_t)p * kPageTokens * 64, c.kv_map, 64 * half, row, &s_av_bar[kAxVRing + 1]);
        }
    } else if (lane == 0) {
      for (int st = warp; st < kAxVRing && st < nst; st += kThreads / 32) av_issue(c, bt, layer, g, half, st, n, smem);
    }
    mbar_wait(&s_av_bar[kAxVRing], (par >> kAxVRing) & 1u, c.err);
    if (mk && row == 0) mk[5] = clock64();
    // ---- softmax of head h0 + warp (warps < Gs), in place: scores ->
    // exponentials (positions below nv) -> weights (times 1/sum, all n)
    float *W = ssc_i + (size_t)(warp < Gs ? warp : 0) * ld;
    if (warp < Gs) {
      float mx = -INFINITY;
      for (int i4 = lane; i4 < ld / 4; i4 += 32) {
        const float4 v = lds_f4(W + 4 * i4);
        const int t = 4 * i4;
        mx = fmaxf(mx, t < n ? v.x : -INFINITY);
        mx = fmaxf(mx, t + 1 < n ? v.y : -INFINITY);
        mx = fmaxf(mx, t + 2 < n ? v.z : -INFINITY);
        mx = fmaxf(mx, t + 3 < n ? v.w : -INFINITY);
      }
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      // exponentials, four independent ones per lane at a time
      for (int t0 = 4 * lane; t0 < nv; t0 += 128) {
        const float4 v = lds_f4(W + t0);  // nv is a multiple of 16: t0 + 3 < nv
        *(float4 *)(W + t0) = make_float4(exp_fma(__fsub_rn(v.x, mx)), exp_fma(__fsub_rn(v.y, mx)),
                                          exp_fma(__fsub_rn(v.z, mx)), exp_fma(__fsub_rn(v.w, mx)));
      }
      __syncwarp();
      // lane chains: lane l (< 16) adds e_l, e_{l+16}, ... in order; loads
      // eight steps ahead of the adds
      float acc = 0.0f;
      if (lane < 16) {
        int t = lane;
        for (; t + 7 * 16 < nv; t += 8 * 16) {
          float e[8];
#pragma unroll
          for (int u = 0; u < 8; u++) e[u] = W[t + 16 * u];
#pragma unroll
          for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, e[u]);
        }
        for (; t < nv; t += 16) acc = __fadd_rn(acc, W[t]);
      }
      // tree16 of lanes 0..15: (l, l+8), (l, l+4), then (0+2)+(1+3)
      float a = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 2));
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 1));
      const float inv = __shfl_sync(0xffffffffu, __fdiv_rn(1.0f, a), 0);
      // weights: exponential (or the tail's raw score) times 1/sum (the
      // stride's padding past n is scaled too and never read)
      for (int t0 = 4 * lane; t0 < ld; t0 += 128) {
        const float4 v = lds_f4(W + t0);
        *(float4 *)(W + t0) = make_float4(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv),
                                          __fmul_rn(v.w, inv));
      }
      __syncwarp();
    }
    if (mk && row == 0) mk[6] = clock64();
    // ---- value chains: warp h, dims 64 half + 2 lane, +1
    f2x o = 0ull;
    if (whole) {
      mbar_wait(&s_av_bar[kAxVRing + 1], (par >> (kAxVRing + 1)) & 1u, c.err);
      if (warp < Gs) {
        // o = w_0 v_0, then batches of 16 positions: their V pairs and
        // weights loaded, then the FMAs in position order
        const float *vb = smem + 2 * lane;
        o = f2_mul(f2_pack(W[0], W[0]), *(const f2x *)vb);
        int t = 1;
#pragma unroll 1
        for (; t + 16 <= n; t += 16) {
          f2x v[16];
          float w[16];
#pragma unroll
          for (int u = 0; u < 16; u++) {
            v[u] = *(const f2x *)(vb + (t + u) * 64);
            w[u] = W[t + u];
          }
#pragma unroll
          for (int u = 0; u < 16; u++) o = f2_fma(f2_pack(w[u], w[u]), v[u], o);
        }
#pragma unroll 1
        for (; t < n; t++) o = f2_fma(f2_pack(W[t], W[t]), *(const f2x *)(vb + t * 64), o);
      }
    }
    // ring: buffer b serves steps b, b + kAxVRing, ...; every warp releases a
    // step's buffer (s_av_free, whose completions pair with the buffer's
    // loads, so one parity serves both) and the step one behind is refilled
    // by the warp whose turn it is, so no block barrier runs per step
#pragma unroll 1
    for (int st = 0; st < (whole ? 0 : nst); st++) {
      const int t0 = st * kAxVTok;
      const int b = st % kAxVRing;
      // step st's rows (use st / kAxVRing of buffer b); every warp waits for
      // them, so that no warp's release of a later use of the buffer can
      // count toward this one
      mbar_wait(&s_av_bar[b], ((par >> b) ^ (uint32_t)(st / kAxVRing)) & 1u, c.err);
      if (warp < Gs) {
        const float *vb = ax_vbuf(smem, b) + 2 * lane;
        const float *wt = W + t0;  // 16-byte aligned: rows start on 4-float boundaries, t0 % 32 == 0
        const int cnt = min(kAxVTok, n - t0);
        // the chain o = fma(w_t, v_t, o) is sequential; four weights per
        // shared load, a batch's loads ahead of its FMAs
        int i = 0;
        if (st == 0) {
          const float w0 = wt[0];
          o = f2_mul(f2_pack(w0, w0), *(const f2x *)vb);
          i = 1;
        }
        if (cnt == kAxVTok && i == 0) {
#pragma unroll
          for (int u0 = 0; u0 < kAxVTok; u0 += 8) {
            const float4 wa = *(const float4 *)(wt + u0), wb = *(const float4 *)(wt + u0 + 4);
            const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
            f2x v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = *(const f2x *)(vb + (u0 + u) * 64);
#pragma unroll
            for (int u = 0; u < 8; u++) o = f2_fma(f2_pack(w[u], w[u]), v[u], o);
          }
        } else {
#pragma unroll 8
          for (; i < cnt; i++) {
            const float wi = wt[i];
            o = f2_fma(f2_pack(wi, wi), *(const f2x *)(vb + i * 64), o);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(smem_u32(&s_av_free[b])) : "memory");
        const int rs = st - 1 + kAxVRing;  // the next step of the previous step's buffer
        if (st >= 1 && rs < nst && warp == (st - 1) % (kThreads / 32)) {
          const int bp = (st - 1) % kAxVRing;
          mbar_wait(&s_av_free[bp], ((par >> bp) ^ (uint32_t)((st - 1) / kAxVRing)) & 1u, c.err, true);
          av_issue(c, bt, layer, g, half, rs, n, smem);
        }
      }
    }
    if (warp < Gs) {
      float2 r;
      r.x = f2_lo(o);
      r.y = f2_hi(o);
      *(float2 *)(c.head + ((size_t)m * c.QH + (size_t)g * G + h0 + warp) * kHeadDim + 64 * half + 2 * lane) = r;
    }
    if (threadIdx.x == 0) {
      // step i completed a phase of buffer i % kAxVRing; the scores one
      uint32_t p = par;
      if (whole) {
        p ^= 1u << (kAxVRing + 1);
      } else {
        for (int j = 0; j < kAxVRing; j++)
          if (nst > j && (((nst - 1 - j) / kAxVRing) & 1) == 0) p ^= 1u << j;
      }
      p ^= 1u << kAxVRing;
      s_av_par = p;
    }
    __syncthreads();  // the scores' copy and s_av_par are settled for the next item
    if (mk && row == 0) mk[15] = clock64();
  }
}

// KV append of the long caches without attention (the last layer of a step
// that needs no logits): one warp per (sequence, kv head).
__device__ void phase_append_long(const Ctx &c, int layer) {
  const StepParams &sp = *c.sp;
  const size_t qkvld = (size_t)(c.QH + 2 * c.KVH) * kHeadDim;
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (kThreads / 32);
  for (int p = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); p < sp.M * c.KVH; p += nw) {
    const int m = p / c.KVH, g = p % c.KVH;
    const int len = sp.seq[m].len;
    if (len + 1 <= kAttnChunk) continue;
    const float *row = c.qkv + (size_t)m * qkvld;
    const int *pos = sp.seq[m].pos;
    if (lane < 16) {
      const float4 *kn = (const float4 *)(row + (size_t)(c.QH + g) * kHeadDim);
      float4 a = __ldcg(kn + lane), b = __ldcg(kn + lane + 16);
      if (pos[0] != 0 || pos[1] != 0 || pos[2] != 0) {
        float cs[4], sn[4];
        rope_cs4(c, pos, lane, cs, sn);
        rope4(a, b, cs, sn);
      }
      float4 *kd = (float4 *)kv_ptr(c, sp.seq[m].bt, layer, 0, g, len);
      kd[lane] = a;
      kd[lane + 16] = b;
    }
    ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, 1, g, len))[lane] =
        __ldcg((const float4 *)(row + (size_t)(c.QH + c.KVH + g) * kHeadDim) + lane);
  }
}

}  // namespace ocrvl
