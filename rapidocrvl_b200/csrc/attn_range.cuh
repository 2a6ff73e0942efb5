// Attention over long caches (more than kAttnChunk positions), streamed in
// contiguous page ranges.  Included by decoder.cuh after the KV, RoPE,
// mbarrier and stage-ring helpers.
//
// Segments.  The np pages of a (sequence m, kv head g) pair split into
// segments of S pages: S = 1 when np <= kSegMax, else the even number
// 2 * ceil(np / (2 kSegMax)), so a pair has at most kSegMax segments and a
// segment is a whole number of 32-token chunks.  The split depends on the
// cache length only: a sequence's result does not depend on the other
// sequences of the step (a batched step equals the single steps bit for bit).
//
// Blocks.  The segments of the step, in (m, g, segment) order, go to the
// blocks balanced by pages: block b takes those whose first page falls in
// [ceil(P b / nb), ceil(P (b + 1) / nb)) of the P pages of the step.  A block
// streams its segments' pages in chunks of two pages (K then V, 32 tokens,
// one 32 KB buffer) through kRangeBufs buffers filled by TMA bulk copies, the
// first ones issued before the phase when the block's shared memory allows.
//
// Softmax per query head and segment, online:
//   m_s  running max over all scores,
//   l_s  sum of exp(s - m_s) over the positions below nv = 16 floor(n / 16),
//   o_s  sum of exp(s - m_s) v (scaled by exp(m_old - m_new) when m grows),
//   T    sum of s v over the positions at or above nv, which the reference
//        weights by their raw score (expF32VecFMA leaves the tail
//        unexponentiated, internal/tensor/dot_amd64.s:6131-6168).
// The block that completes the last segment of (m, g) merges, in segment
// order: head = (T + sum_k exp(m_k - M) o_k) / sum_k exp(m_k - M) l_k with
// M = max_k m_k (the reference's max over all n scores and its 1/sum).
//
// Chunk work (256 threads).  Scores: warp w takes the chunk's tokens
// 4w .. 4w+3, lanes 0-15 the first two and lanes 16-31 the other two, for all
// G query heads of the kv head.  Lane slot s multiplies dims s + 16 j
// (j = 0..7) and sums them as ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)); a
// reduce-scatter over the 16 slots (xor 8, 4, 2, 1) then leaves one
// (token, head) score per lane.  That is the reference's dotF32 order (16
// slot accumulators, the tree16 of the slots), so each score equals the
// single-item path's bit for bit.  Softmax: warp h updates head h over the
// chunk's 32 scores.  Values: thread (dim d, token half) accumulates d of all
// G heads over its 16 tokens; the halves are added at the segment's end.

namespace ocrvl {

constexpr int kSegMax = 32;    // segments of one (sequence, kv head) pair at most
constexpr int kRangeBufs = 4;  // chunk buffers per block
constexpr int kRangeTok = 32;  // tokens per chunk (two KV pages)
static_assert(2 * kRangeTok * kHeadDim * 4 == kStageBytes, "a chunk's K and V fill one ring slot");
static_assert(kRangeBufs <= kStagesM1 - 1, "single-sequence layout: buffers in ring slots 1..");
static_assert(kMaxGroup == 8 && kHeadDim == 128, "score layout: 8 heads x 2 tokens per half-warp");
static_assert(kSegMax <= 32, "merge: one segment per lane");

// Small arrays of the range phase (floats from their base).
constexpr int kRgQs = 0;                                  // [8][128] rotated q
constexpr int kRgPreLen = 8 * 128 + 128 + 128 + 64 + 64;  // raw q | new k | new v | cos | sin
constexpr int kRgPre = kRgQs + 8 * 128;                   // two prefetch buffers
constexpr int kRgKnew = kRgPre + 2 * kRgPreLen;           // [128] rotated new k, [128] new v
constexpr int kRgS = kRgKnew + 256;                       // [8 heads][32 tokens] scores
constexpr int kRgW = kRgS + 256;                          // [32 tokens][8 heads] weights
constexpr int kRgAlpha = kRgW + 256;                      // [8] rescale factors
constexpr int kRgRed = kRgAlpha + 32;                     // [8][128] o of token half 1
constexpr int kRgT = kRgRed + 8 * 128;                    // [2 halves][8][128] raw-weighted tail sums
constexpr int kRgFloats = kRgT + 2 * 8 * 128;
static_assert(kRgFloats * 4 <= kStageBytes, "small arrays fit one ring slot");
static_assert(kRgPreLen % 4 == 0 && kRgPre % 4 == 0, "16-byte aligned prefetch buffers");

// Shared memory the range phase needs when M > 1 (its buffers then start at
// the base of the dynamic shared memory; for M <= 1 they use ring slots
// kStagesM1-1 .. kStagesM1-kRangeBufs and the small arrays ring slot 0).
__host__ __device__ __forceinline__ size_t rg_smem_bytes_multi() {
  return (size_t)kRangeBufs * kStageBytes + (size_t)kRgFloats * 4;
}

__device__ __forceinline__ float *rg_buf(const Ctx &c, int M, float *smem, int j) {
  if (M <= 1)
    return (float *)((uint8_t *)smem + gemv_prologue_bytes(c.qtype, 1, c.pro_cols) +
                     (size_t)(kStagesM1 - 1 - j) * kStageBytes);
  return (float *)((uint8_t *)smem + (size_t)j * kStageBytes);
}
__device__ __forceinline__ float *rg_small(const Ctx &c, int M, float *smem) {
  if (M <= 1) return (float *)((uint8_t *)smem + gemv_prologue_bytes(c.qtype, 1, c.pro_cols));
  return (float *)((uint8_t *)smem + (size_t)kRangeBufs * kStageBytes);
}

__host__ __device__ __forceinline__ int rg_seg_pages(int np) {
  return np <= kSegMax ? 1 : 2 * ((np + 2 * kSegMax - 1) / (2 * kSegMax));
}

// Position in the step's stream of segments and chunks.
struct RgCur {
  int m;               // sequence, -1 past the last long cache
  int g, k, j;         // kv head, segment of (m, g), chunk of the segment
  int n, np, S, nseg;  // positions (incl. the new one), pages, pages per segment, segments
  int pbase, sbase;    // pages and segments of the long caches before m
};

// Moves to the first long cache at or after sequence m (pbase / sbase are the
// caller's).
__device__ __forceinline__ void rg_load_seq(const StepParams &sp, RgCur &r, int m) {
  while (m < sp.M && sp.seq[m].len + 1 <= kAttnChunk) m++;
  r.g = r.k = r.j = 0;
  if (m >= sp.M) {
    r.m = -1;
    return;
  }
  r.m = m;
  r.n = sp.seq[m].len + 1;
  r.np = (r.n + kPageTokens - 1) / kPageTokens;
  r.S = rg_seg_pages(r.np);
  r.nseg = (r.np + r.S - 1) / r.S;
}

__device__ __forceinline__ int rg_seg_np(const RgCur &r) { return min(r.np, (r.k + 1) * r.S) - r.k * r.S; }
__device__ __forceinline__ int rg_start(const RgCur &r) { return r.pbase + r.g * r.np + r.k * r.S; }
__device__ __forceinline__ bool rg_in(const RgCur &r, int hi) { return r.m >= 0 && rg_start(r) < hi; }
__device__ __forceinline__ int rg_seg_index(const RgCur &r) { return r.sbase + r.g * r.nseg + r.k; }

__device__ __forceinline__ void rg_next_seg(const Ctx &c, const StepParams &sp, RgCur &r) {
  r.j = 0;
  if (++r.k < r.nseg) return;
  r.k = 0;
  if (++r.g < c.KVH) return;
  r.pbase += c.KVH * r.np;
  r.sbase += c.KVH * r.nseg;
  rg_load_seq(sp, r, r.m + 1);
}

__device__ __forceinline__ void rg_next_chunk(const Ctx &c, const StepParams &sp, RgCur &r) {
  if (2 * (r.j + 1) < rg_seg_np(r)) {
    r.j++;
    return;
  }
  rg_next_seg(c, sp, r);
}

__device__ __forceinline__ int rg_total_pages(const Ctx &c, const StepParams &sp) {
  int P = 0;
  for (int m = 0; m < sp.M; m++) {
    const int n = sp.seq[m].len + 1;
    if (n > kAttnChunk) P += c.KVH * ((n + kPageTokens - 1) / kPageTokens);
  }
  return P;
}

__device__ __forceinline__ int rg_bound(int P, int b, int nb) { return (int)(((long long)P * b + nb - 1) / nb); }

// First segment whose first page is at or after page `lo` of the step.
__device__ void rg_seek(const Ctx &c, const StepParams &sp, int lo, RgCur &r) {
  r.pbase = r.sbase = 0;
  rg_load_seq(sp, r, 0);
  while (r.m >= 0) {
    const int tot = c.KVH * r.np;
    if (lo < r.pbase + tot) {
      const int off = max(0, lo - r.pbase);
      int g = off / r.np;
      const int rem = off - g * r.np;
      int k = (rem + r.S - 1) / r.S;
      if (k >= r.nseg) {
        k = 0;
        g++;
      }
      if (g < c.KVH) {
        r.g = g;
        r.k = k;
        r.j = 0;
        return;
      }
    }
    r.pbase += tot;
    r.sbase += c.KVH * r.nseg;
    rg_load_seq(sp, r, r.m + 1);
  }
}

// Per-block state of the range loads, kept across the phases of a launch:
// s_rg_full[j] completes when buffer j's copies land, s_rg_par bit j is the
// parity of its next completion, s_rg_issued counts the chunks of the coming
// attention phase already issued (into buffers 0 .. s_rg_issued-1).
__shared__ __align__(8) uint64_t s_rg_full[kRangeBufs];
__shared__ uint32_t s_rg_par;
__shared__ int s_rg_issued;

__device__ __forceinline__ void rg_block_init() {
  if (threadIdx.x == 0) {
    for (int j = 0; j < kRangeBufs; j++) mbar_init(&s_rg_full[j], 1);
    mbar_fence_init();
    s_rg_par = 0;
    s_rg_issued = 0;
  }
}

// Waits for range copies issued ahead of a phase that did not run (thread 0).
__device__ __forceinline__ void rg_drain(const Ctx &c) {
  for (int j = 0; j < s_rg_issued; j++) {
    mbar_wait(&s_rg_full[j], (s_rg_par >> j) & 1u, c.err);
    s_rg_par ^= 1u << j;
  }
  s_rg_issued = 0;
}

// One thread: bulk copies of chunk r's K and V pages into buf.
__device__ __forceinline__ void rg_issue(const Ctx &c, int layer, const RgCur &r, float *buf, uint64_t *bar) {
  const int *bt = c.sp->seq[r.m].bt;
  const int p = r.k * r.S + 2 * r.j;
  const int pages = min(2, r.k * r.S + rg_seg_np(r) - p);
  constexpr uint32_t pb = (uint32_t)kPageTokens * kHeadDim * 4;
  mbar_expect_tx(bar, 2u * pages * pb);
  for (int q = 0; q < pages; q++) {
    bulk_g2s(buf + q * kPageTokens * kHeadDim, kv_ptr(c, bt, layer, 0, r.g, (p + q) * kPageTokens), pb, bar);
    bulk_g2s(buf + (kRangeTok + q * kPageTokens) * kHeadDim, kv_ptr(c, bt, layer, 1, r.g, (p + q) * kPageTokens), pb,
             bar);
  }
}

// One thread: issues this block's chunks s_rg_issued .. upto-1 (chunk i into
// buffer i); r is left at the next chunk to issue and i at its index.
__device__ void rg_issue_ahead(const Ctx &c, int layer, float *smem, int upto, RgCur &r, int &i) {
  const StepParams &sp = *c.sp;
  const int P = rg_total_pages(c, sp);
  i = 0;
  r.m = -1;
  if (P == 0) return;
  const int hi = rg_bound(P, blockIdx.x + 1, gridDim.x);
  rg_seek(c, sp, rg_bound(P, blockIdx.x, gridDim.x), r);
  for (; i < s_rg_issued && rg_in(r, hi); i++) rg_next_chunk(c, sp, r);
  // the buffers were last touched by ordinary loads and stores
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  for (; i < upto && rg_in(r, hi); i++) {
    rg_issue(c, layer, r, rg_buf(c, sp.M, smem, i), &s_rg_full[i]);
    rg_next_chunk(c, sp, r);
  }
  s_rg_issued = i;
}

// All threads: cp.async copies of segment r's raw q (G heads), its new k and
// v (last segment of the pair) and the cos / sin of the sequence's position.
__device__ __forceinline__ void rg_prefetch_seg(const Ctx &c, const StepParams &sp, const RgCur &r, float *pre) {
  const int G = c.QH / c.KVH;
  const size_t qkvld = (size_t)(c.QH + 2 * c.KVH) * kHeadDim;
  const float *row = c.qkv + (size_t)r.m * qkvld;
  const int t = threadIdx.x;
  if (t < G * 32) cp_async16(pre + 4 * t, row + (size_t)r.g * G * kHeadDim + 4 * t);
  if (r.k == r.nseg - 1 && t < 64) {
    const int kind = t >> 5, i4 = t & 31;
    cp_async16(pre + 1024 + 128 * kind + 4 * i4, row + (size_t)(c.QH + kind * c.KVH + r.g) * kHeadDim + 4 * i4);
  }
  if (t >= 128 && t < 256) {
    const int i = (t - 128) & 63;
    const int p = sp.seq[r.m].pos[c.sec_axis[i]];
    const float *tab = t < 192 ? c.rope_cos : c.rope_sin;
    cp_async4(pre + 1280 + (t - 128), tab + (size_t)p * (kHeadDim / 2) + i);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Warps h < G of the block that completed (m, g): merge head h's segments.
__device__ void rg_merge(const Ctx &c, int m, int g, int n, int sb, int nseg) {
  const int G = c.QH / c.KVH;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= G) return;
  const float *ml = c.part_ml + ((size_t)sb * G + h) * 2;  // segment k at + 2 G k
  const float mk = lane < nseg ? __ldcg(ml + (size_t)2 * G * lane) : -INFINITY;
  const float lk = lane < nseg ? __ldcg(ml + (size_t)2 * G * lane + 1) : 0.0f;
  float mx = mk;
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float sk = lane < nseg ? exp_fma(__fsub_rn(mk, mx)) : 0.0f;
  float den = __fmul_rn(sk, lk);
  for (int o = 16; o > 0; o >>= 1) den = __fadd_rn(den, __shfl_xor_sync(0xffffffffu, den, o));
  const size_t hq = (size_t)m * c.QH + (size_t)g * G + h;
  float4 acc = (n & 15) ? __ldcg((const float4 *)(c.part_t + hq * kHeadDim) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 *po = (const float4 *)(c.part_o + ((size_t)sb * G + h) * kHeadDim) + lane;
  const size_t pstride = (size_t)G * (kHeadDim / 4);  // float4 per segment
#pragma unroll 1
  for (int k0 = 0; k0 < nseg; k0 += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (k0 + u < nseg) v[u] = __ldcg(po + (size_t)(k0 + u) * pstride);
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const float s = __shfl_sync(0xffffffffu, sk, (k0 + u) & 31);
      if (k0 + u < nseg) {
        acc.x = __fmaf_rn(s, v[u].x, acc.x);
        acc.y = __fmaf_rn(s, v[u].y, acc.y);
        acc.z = __fmaf_rn(s, v[u].z, acc.z);
        acc.w = __fmaf_rn(s, v[u].w, acc.w);
      }
    }
  }
  const float di = __fdiv_rn(1.0f, den);
  ((float4 *)(c.head + hq * kHeadDim))[lane] =
      make_float4(__fmul_rn(acc.x, di), __fmul_rn(acc.y, di), __fmul_rn(acc.z, di), __fmul_rn(acc.w, di));
}

// Attention of the step's long caches (see the top of this file).
__device__ __noinline__ void phase_attn_range(const Ctx *cp, int layer, float *smem) {
  const Ctx &c = *cp;
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = lane & 15, grp = lane >> 4;
  const int d = threadIdx.x & 127, th = threadIdx.x >> 7;
  const int P = rg_total_pages(c, sp);
  if (P == 0) return;
  const int hi = rg_bound(P, blockIdx.x + 1, gridDim.x);
  float *sm = rg_small(c, sp.M, smem);
  float *qs = sm + kRgQs, *S = sm + kRgS, *W = sm + kRgW, *alph = sm + kRgAlpha, *red = sm + kRgRed;
  float *knew = sm + kRgKnew, *Tsm = sm + kRgT;
  __shared__ int s_merge;
  RgCur cur;
  rg_seek(c, sp, rg_bound(P, blockIdx.x, gridDim.x), cur);
  if (!rg_in(cur, hi)) return;
  // thread 0: the issue cursor (next chunk to copy) and its index
  RgCur icur;
  int inext = 0;
  if (threadIdx.x == 0) rg_issue_ahead(c, layer, smem, kRangeBufs, icur, inext);
  rg_prefetch_seg(c, sp, cur, sm + kRgPre);
  int ci = 0;    // chunk index in the block's stream
  int sidx = 0;  // segment index in the block's stream
  while (rg_in(cur, hi)) {
    // ---- segment start: rotated q (and new k) from the prefetched rows
    const float *pre = sm + kRgPre + (sidx & 1) * kRgPreLen;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int m = cur.m, g = cur.g, n = cur.n, len = n - 1, nv = n & ~15;
    const bool last_seg = cur.k == cur.nseg - 1;
    const int *pos = sp.seq[m].pos;
    const bool has_rope = pos[0] != 0 || pos[1] != 0 || pos[2] != 0;
    const float *rc = pre + 1280, *rs = pre + 1344;
    for (int p = threadIdx.x; p < G * 16 + (last_seg ? 48 : 0); p += kThreads) {
      if (p < G * 16) {
        const int hh = p >> 4, i4 = p & 15;
        float4 a = ((const float4 *)(pre + hh * kHeadDim))[i4], b = ((const float4 *)(pre + hh * kHeadDim + 64))[i4];
        if (has_rope) rope4(a, b, rc + 4 * i4, rs + 4 * i4);
        ((float4 *)(qs + hh * kHeadDim))[i4] = a;
        ((float4 *)(qs + hh * kHeadDim + 64))[i4] = b;
      } else if (p < G * 16 + 16) {
        const int i4 = p - G * 16;
        float4 a = ((const float4 *)(pre + 1024))[i4], b = ((const float4 *)(pre + 1024 + 64))[i4];
        if (has_rope) rope4(a, b, rc + 4 * i4, rs + 4 * i4);
        ((float4 *)knew)[i4] = a;
        ((float4 *)knew)[i4 + 16] = b;
      } else {
        const int i4 = p - G * 16 - 16;
        ((float4 *)(knew + 128))[i4] = ((const float4 *)(pre + 1152))[i4];
      }
    }
    __syncthreads();
    RgCur nxt = cur;
    rg_next_seg(c, sp, nxt);
    if (rg_in(nxt, hi)) rg_prefetch_seg(c, sp, nxt, sm + kRgPre + ((sidx + 1) & 1) * kRgPreLen);
    float qr[8][8];
#pragma unroll
    for (int h = 0; h < 8; h++)
#pragma unroll
      for (int jj = 0; jj < 8; jj++) qr[h][jj] = h < G ? qs[h * kHeadDim + 16 * (jj ^ grp) + slot] : 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;  // warp h < G: head h
    float o[8];
#pragma unroll
    for (int h = 0; h < 8; h++) o[h] = 0.0f;
    const int seg_np = rg_seg_np(cur);
    const int nck = (seg_np + 1) / 2;
    const int sp0 = cur.k * cur.S;  // first page of the segment
#pragma unroll 1
    for (int j = 0; j < nck; j++, ci++) {
      const int b = ci % kRangeBufs;
      float *Kb = rg_buf(c, sp.M, smem, b), *Vb = Kb + kRangeTok * kHeadDim;
      const int p0 = sp0 + 2 * j;
      const int t0 = p0 * kPageTokens;
      const int cnt = min(min(2, sp0 + seg_np - p0) * kPageTokens, n - t0);
      mbar_wait(&s_rg_full[b], (s_rg_par >> b) & 1u, c.err);
      if (t0 <= len && len < t0 + cnt) {
        // the new token: appended to the cache (kvCache.append,
        // internal/model/model.go:5593-5612) and patched into the chunk
        if (threadIdx.x < 64) {
          const int kind = threadIdx.x >> 5, i4 = threadIdx.x & 31;
          const float4 v = ((const float4 *)(knew + kind * 128))[i4];
          ((float4 *)((kind ? Vb : Kb) + (size_t)(len - t0) * kHeadDim))[i4] = v;
          ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, kind, g, len))[i4] = v;
        }
        __syncthreads();
      }
      // ---- scores
      {
        float part[16];
#pragma unroll
        for (int tl = 0; tl < 2; tl++) {
          const float *kr = Kb + (size_t)(4 * warp + 2 * grp + tl) * kHeadDim;
          float kk[8];
#pragma unroll
          for (int jj = 0; jj < 8; jj++) kk[jj] = kr[16 * (jj ^ grp) + slot];
#pragma unroll
          for (int h = 0; h < 8; h++) {
            float pr[8];
#pragma unroll
            for (int jj = 0; jj < 8; jj++) pr[jj] = __fmul_rn(qr[h][jj], kk[jj]);
            part[tl * 8 + h] = __fadd_rn(__fadd_rn(__fadd_rn(pr[0], pr[1]), __fadd_rn(pr[2], pr[3])),
                                         __fadd_rn(__fadd_rn(pr[4], pr[5]), __fadd_rn(pr[6], pr[7])));
          }
        }
        // reduce-scatter over the slots: lane keeps value (slot) = token
        // half (slot >> 3), head (slot & 7)
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const bool up = lane & 8;
          const float send = up ? part[i] : part[8 + i];
          part[i] = __fadd_rn(up ? part[8 + i] : part[i], __shfl_xor_sync(0xffffffffu, send, 8));
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const bool up = lane & 4;
          const float send = up ? part[i] : part[4 + i];
          part[i] = __fadd_rn(up ? part[4 + i] : part[i], __shfl_xor_sync(0xffffffffu, send, 4));
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
          const bool up = lane & 2;
          const float send = up ? part[i] : part[2 + i];
          part[i] = __fadd_rn(up ? part[2 + i] : part[i], __shfl_xor_sync(0xffffffffu, send, 2));
        }
        {
          const bool up = lane & 1;
          const float send = up ? part[0] : part[1];
          part[0] = __fadd_rn(up ? part[1] : part[0], __shfl_xor_sync(0xffffffffu, send, 1));
        }
        S[(slot & 7) * 32 + 4 * warp + 2 * grp + (slot >> 3)] = __fmul_rn(part[0], c.attn_scale);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        s_rg_par ^= 1u << b;
        // every thread is past the previous chunk: its buffer takes the next copy
        while (inext <= ci - 1 + kRangeBufs && rg_in(icur, hi)) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          const int bb = inext % kRangeBufs;
          rg_issue(c, layer, icur, rg_buf(c, sp.M, smem, bb), &s_rg_full[bb]);
          rg_next_chunk(c, sp, icur);
          inext++;
        }
      }
      // ---- online softmax, warp h = head h
      if (warp < G) {
        const float s = S[warp * 32 + lane];
        const bool valid = lane < cnt;
        float pm = valid ? s : -INFINITY;
        for (int o2 = 16; o2 > 0; o2 >>= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o2));
        const float m_new = fmaxf(m_run, pm);
        const float alpha = m_run == -INFINITY ? 0.0f : exp_fma(__fsub_rn(m_run, m_new));
        const bool raw = t0 + lane >= nv;
        float e = 0.0f;
        if (valid) e = raw ? s : exp_fma(__fsub_rn(s, m_new));
        float le = valid && !raw ? e : 0.0f;
        for (int o2 = 16; o2 > 0; o2 >>= 1) le = __fadd_rn(le, __shfl_xor_sync(0xffffffffu, le, o2));
        l_run = __fadd_rn(__fmul_rn(l_run, alpha), le);
        m_run = m_new;
        W[lane * 8 + warp] = e;
        if (lane == 0) alph[warp] = alpha;
      }
      __syncthreads();
      // ---- values: thread (d, th), tokens th*16 .. th*16+15 of the chunk
      {
        float av[8];
#pragma unroll
        for (int h = 0; h < 8; h++) av[h] = h < G ? alph[h] : 0.0f;
#pragma unroll
        for (int h = 0; h < 8; h++) o[h] = __fmul_rn(o[h], av[h]);
        const int tb = th * 16, te = min(cnt, tb + 16);
        const int tt = min(max(nv - t0, tb), te);  // [tb, tt) exponentiated, [tt, te) raw
#pragma unroll 4
        for (int t = tb; t < tt; t++) {
          const float v = Vb[(size_t)t * kHeadDim + d];
          const float4 w0 = ((const float4 *)(W + t * 8))[0], w1 = ((const float4 *)(W + t * 8))[1];
          o[0] = __fmaf_rn(w0.x, v, o[0]);
          o[1] = __fmaf_rn(w0.y, v, o[1]);
          o[2] = __fmaf_rn(w0.z, v, o[2]);
          o[3] = __fmaf_rn(w0.w, v, o[3]);
          o[4] = __fmaf_rn(w1.x, v, o[4]);
          o[5] = __fmaf_rn(w1.y, v, o[5]);
          o[6] = __fmaf_rn(w1.z, v, o[6]);
          o[7] = __fmaf_rn(w1.w, v, o[7]);
        }
        if (t0 + cnt > nv) {
          // the chunk holding the positions at or above nv (the last one of
          // the pair): this half's raw-weighted sums, zero when it has none
          float ta[8];
#pragma unroll
          for (int h = 0; h < 8; h++) ta[h] = 0.0f;
#pragma unroll 1
          for (int t = tt; t < te; t++) {
            const float v = Vb[(size_t)t * kHeadDim + d];
            const float4 w0 = ((const float4 *)(W + t * 8))[0], w1 = ((const float4 *)(W + t * 8))[1];
            ta[0] = __fmaf_rn(w0.x, v, ta[0]);
            ta[1] = __fmaf_rn(w0.y, v, ta[1]);
            ta[2] = __fmaf_rn(w0.z, v, ta[2]);
            ta[3] = __fmaf_rn(w0.w, v, ta[3]);
            ta[4] = __fmaf_rn(w1.x, v, ta[4]);
            ta[5] = __fmaf_rn(w1.y, v, ta[5]);
            ta[6] = __fmaf_rn(w1.z, v, ta[6]);
            ta[7] = __fmaf_rn(w1.w, v, ta[7]);
          }
#pragma unroll
          for (int h = 0; h < 8; h++) Tsm[th * 1024 + h * kHeadDim + d] = ta[h];
        }
      }
    }
    // ---- segment end: the partial (halves added in order), arrival, merge
    const bool has_tail = last_seg && (n & 15) != 0;
    const int seg = rg_seg_index(cur);
    if (th == 1) {
#pragma unroll
      for (int h = 0; h < 8; h++)
        if (h < G) red[h * kHeadDim + d] = o[h];
    }
    __syncthreads();
    if (th == 0) {
#pragma unroll
      for (int h = 0; h < 8; h++)
        if (h < G) {
          c.part_o[((size_t)seg * G + h) * kHeadDim + d] = __fadd_rn(o[h], red[h * kHeadDim + d]);
          if (has_tail)
            c.part_t[((size_t)m * c.QH + (size_t)g * G + h) * kHeadDim + d] =
                __fadd_rn(Tsm[h * kHeadDim + d], Tsm[1024 + h * kHeadDim + d]);
        }
    }
    if (warp < G && lane == 0) {
      c.part_ml[((size_t)seg * G + warp) * 2] = m_run;
      c.part_ml[((size_t)seg * G + warp) * 2 + 1] = l_run;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      // release: the block's partials (ordered before by the barrier) become
      // visible with the count; acquire: the merger sees the others' partials
      unsigned *cntp = c.attn_count + 2 * (m * c.KVH + g);
      unsigned v;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(v) : "l"(cntp) : "memory");
      s_merge = (int)v == cur.nseg - 1;
      if (s_merge) cntp[0] = 0u;
    }
    __syncthreads();
    if (s_merge) rg_merge(c, m, g, n, cur.sbase + g * cur.nseg, cur.nseg);
    cur = nxt;
    sidx++;
  }
  if (threadIdx.x == 0) s_rg_issued = 0;
  __syncthreads();
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
