// Attention over long caches (more than kAttnChunk positions), streamed in
// contiguous page ranges.  Included by decoder.cuh after the KV, RoPE,
// mbarrier and stage-ring helpers.
//
// Segments.  The np pages of a (sequence m, kv head g) pair split into
// segments of S = 2 ceil(np / 64) pages for np <= 64, S = 2 ceil(np / 32)
// pages above (rg_seg_pages), so a pair has at most kSegMax segments and a
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
// The block holding the last segment of (m, g) merges, once every segment
// has arrived, in segment order: head = (T + sum_k exp(m_k - M) o_k) / sum_k exp(m_k - M) l_k with
// M = max_k m_k (the reference's max over all n scores and its 1/sum).
//
// Chunk work (256 threads, each warp on its own).  Warp w takes the chunk's
// tokens 4w .. 4w+3 for all G query heads of the kv head, with the run's q in
// registers.  Scores: lanes 0-15 the first two tokens, lanes 16-31 the other
// two; lane slot s multiplies dims s + 16 j (j = 0..7) and sums them as
// ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)) (packed in pairs (p_j, p_j+4)); a
// reduce-scatter over the 16 slots (xor 8, 4, 2, 1) then leaves one
// (token, head) score per lane.  That is the reference's dotF32 order (16
// slot accumulators, the tree16 of the slots), so each score equals the
// single-item path's bit for bit.  The warp keeps its own running max, sum
// and o (lane dims 4 lane .. 4 lane + 3 of every head) over its tokens of the
// segment, so a chunk needs no block barrier; at the segment's end the
// warps' partials are combined in warp order through the buffer of the
// segment's last chunk.  A warp done with a buffer counts itself out; the
// last one issues the buffer's next chunk.

namespace ocrvl {

constexpr int kSegMax = 32;    // segments of one (sequence, kv head) pair at most
constexpr int kRangeBufs = 4;  // chunk buffers per block
constexpr int kRangeTok = 32;  // tokens per chunk (two KV pages)
static_assert(2 * kRangeTok * kHeadDim * 4 == kStageBytes, "a chunk's K and V fill one ring slot");
static_assert(kRangeBufs <= kStagesM1 - 1, "single-sequence layout: buffers in ring slots 1..");
static_assert(kMaxGroup == 8 && kHeadDim == 128, "score layout: 8 heads x 2 tokens per half-warp");
static_assert(kSegMax <= 32, "merge: one segment per lane");

// Small arrays of the range phase (floats from their base).
// rotated q by lane: [half-warp grp][head][2][slot][4]: for lane slot s, the
// dims (16 (j ^ grp) + s, +64) for j = 0, 1 then j = 2, 3
constexpr int kRgQs = 0;
constexpr int kRgPreLen = 8 * 128 + 128 + 128 + 64 + 64;  // raw q | new k | new v | cos | sin
constexpr int kRgPre = kRgQs + 2 * 8 * 128;               // two prefetch buffers
constexpr int kRgKnew = kRgPre + 2 * kRgPreLen;           // [128] rotated new k, [128] new v
constexpr int kRgWarps = kThreads / 32;                   // warps of the block
// per warp: weights [4 tokens][8 heads] as (w, w) pairs | rescale factors [8]
// as (a, a) pairs | raw weights [4 tokens][8 heads]
constexpr int kRgWpW = 0, kRgWpA = 64, kRgWpRaw = 80, kRgWpLen = 112;
constexpr int kRgWp = kRgKnew + 256;                      // [kRgWarps][kRgWpLen]
constexpr int kRgMl = kRgWp + kRgWarps * kRgWpLen;        // [kRgWarps][8 heads][2] running max, sum
constexpr int kRgMerges = 2 * kMaxSeqs;                   // pairs a block can complete in one phase
constexpr int kRgMerge = kRgMl + kRgWarps * 8 * 2;        // count, then [kRgMerges][2] pairs to merge (ints)
constexpr int kRgFloats = kRgMerge + 4 + 2 * kRgMerges;
static_assert(kRgFloats * 4 <= kStageBytes, "small arrays fit one ring slot");
static_assert(kRgPreLen % 4 == 0 && kRgPre % 4 == 0 && kRgWp % 4 == 0 && kRgWpLen % 4 == 0, "16-byte aligned arrays");
static_assert(kRgWarps * kMaxGroup * kHeadDim * 4 <= kStageBytes, "the warps' partials fit one chunk buffer");

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

// Pages per segment: up to 2 kSegMax pages, 2-page segments (at most kSegMax
// of them, for the parallelism of short steps); longer caches, whose pairs
// carry more chunks each, half as many segments (each segment's end costs a
// combine of the warps' partials and a partial for the merge).
__host__ __device__ __forceinline__ int rg_seg_pages(int np) {
  const int t = np <= 2 * kSegMax ? kSegMax : kSegMax / 2;  // target segments
  return 2 * ((np + 2 * t - 1) / (2 * t));
}

// Position in the step's stream of segments and chunks.
struct RgCur {
  int m;               // sequence, -1 past the last long cache
  int g, k, j;         // kv head, segment of (m, g), chunk of the segment
  int n, np, S, nseg;  // positions (incl. the new one), pages, pages per segment, segments
  int pbase, sbase;    // pages and segments of the long caches before m
};

// Geometry of the step's long caches, fixed for a launch (the sequences and
// their lengths do not change within it) and computed once at its start
// (rg_launch_init): per sequence its pages (0 for a cache of n <= kAttnChunk
// positions), pages per segment and segments; the prefix sums of pages and
// segments over the sequences before it (kv heads included); this block's
// first segment, the end of its page range and the pool pages of its range
// (block-table entries, s_rg_pg[i] for the block's page i); the sequences
// with caches of n <= kAttnChunk positions, in order.
constexpr int kRgPgCap = 512;  // pool pages of a block's range held in shared memory
__shared__ int s_rg_np[kMaxSeqs], s_rg_S[kMaxSeqs], s_rg_nseg[kMaxSeqs];
__shared__ int s_rg_pbase[kMaxSeqs + 1], s_rg_sbase[kMaxSeqs + 1];
__shared__ RgCur s_rg_first;
__shared__ int s_rg_hi, s_rg_p0, s_rg_npg;
__shared__ int s_rg_pg[kRgPgCap];
__shared__ int s_ex_n, s_ex_m[kMaxSeqs];
// The block's chunks in stream order (pool page of each of their one or two
// pages, -1 for none, and the kv head), when there are at most kRgChCap of
// them (s_rg_nch their count, -1 otherwise): a buffer refill then reads its
// chunk's copies from here instead of walking the cursor.
constexpr int kRgChCap = 256;
__shared__ int4 s_rg_ch[kRgChCap];
__shared__ int s_rg_nch;

// Moves to the first long cache at or after sequence m.
__device__ __forceinline__ void rg_load_seq(const StepParams &sp, RgCur &r, int m) {
  while (m < sp.M && s_rg_np[m] == 0) m++;
  r.g = r.k = r.j = 0;
  if (m >= sp.M) {
    r.m = -1;
    return;
  }
  r.m = m;
  r.n = sp.seq[m].len + 1;
  r.np = s_rg_np[m];
  r.S = s_rg_S[m];
  r.nseg = s_rg_nseg[m];
  r.pbase = s_rg_pbase[m];
  r.sbase = s_rg_sbase[m];
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
  rg_load_seq(sp, r, r.m + 1);
}

__device__ __forceinline__ void rg_next_chunk(const Ctx &c, const StepParams &sp, RgCur &r) {
  if (2 * (r.j + 1) < rg_seg_np(r)) {
    r.j++;
    return;
  }
  rg_next_seg(c, sp, r);
}

__device__ __forceinline__ int rg_bound(int P, int b, int nb) { return (int)(((long long)P * b + nb - 1) / nb); }

// Per-block state of the range loads, kept across the phases of a launch:
// s_rg_full[j] completes when buffer j's copies land, s_rg_par bit j is the
// parity of its next completion; s_rg_issued counts the chunks of the coming
// (or running) attention phase issued so far (chunk i into buffer
// i % kRangeBufs) and s_rg_icur is the next chunk to issue.
__shared__ __align__(8) uint64_t s_rg_full[kRangeBufs];
__shared__ __align__(8) uint64_t s_rg_mbar;  // merge copies
__shared__ uint32_t s_rg_par, s_rg_mpar;
__shared__ int s_rg_issued;
__shared__ RgCur s_rg_icur;
__shared__ unsigned s_rg_rel[kRangeBufs];  // warps done with each buffer's current chunk

__device__ __forceinline__ void rg_block_init() {
  if (threadIdx.x == 0) {
    for (int j = 0; j < kRangeBufs; j++) {
      mbar_init(&s_rg_full[j], 1);
      s_rg_rel[j] = 0;
    }
    mbar_init(&s_rg_mbar, 1);
    mbar_fence_init();
    s_rg_par = 0;
    s_rg_mpar = 0;
    s_rg_issued = 0;
  }
}

// Pool page of the block's range page o (global page order), from the table
// or the block table.
__device__ __forceinline__ int rg_pool_page(const StepParams &sp, const RgCur &r, int o) {
  const int i = o - s_rg_p0;
  if (i >= 0 && i < s_rg_npg) return s_rg_pg[i];
  return __ldg(sp.seq[r.m].bt + (o - r.pbase) % r.np);
}

// All threads, once per launch (after the step parameters are in shared
// memory and rg_block_init): the geometry tables, this block's range and its
// pool pages.  The block takes the segments whose first page lies in
// [ceil(P b / nb), ceil(P (b+1) / nb)).
__device__ void rg_launch_init(const Ctx &c) {
  const StepParams &sp = *c.sp;
  for (int m = threadIdx.x; m < sp.M; m += kThreads) {
    const int n = sp.seq[m].len + 1;
    const int np = n > kAttnChunk ? (n + kPageTokens - 1) / kPageTokens : 0;
    const int S = np ? rg_seg_pages(np) : 1;
    s_rg_np[m] = np;
    s_rg_S[m] = S;
    s_rg_nseg[m] = np ? (np + S - 1) / S : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int pb = 0, sb = 0, ne = 0, smax = 1;
    for (int m = 0; m < sp.M; m++) {
      s_rg_pbase[m] = pb;
      s_rg_sbase[m] = sb;
      pb += c.KVH * s_rg_np[m];
      sb += c.KVH * s_rg_nseg[m];
      smax = max(smax, s_rg_S[m]);
      if (s_rg_np[m] == 0) s_ex_m[ne++] = m;
    }
    s_ex_n = ne;
    s_rg_pbase[sp.M] = pb;
    s_rg_sbase[sp.M] = sb;
    const int lo = rg_bound(pb, blockIdx.x, gridDim.x);
    const int hi = rg_bound(pb, blockIdx.x + 1, gridDim.x);
    s_rg_hi = hi;
    // first segment starting at or after page lo
    RgCur r;
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
          break;
        }
      }
      rg_load_seq(sp, r, r.m + 1);
    }
    s_rg_first = r;
    s_rg_icur = r;
    // pages of the block's segments: from the first one's start to at most
    // the largest segment past the end of the range
    const int p0 = rg_in(r, hi) ? rg_start(r) : pb;
    s_rg_p0 = p0;
    s_rg_npg = min(kRgPgCap, max(0, min(pb, hi + smax) - p0));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < s_rg_npg; i += kThreads) {
    const int o = s_rg_p0 + i;
    int lo = 0, hi = sp.M - 1;  // last sequence with pbase <= o (binary search)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_rg_pbase[mid] <= o) lo = mid;
      else hi = mid - 1;
    }
    const int rem = o - s_rg_pbase[lo];
    const int p = rem % s_rg_np[lo];
    s_rg_pg[i] = __ldg(sp.seq[lo].bt + p);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    RgCur r = s_rg_first;
    int i = 0;
    for (; i < kRgChCap && rg_in(r, s_rg_hi); i++) {
      const int o = rg_start(r) + 2 * r.j;
      const bool two = rg_seg_np(r) - 2 * r.j >= 2;
      s_rg_ch[i] = make_int4(rg_pool_page(sp, r, o), two ? rg_pool_page(sp, r, o + 1) : -1, r.g, 0);
      rg_next_chunk(c, sp, r);
    }
    s_rg_nch = rg_in(r, s_rg_hi) ? -1 : i;
  }
}

// Per-block time stamp i (thread 0; the last layer's values remain):
// 0 phase entry, 1 long-cache part entry, 2 first copies issued, 3 first
// segment's rows landed, 4 q rotated, 5 first chunk landed, 6 its scores,
// 7 first segment's chunks done, 8 arrival counted, 9 phase done; 10-13 the
// second chunk: start, landed, scores, softmax; 14 chunks * 1000 + runs,
// 15 merges * 1000 + their segments.
__device__ __forceinline__ void rg_bmark(const Ctx &c, int i) {
  if (c.trace && threadIdx.x == 0) c.trace[4 * kTraceRows + kTraceMarks * blockIdx.x + i] = gtimer();
}

// K rows then V rows of (layer, kv head g) in pool page `page`: 16 KB.
__device__ __forceinline__ const float *rg_page_kv(const Ctx &c, int page, int layer, int g) {
  return c.kv_pool + (size_t)page * c.page_floats + ((size_t)layer * c.KVH + g) * 2 * kPageTokens * c.D;
}
// Pairs of floats in one 64-bit register pair and the sm_100 packed FP32
// operations on them (each half rounded to nearest even, as the scalar
// __fmul_rn / __fadd_rn / __fmaf_rn).
typedef unsigned long long f2x;
__device__ __forceinline__ f2x f2_pack(float a, float b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float f2_lo(f2x r) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
  return a;
}
__device__ __forceinline__ float f2_hi(f2x r) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
  return b;
}
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

// Row of position t (0..31) of a chunk buffer: page t / 16 of the chunk at
// 32 rows per page, K rows first.
__device__ __forceinline__ float *rg_row(float *buf, int t, int kind) {
  return buf + (size_t)(((t >> 4) * 2 + kind) * kPageTokens + (t & 15)) * kHeadDim;
}

// One thread: the copies of the chunk at cursor r (its one or two pages, K
// and V rows of each) into buffer b.
__device__ __forceinline__ void rg_issue_chunk(const Ctx &c, int layer, float *smem, const RgCur &r, int b) {
  const StepParams &sp = *c.sp;
  constexpr uint32_t pb = 2u * kPageTokens * kHeadDim * 4;  // K and V rows of one page
  float *buf = rg_buf(c, sp.M, smem, b);
  const int o = rg_start(r) + 2 * r.j;
  const bool two = rg_seg_np(r) - 2 * r.j >= 2;
  const int pg0 = rg_pool_page(sp, r, o);
  const int pg1 = two ? rg_pool_page(sp, r, o + 1) : 0;
  uint64_t *bar = &s_rg_full[b];
  mbar_expect_tx(bar, (two ? 2u : 1u) * pb);
  bulk_g2s(buf, rg_page_kv(c, pg0, layer, r.g), pb, bar);
  if (two) bulk_g2s(buf + 2 * kPageTokens * kHeadDim, rg_page_kv(c, pg1, layer, r.g), pb, bar);
}

// One thread: issues chunks while fewer than `upto` have been issued and the
// block's range has more (chunk i into buffer i % kRangeBufs).
__device__ void rg_issue_upto(const Ctx &c, int layer, float *smem, int upto) {
  const StepParams &sp = *c.sp;
  const int hi = s_rg_hi;
  RgCur r = s_rg_icur;
  int i = s_rg_issued;
  if (i >= upto || !rg_in(r, hi)) return;
  // before a phase's first copy: the buffers were last written by ordinary
  // stores in earlier phases (later, the threads that store into a buffer
  // fence their own stores; reads need no fence before a copy overwrites them)
  if (i == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  for (; i < upto && rg_in(r, hi); i++) {
    rg_issue_chunk(c, layer, smem, r, i % kRangeBufs);
    rg_next_chunk(c, sp, r);
  }
  s_rg_icur = r;
  s_rg_issued = i;
}

// One lane of each warp, once the warp is done with the buffer of chunk ci
// (cursor r): the last of the kRgWarps arrivals (atom.inc wraps the count
// back to 0) issues the chunk kRangeBufs later in the block's range into the
// same buffer.
__device__ __forceinline__ void rg_release(const Ctx &c, int layer, float *smem, RgCur r, int ci) {
  const int b = ci % kRangeBufs;
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.inc.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(smem_u32(&s_rg_rel[b])), "r"((unsigned)(kRgWarps - 1))
               : "memory");
  if (old != (unsigned)(kRgWarps - 1)) return;
  const int nch = s_rg_nch;
  if (nch >= 0) {
    const int i = ci + kRangeBufs;
    if (i >= nch) return;
    constexpr uint32_t pb = 2u * kPageTokens * kHeadDim * 4;  // K and V rows of one page
    const int4 d = s_rg_ch[i];
    float *buf = rg_buf(c, c.sp->M, smem, b);
    uint64_t *bar = &s_rg_full[b];
    mbar_expect_tx(bar, (d.y >= 0 ? 2u : 1u) * pb);
    bulk_g2s(buf, rg_page_kv(c, d.x, layer, d.z), pb, bar);
    if (d.y >= 0) bulk_g2s(buf + 2 * kPageTokens * kHeadDim, rg_page_kv(c, d.y, layer, d.z), pb, bar);
    return;
  }
  const StepParams &sp = *c.sp;
#pragma unroll 1
  for (int i = 0; i < kRangeBufs && r.m >= 0; i++) rg_next_chunk(c, sp, r);
  if (rg_in(r, s_rg_hi)) rg_issue_chunk(c, layer, smem, r, b);
}

// Waits for range copies issued ahead of a phase that did not run (thread 0).
__device__ __forceinline__ void rg_drain(const Ctx &c) {
  for (int j = 0; j < s_rg_issued && j < kRangeBufs; j++) {
    mbar_wait(&s_rg_full[j], (s_rg_par >> j) & 1u, c.err);
    s_rg_par ^= 1u << j;
  }
  s_rg_issued = 0;
  s_rg_icur = s_rg_first;
}


// All threads: cp.async copies of the raw q (G heads), new k and v of pair
// (r.m, r.g) and the cos / sin of the sequence's position.
__device__ __forceinline__ void rg_prefetch_run(const Ctx &c, const StepParams &sp, const RgCur &r, float *pre) {
  const int G = c.QH / c.KVH;
  const size_t qkvld = (size_t)(c.QH + 2 * c.KVH) * kHeadDim;
  const float *row = c.qkv + (size_t)r.m * qkvld;
  const int t = threadIdx.x;
  if (t < G * 32) cp_async16(pre + 4 * t, row + (size_t)r.g * G * kHeadDim + 4 * t);
  if (t < 64) {
    const int kind = t >> 5, i4 = t & 31;
    cp_async16(pre + 1024 + 128 * kind + 4 * i4, row + (size_t)(c.QH + kind * c.KVH + r.g) * kHeadDim + 4 * i4);
  }
  if (t >= 128 && t < 256 && !(s_rope_ready && r.m < kMaxBatch)) {
    const int i = (t - 128) & 63;
    const int p = sp.seq[r.m].pos[c.sec_axis[i]];
    const float *tab = t < 192 ? c.rope_cos : c.rope_sin;
    cp_async4(pre + 1280 + (t - 128), tab + (size_t)p * (kHeadDim / 2) + i);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// All threads of the block that merges pair (m, g): its segments'
// partials (o [nseg][G][128], maxima / sums [nseg][G][2], the tail sums
// [G][128]) arrive by bulk copies in `stage` (nseg * 4 KB <= 128 KB) and
// `aux`; warp h merges head h, lane dims 4 lane .. 4 lane + 3.
__device__ __forceinline__ void rg_merge(const Ctx &c, int m, int g, int n, int sb, int nseg, float *stage, float *aux) {
  const int G = c.QH / c.KVH;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t hq0 = (size_t)m * c.QH + (size_t)g * G;
  const bool tail = (n & 15) != 0;
  float *mls = aux, *ts = aux + 2 * kSegMax * kMaxGroup;  // [nseg][G][2], [G][128]
  if (threadIdx.x == 0) {
    // partials of other blocks (released with their arrival counts, which
    // this block acquired) are read through the async proxy
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const uint32_t ob = (uint32_t)(nseg * G * kHeadDim * 4), mb = (uint32_t)(nseg * G * 8),
                   tb = tail ? (uint32_t)(G * kHeadDim * 4) : 0u;
    mbar_expect_tx(&s_rg_mbar, ob + mb + tb);
    bulk_g2s(stage, c.part_o + (size_t)sb * G * kHeadDim, ob, &s_rg_mbar);
    bulk_g2s(mls, c.part_ml + (size_t)sb * G * 2, mb, &s_rg_mbar);
    if (tail) bulk_g2s(ts, c.part_t + hq0 * kHeadDim, tb, &s_rg_mbar);
  }
  mbar_wait(&s_rg_mbar, s_rg_mpar, c.err);
  if (h < G) {
    const float mk = lane < nseg ? mls[(lane * G + h) * 2] : -INFINITY;
    const float lk = lane < nseg ? mls[(lane * G + h) * 2 + 1] : 0.0f;
    float mx = mk;
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float sk = lane < nseg ? exp_fma(__fsub_rn(mk, mx)) : 0.0f;
    float den = __fmul_rn(sk, lk);
    for (int o = 16; o > 0; o >>= 1) den = __fadd_rn(den, __shfl_xor_sync(0xffffffffu, den, o));
    float4 acc = tail ? ((const float4 *)(ts + h * kHeadDim))[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int u = 0; u < nseg; u++) {
      const float s = __shfl_sync(0xffffffffu, sk, u);
      const float4 v = ((const float4 *)(stage + ((size_t)u * G + h) * kHeadDim))[lane];
      acc.x = __fmaf_rn(s, v.x, acc.x);
      acc.y = __fmaf_rn(s, v.y, acc.y);
      acc.z = __fmaf_rn(s, v.z, acc.z);
      acc.w = __fmaf_rn(s, v.w, acc.w);
    }
    const float di = __fdiv_rn(1.0f, den);
    ((float4 *)(c.head + (hq0 + h) * kHeadDim))[lane] =
        make_float4(__fmul_rn(acc.x, di), __fmul_rn(acc.y, di), __fmul_rn(acc.z, di), __fmul_rn(acc.w, di));
  }
  // the stage is free again once every warp has read it
  __syncthreads();
  if (threadIdx.x == 0) s_rg_mpar ^= 1u;
}

// Trace (OCRVL_TRACE): latest time over the blocks at which their first
// segment reached point i (0 q rotated, 1 chunks done, 2 arrival counted, 3
// phase done), in trace row 200 + layer.
__device__ __forceinline__ void rg_mark(const Ctx &c, int layer, int i) {
  if (c.trace && threadIdx.x == 0 && layer < 26) atomicMax(c.trace + 4 * (200 + layer) + i, gtimer());
}

// Attention of the step's long caches (see the top of this file).
__device__ __noinline__ void phase_attn_range(const Ctx *cp, int layer, float *smem) {
  const Ctx &c = *cp;
  const StepParams &sp = *c.sp;
  const int G = c.QH / c.KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = lane & 15, grp = lane >> 4;
  rg_bmark(c, 1);
  const int hi = s_rg_hi;
  float *sm = rg_small(c, sp.M, smem);
  float *qs = sm + kRgQs, *knew = sm + kRgKnew, *mlw = sm + kRgMl;
  float *wp = sm + kRgWp + warp * kRgWpLen;  // this warp's weights and rescale factors
  RgCur cur = s_rg_first;
  if (threadIdx.x == 0) ((int *)(sm + kRgMerge))[0] = 0;
  if (!rg_in(cur, hi)) return;
  if (threadIdx.x == 0) rg_issue_upto(c, layer, smem, kRangeBufs);
  const uint32_t par0 = s_rg_par;  // parity of each buffer's next completion
  rg_bmark(c, 2);
  rg_prefetch_run(c, sp, cur, sm + kRgPre);
  int ci = 0;    // chunk index in the block's stream
  int ridx = 0;  // run index in the block's stream
  while (rg_in(cur, hi)) {
    // ---- run start (the block's consecutive segments of one pair): rotated
    // q and new k from the prefetched rows
    const float *pre = sm + kRgPre + (ridx & 1) * kRgPreLen;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (ridx == 0) rg_bmark(c, 3);
    const int m = cur.m, g = cur.g, n = cur.n, len = n - 1, nv = n & ~15;
    // segments k0 .. k1-1 of the pair are this block's (first page < hi)
    const int k0 = cur.k;
    const int k1 = min(cur.nseg, (hi - cur.pbase - g * cur.np + cur.S - 1) / cur.S);
    {
      const int *pos = sp.seq[m].pos;
      const bool has_rope = pos[0] != 0 || pos[1] != 0 || pos[2] != 0;
      const bool tab = s_rope_ready && m < kMaxBatch;  // the launch's RoPE tables hold sequence m
      const float *rc = tab ? s_rope_cs[m] : pre + 1280, *rs = tab ? s_rope_sn[m] : pre + 1344;
      for (int p = threadIdx.x; p < G * 16 + 48; p += kThreads) {
        if (p < G * 16) {
          const int hh = p >> 4, i4 = p & 15;
          float4 a = ((const float4 *)(pre + hh * kHeadDim))[i4], b = ((const float4 *)(pre + hh * kHeadDim + 64))[i4];
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
          float4 a = ((const float4 *)(pre + 1024))[i4], b = ((const float4 *)(pre + 1024 + 64))[i4];
          if (has_rope) rope4(a, b, rc + 4 * i4, rs + 4 * i4);
          ((float4 *)knew)[i4] = a;
          ((float4 *)knew)[i4 + 16] = b;
        } else {
          const int i4 = p - G * 16 - 16;
          ((float4 *)(knew + 128))[i4] = ((const float4 *)(pre + 1152))[i4];
        }
      }
    }
    __syncthreads();
    if (ridx == 0) {
      rg_mark(c, layer, 0);
      rg_bmark(c, 4);
    }
    // this lane's q pairs of head h: qlane[2 h], qlane[2 h + 1]
    const ulonglong2 *qlane = (const ulonglong2 *)qs + (grp * 8 * 2) * 16 + slot;
    RgCur nxt = cur;  // the next run: the first segment after this run
    nxt.k = k1 - 1;
    rg_next_seg(c, sp, nxt);
    if (rg_in(nxt, hi)) rg_prefetch_run(c, sp, nxt, sm + kRgPre + ((ridx + 1) & 1) * kRgPreLen);
#pragma unroll 1
    for (int k = k0; k < k1; k++) {
      cur.k = k;
      // warp state over its tokens of the segment: running max and sum of
      // head (lane & 7); o of head h at dims (4 lane, +1), (4 lane + 2, +3)
      float m_run = -INFINITY, l_run = 0.0f;
      f2x o2[8][2];
#pragma unroll
      for (int h = 0; h < 8; h++) o2[h][0] = o2[h][1] = 0ull;
      const int seg_np = rg_seg_np(cur);
      const int nck = (seg_np + 1) / 2;
      const int sp0 = k * cur.S;  // first page of the segment
#pragma unroll 1
      for (int j = 0; j < nck; j++, ci++) {
        cur.j = j;
        const int b = ci % kRangeBufs;
        float *Kb = rg_buf(c, sp.M, smem, b);  // rows by rg_row
        const int t0 = (sp0 + 2 * j) * kPageTokens;
        const int cnt = min(min(2, seg_np - 2 * j) * kPageTokens, n - t0);
        mbar_wait(&s_rg_full[b], ((par0 >> b) ^ (uint32_t)(ci / kRangeBufs)) & 1u, c.err);
        if (ci == 0) rg_bmark(c, 5);
        // ---- scores of the warp's tokens 4 warp .. 4 warp + 3: half grp
        // takes tokens 4 warp + 2 grp + {0, 1}; the reduce-scatter over the
        // 16 slots leaves (token lane >> 3, head lane & 7) on each lane
        float v[16];
        {
          f2x kp[2][4];  // K of token (4 warp + 2 grp + tl) at dims (16 (j ^ grp) + slot, +64)
#pragma unroll
          for (int tl = 0; tl < 2; tl++) {
            const int tok = 4 * warp + 2 * grp + tl;
            const float *kr = t0 + tok == len ? knew : rg_row(Kb, tok, 0);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
              const int idx = 16 * (jj ^ grp) + slot;
              kp[tl][jj] = f2_pack(kr[idx], kr[idx + 64]);
            }
          }
#pragma unroll
          for (int h = 0; h < 8; h++) {
            const ulonglong2 qa = qlane[(2 * h) * 16], qb = qlane[(2 * h + 1) * 16];
#pragma unroll
            for (int tl = 0; tl < 2; tl++) {
              // (p_j, p_j+4) pairs: ((p0+p1)+(p2+p3)) + ((p4+p5)+(p6+p7))
              const f2x z = f2_add(f2_add(f2_mul(qa.x, kp[tl][0]), f2_mul(qa.y, kp[tl][1])),
                                   f2_add(f2_mul(qb.x, kp[tl][2]), f2_mul(qb.y, kp[tl][3])));
              v[tl * 8 + h] = h < G ? __fadd_rn(f2_lo(z), f2_hi(z)) : 0.0f;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const bool up = lane & 8;
          const float send = up ? v[i] : v[8 + i];
          v[i] = __fadd_rn(up ? v[8 + i] : v[i], __shfl_xor_sync(0xffffffffu, send, 8));
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const bool up = lane & 4;
          const float send = up ? v[i] : v[4 + i];
          v[i] = __fadd_rn(up ? v[4 + i] : v[i], __shfl_xor_sync(0xffffffffu, send, 4));
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
          const bool up = lane & 2;
          const float send = up ? v[i] : v[2 + i];
          v[i] = __fadd_rn(up ? v[2 + i] : v[i], __shfl_xor_sync(0xffffffffu, send, 2));
        }
        float s;
        {
          const bool up = lane & 1;
          const float send = up ? v[0] : v[1];
          s = __fmul_rn(__fadd_rn(up ? v[1] : v[0], __shfl_xor_sync(0xffffffffu, send, 1)), c.attn_scale);
        }
        if (ci == 0) rg_bmark(c, 6);
        // ---- online softmax of the warp's tokens: head h on lanes h, h+8,
        // h+16, h+24 (its four tokens)
        const int tok = 4 * warp + (lane >> 3);
        const bool valid = tok < cnt, raw = t0 + tok >= nv;
        float pm = valid ? s : -INFINITY;
        pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
        pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 16));
        const float m_new = fmaxf(m_run, pm);
        const float alpha = m_run == -INFINITY ? 0.0f : exp_fma(__fsub_rn(m_run, m_new));
        float e = 0.0f;
        if (valid) e = raw ? s : exp_fma(__fsub_rn(s, m_new));
        float le = valid && !raw ? e : 0.0f;
        le = __fadd_rn(le, __shfl_xor_sync(0xffffffffu, le, 8));
        le = __fadd_rn(le, __shfl_xor_sync(0xffffffffu, le, 16));
        l_run = __fadd_rn(__fmul_rn(l_run, alpha), le);
        m_run = m_new;
        {
          const float w = valid && !raw ? e : 0.0f;
          ((float2 *)(wp + kRgWpW))[lane] = make_float2(w, w);
        }
        if (lane < 8) ((float2 *)(wp + kRgWpA))[lane] = make_float2(alpha, alpha);
        if (t0 + cnt > nv) wp[kRgWpRaw + lane] = valid && raw ? e : 0.0f;  // raw weights, for the tail sums
        const bool rescale = !__all_sync(0xffffffffu, alpha == 1.0f);
        __syncwarp();
        // ---- values: lane dims 4 lane .. 4 lane + 3 of the G heads
        if (rescale) {
#pragma unroll
          for (int h2 = 0; h2 < 4; h2++) {
            const ulonglong2 a = ((const ulonglong2 *)(wp + kRgWpA))[h2];
            o2[2 * h2][0] = f2_mul(o2[2 * h2][0], a.x);
            o2[2 * h2][1] = f2_mul(o2[2 * h2][1], a.x);
            o2[2 * h2 + 1][0] = f2_mul(o2[2 * h2 + 1][0], a.y);
            o2[2 * h2 + 1][1] = f2_mul(o2[2 * h2 + 1][1], a.y);
          }
        }
        const int nvw = min(4, cnt - 4 * warp);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          if (i < nvw) {
            const int tk = 4 * warp + i;
            const float *vr = t0 + tk == len ? knew + kHeadDim : rg_row(Kb, tk, 1);
            const ulonglong2 vq = ((const ulonglong2 *)vr)[lane];
#pragma unroll
            for (int h2 = 0; h2 < 4; h2++) {
              const ulonglong2 w = ((const ulonglong2 *)(wp + kRgWpW + 16 * i))[h2];
              o2[2 * h2][0] = f2_fma(w.x, vq.x, o2[2 * h2][0]);
              o2[2 * h2][1] = f2_fma(w.x, vq.y, o2[2 * h2][1]);
              o2[2 * h2 + 1][0] = f2_fma(w.y, vq.x, o2[2 * h2 + 1][0]);
              o2[2 * h2 + 1][1] = f2_fma(w.y, vq.y, o2[2 * h2 + 1][1]);
            }
          }
        }
        if (t0 <= len && len < t0 + cnt && ((len - t0) >> 2) == warp) {
          // the new token: appended to the cache (kvCache.append,
          // internal/model/model.go:5593-5612)
          ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, 0, g, len))[lane] = ((const float4 *)knew)[lane];
          ((float4 *)kv_ptr(c, sp.seq[m].bt, layer, 1, g, len))[lane] = ((const float4 *)(knew + kHeadDim))[lane];
        }
        __syncwarp();
        // the warp is done with the chunk's rows (the segment's last chunk
        // after the partials below)
        if (j + 1 < nck && lane == 0) rg_release(c, layer, smem, cur, ci);
      }
      // ---- segment end: the warps' partials combined through the buffer of
      // the segment's last chunk
      if (ridx == 0 && k == k0) {
        rg_mark(c, layer, 1);
        rg_bmark(c, 7);
      }
      const int cl = ci - 1;
      float *Kb = rg_buf(c, sp.M, smem, cl % kRangeBufs);
      const int t0 = (sp0 + 2 * (nck - 1)) * kPageTokens;
      const int cnt = min(min(2, seg_np - 2 * (nck - 1)) * kPageTokens, n - t0);
      const int seg = rg_seg_index(cur);
      const size_t hq0 = (size_t)m * c.QH + (size_t)g * G;
      __syncthreads();  // every warp is past the chunk's rows
      if (t0 + cnt > nv) {
        // the pair's last chunk holds the positions at or above nv: warp h
        // sums head h's raw-weighted rows in position order
        if (warp < G) {
          float4 ta = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
          for (int t = max(nv - t0, 0); t < cnt; t++) {
            const float w = sm[kRgWp + (t >> 2) * kRgWpLen + kRgWpRaw + (t & 3) * 8 + warp];
            const float *vr = t0 + t == len ? knew + kHeadDim : rg_row(Kb, t, 1);
            const float4 vv = ((const float4 *)vr)[lane];
            ta.x = __fmaf_rn(w, vv.x, ta.x);
            ta.y = __fmaf_rn(w, vv.y, ta.y);
            ta.z = __fmaf_rn(w, vv.z, ta.z);
            ta.w = __fmaf_rn(w, vv.w, ta.w);
          }
          ((float4 *)(c.part_t + (hq0 + warp) * kHeadDim))[lane] = ta;
        }
        __syncthreads();  // the rows are read before the partials overwrite them
      }
      {
        ulonglong2 *cb = (ulonglong2 *)(Kb + (size_t)warp * kMaxGroup * kHeadDim);  // [warp][head][128]
#pragma unroll
        for (int h = 0; h < 8; h++) cb[h * (kHeadDim / 4) + lane] = make_ulonglong2(o2[h][0], o2[h][1]);
        if (lane < 8) ((float2 *)mlw)[warp * 8 + lane] = make_float2(m_run, l_run);
        // the buffer's next copy (async proxy) follows these stores
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncthreads();
      if (warp < G) {
        // head h = warp: M = max over the warps, o and l summed over the
        // warps in order, each scaled by exp(m_w - M)
        const int h = warp;
        const float2 ml = lane < 8 ? ((const float2 *)mlw)[lane * 8 + h] : make_float2(-INFINITY, 0.0f);
        float mx = ml.x;
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float sc = lane < 8 && ml.x != -INFINITY ? exp_fma(__fsub_rn(ml.x, mx)) : 0.0f;
        float l = __fmul_rn(sc, ml.y);
        l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, 1));
        l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, 2));
        l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, 4));
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kRgWarps; w++) {
          const float sw = __shfl_sync(0xffffffffu, sc, w);
          const float4 ov = ((const float4 *)(Kb + (size_t)(w * kMaxGroup + h) * kHeadDim))[lane];
          acc.x = __fmaf_rn(sw, ov.x, acc.x);
          acc.y = __fmaf_rn(sw, ov.y, acc.y);
          acc.z = __fmaf_rn(sw, ov.z, acc.z);
          acc.w = __fmaf_rn(sw, ov.w, acc.w);
        }
        ((float4 *)(c.part_o + ((size_t)seg * G + h) * kHeadDim))[lane] = acc;
        if (lane == 0) ((float2 *)c.part_ml)[(size_t)seg * G + h] = make_float2(mx, l);
      }
      __syncwarp();
      if (lane == 0) rg_release(c, layer, smem, cur, cl);
    }
    // ---- run end: arrival of the run's segments (no reply awaited); the
    // block holding the pair's last segment merges it after its range work.
    // The merger reads the partials with bulk copies (async proxy).
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      // release: the block's partials (ordered before by the barrier) become
      // visible with the count
      unsigned *cntp = c.attn_count + 2 * (m * c.KVH + g);
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(cntp), "r"(k1 - k0) : "memory");
      if (k1 == cur.nseg) {
        // merged after the phase (rg_merge_pending); a step has at most
        // kRgMerges (sequence, kv head) pairs (checked on the host)
        int *mlist = (int *)(sm + kRgMerge);
        const int q = mlist[0];
        mlist[4 + 2 * q] = m | g << 8 | cur.nseg << 16;
        mlist[4 + 2 * q + 1] = cur.sbase + g * cur.nseg;
        mlist[0] = q + 1;
        if (c.trace) c.trace[4 * kTraceRows + kTraceMarks * blockIdx.x + 15] += 1000 + cur.nseg;
      }
    }
    if (ridx == 0) {
      rg_mark(c, layer, 2);
      rg_bmark(c, 8);
    }
    cur = nxt;
    ridx++;
  }
  if (threadIdx.x == 0) {
    // chunk i completed a phase of buffer i % kRangeBufs
    for (int b = 0; b < kRangeBufs; b++)
      if (ci > b && (((ci - 1 - b) / kRangeBufs) & 1) == 0) s_rg_par ^= 1u << b;
    s_rg_issued = 0;
    s_rg_icur = s_rg_first;
  }
  __syncthreads();
  rg_mark(c, layer, 3);
  rg_bmark(c, 9);
  if (c.trace && threadIdx.x == 0) c.trace[4 * kTraceRows + kTraceMarks * blockIdx.x + 14] = (unsigned long long)ci * 1000 + ridx;
}

// All threads, after phase_attn_range: the merges of the pairs whose last
// segment this block holds, staged through the chunk buffers (contiguous: ring slots
// 1 .. kRangeBufs for single-sequence steps, the first kRangeBufs slots
// otherwise) and the small arrays before the list.
__device__ __noinline__ void rg_merge_pending(const Ctx *cp, float *smem) {
  const Ctx &c = *cp;
  const StepParams &sp = *c.sp;
  float *sm = rg_small(c, sp.M, smem);
  const int *ml = (const int *)(sm + kRgMerge);
  float *stage = rg_buf(c, sp.M, smem, sp.M <= 1 ? kRangeBufs - 1 : 0);
  __shared__ int s_ok;
  const int q = ml[0];
  for (int i = 0; i < q; i++) {
    const int a = ml[4 + 2 * i], sb = ml[4 + 2 * i + 1];
    const int m = a & 255, g = (a >> 8) & 255, nseg = a >> 16;
    if (threadIdx.x == 0) {
      // every segment of the pair has arrived (bounded wait: every block
      // posts all its arrivals before it waits for any)
      unsigned *cntp = c.attn_count + 2 * (m * c.KVH + g);
      long long spins = 0;
      int ok = 1;
      while (true) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cntp) : "memory");
        if ((int)v >= nseg) break;
        if (++spins > kMbarSpins || *(volatile int *)c.err) {
          atomicExch(c.err, 1);
          ok = 0;
          break;
        }
      }
      if (ok) cntp[0] = 0u;  // for the next layer (its arrivals follow a grid barrier)
      s_ok = ok;
    }
    __syncthreads();
    if (s_ok) rg_merge(c, m, g, sp.seq[m].len + 1, sb, nseg, stage, sm);
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
