// Batched decode step (more than kMaxBatch sequences, Q4 / Q6 weights): the
// projections run as int8 GEMMs on the 5th-generation tensor cores.
//
// The reference's int8-activation numerics (quantizeXForVNNI + finalizeDotQ8
// VNNI, internal/tensor/quant.go:2087-2115, dot_vnni_amd64.s:434-500,
// 1043-1090) are exact integer dots, so they map onto tcgen05.mma kind::i8
// with A = activations (uint8, one row per sequence, M = 64) and B = weights
// (signed int8, one row per output row): D = sum_k xq[m][k] * q[row][k] in
// int32, then (float(D) - 128 * float(rowsum)) * sx[m] * scale[row] as the
// reference (and the single-sequence kernels) compute it.  The results are
// bit-identical to the per-sequence path.
//
// Per layer the batched step runs nine phases, each followed by a grid
// barrier: input quantisation (one block per sequence: the RMSNorm or fused
// AddRMSNorm in the reference order, the activation scale and the uint8
// activations, written to a global "activation image" laid out as the MMA's
// A operand) and the GEMM, for QKV, o, gate/up and down, with the attention
// phase between QKV and o.
//
// GEMM phase, per block (its slab of output rows, in N tiles of <= 256):
//   for each K tile of kKT = 128 activations:
//     A tile  (64 rows x 128 bytes, 8 KB): one bulk copy of the activation image
//     B tile  (N rows x packed bytes): one 2-D TMA copy of the packed weight
//             rows, unpacked by all threads to int8 in the K-major core-matrix
//             layout (8 rows x 16 bytes contiguous; 8-row groups 1 KB apart)
//     4 MMAs (K = 32 bytes each) issued by one thread into TMEM
//   through a ring of up to kGemmStages stages of u K tiles (u A tiles in one
//   bulk copy, the packed B rows of u tiles in one 2-D box), as many as the
//   shared memory holds, issued ahead so later copies overlap the unpacking
//   and the tensor core's work; per stage all threads unpack its u tiles into
//   one of two groups of int8 buffers, one barrier, and one thread issues
//   its 4u MMAs and commits them to mbarriers that free the group and the
//   stage.  The epilogue reads D with tcgen05.ld
//   (M = 64 puts sequence r in TMEM lane 32*(r/16) + r%16) and applies the
//   same finalize and epilogue (store, residual, SwiGLU, argmax) as the
//   single-sequence kernels.
#pragma once

namespace ocrvl {

constexpr int kKT = 128;          // activations (int8 columns) per K tile
constexpr int kMmaM = 64;         // A rows (sequences) per MMA
constexpr int kMaxNT = 256;       // output rows per N tile
constexpr int kTmemCols = 512;    // TMEM columns a block allocates


struct BatchedW {
  const TmapBytes *tm;  // [L * 5 + 1]: per layer qkv, o, gate, up, down; then lm_head
  uint8_t *act;         // activation image [K tiles][64 rows][kKT]
  float *act_sx;        // [kMaxSeqs] activation scale per sequence
  int32_t *part;        // split-K partial dots of the o / down projection [ks][64][H]
  int smem_avail;       // dynamic shared memory of the step kernel (bytes, after alignment)
};

// Split-K of the residual projections (o and down, whose few output rows per
// CTA would otherwise make K/32 MMAs of N = 16 per CTA): ks groups of CTAs
// each take 1/ks of the K tiles of a slab of rows
// over gridDim.x / ks slabs, so a CTA issues ks times fewer MMAs of a wider N
// tile; the int32 partial dots add exactly and a finalize phase applies the
// epilogue.  At most kDownSplits groups, at least one K tile each.
constexpr int kDownSplits = 6;
__host__ __device__ __forceinline__ int down_splits(int K) {
  const int nk = K / kKT;
  return nk < kDownSplits ? (nk > 0 ? nk : 1) : kDownSplits;
}

__device__ __forceinline__ const TmapBytes *bw_map(const BatchedW &bw, int layer, int which) {
  return bw.tm + (size_t)layer * 5 + which;
}

// ---- tcgen05 helpers -------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols));
}
// One lane of the (converged) warp: the issuing lane for tcgen05 / TMA
// instructions whose operands the whole warp computed (warp-uniform values).
__device__ __forceinline__ bool elect_one_sync() {
  uint32_t p;
  asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}\n" : "=r"(p));
  return p != 0;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of
// 8 rows x 16 bytes, LBO = distance of the two 16-byte K halves (128 B),
// SBO = distance of 8-row groups (kKT * 8 = 1 KB).
__device__ __forceinline__ uint64_t umma_desc(const void *p) {
  const uint64_t a = smem_u32(p);
  uint64_t d = (a >> 4) & 0x3FFFull;
  d |= (uint64_t)((128u >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(((uint32_t)kKT * 8u >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version (sm100)
  return d;
}
// Instruction descriptor: D s32, A uint8, B int8, both K-major, M = 64.
__device__ __forceinline__ uint32_t umma_idesc_i8(int n) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kMmaM >> 4) << 24);
}
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 consecutive columns of this warp's TMEM lane quarter; the caller waits
// with tmem_wait_ld before using the values.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Offset of (row r, byte k) in a K-major core-matrix tile of kKT bytes per row.
__host__ __device__ __forceinline__ int cm_off(int r, int k) {
  return (r & 7) * 16 + (r >> 3) * (kKT * 8) + (k >> 4) * 128 + (k & 15);
}

// ---- quantisation phase ------------------------------------------------------
// One block per sequence: norm (mode) + int8 activations of src[m] (n values),
// written to the activation image row m, scale to act_sx[m].  copy_to: layer
// 0's gathered embedding row becomes the residual.
__device__ __noinline__ void phase_quant_b(const Ctx *cp, const BatchedW *bwp, const float *src, int ld, int src_tok,
                                           int n, int mode, const float *norm_w, float *copy_to, float *smem) {
  const Ctx &c = *cp;
  const BatchedW &bw = *bwp;
  const int M = c.sp->M;
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    const float *s = src + (size_t)(src_tok ? c.sp->seq[m].tok : m) * ld;
    // natural column order (the Q6 layout of the prologue)
    const float sx = xs_prologue(QT_Q6, s, n, mode, norm_w, true, c.eps, smem);
    const uint8_t *q = (const uint8_t *)(smem + 320 + n);
    for (int ch = threadIdx.x; ch < n / 16; ch += kThreads) {
      const int k = ch * 16;
      uint8_t *dst = bw.act + (size_t)(k / kKT) * (kMmaM * kKT) + cm_off(m, k % kKT);
      *(uint4 *)dst = *(const uint4 *)(q + k);
    }
    if (threadIdx.x == 0) bw.act_sx[m] = sx;
    if (copy_to)
      for (int i = threadIdx.x; i < ld / 4; i += kThreads)
        ((float4 *)(copy_to + (size_t)m * ld))[i] = __ldg((const float4 *)s + i);
    __syncthreads();
  }
  // the image is read next by bulk copies (async proxy) in other blocks
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- GEMM phase --------------------------------------------------------------
struct GemmArgs {
  const TmapBytes *mapA, *mapB;  // weight maps (mapB: SwiGLU up matrix)
  DMat A, B;
  int row_begin, row_end, K;     // output rows, input columns
  int nt;                        // rows per N tile = the maps' box height (multiple of 16, <= 256)
  int u;                         // K tiles per copy (gemm_u): the maps' box width is u packed K tiles
  int epi;                       // EPI_*
  float *out;
  int ldo;
  float *resid, *vout;
  int resid_mode;
  unsigned long long *argkey;
  float *logits;
  int argmax_finish, feed;
  int ks;                        // > 1: split-K groups (raw int32 dots to `part`, no epilogue)
  int32_t *part;                 // [ks][64][ldo]
};

// K tiles per copy: N tiles of up to 64 rows move u K tiles per copy (one
// 2-D TMA box of u * KP <= 256 bytes x nt rows, and one bulk copy of u A
// tiles), so a phase issues few, large copies; wider N tiles (lm_head) one.
__host__ __device__ __forceinline__ int gemm_u(int qt, int nt) {
  return nt <= 64 ? (qt == QT_Q4 ? 4 : 2) : 1;
}

// shared-memory layout of the GEMM phase (bytes from the base):
//   row scales [2][kMaxNT] f32 | row sums [2][kMaxNT] i32              4 KB
//   unpacked B tiles [2 groups][u][mats][nt][kKT] int8 (core-matrix layout)
//   stages [S]: u A tiles (u * kGemmA) | packed rows [mats][nt][u * KP]
//   (1 KB aligned)
// S fills the rest (at most kGemmStages, at most the stages of K).
constexpr int kGemmA = kMmaM * kKT;  // 8 KB per A tile
constexpr int kGemmStages = 8;       // ring stages at most
constexpr int kGemmScl = 4 * kMaxNT * 4;
// Least shared memory the phase needs (two stages of the largest tile).
__host__ __device__ __forceinline__ size_t gemm_b_smem_bytes() {
  return (size_t)kGemmScl + 2 * (size_t)kMaxNT * kKT + 2 * ((size_t)kGemmA + (size_t)kMaxNT * kKT * 3 / 4);
}

template <int QT>
__device__ __noinline__ void phase_gemm_b(const Ctx *cp, const BatchedW *bwp, const GemmArgs *gp, uint32_t tmem,
                                          float *smem) {
  const Ctx &c = *cp;
  const BatchedW &bw = *bwp;
  const GemmArgs &a = *gp;
  constexpr int KP = QT == QT_Q4 ? kKT / 2 : kKT * 3 / 4;  // packed bytes per row per K tile
  const bool two = a.epi == EPI_SWIGLU;
  const int mats = two ? 2 : 1;
  const int M = c.sp->M;
  const int NT = a.nt, U = a.u;
  uint8_t *base = (uint8_t *)smem;
  float *s_scl = (float *)base;  // [2][kMaxNT] scales, [2][kMaxNT] row sums
  int32_t *s_rs = (int32_t *)(s_scl + 2 * kMaxNT);
  uint8_t *sB0 = base + kGemmScl;                        // [2][U][mats][NT][kKT]
  const int sbytes = NT * kKT;                           // one unpacked tile of one matrix
  const int gbytes = U * mats * sbytes;                  // one group
  uint8_t *stg = sB0 + 2 * (size_t)gbytes;               // stages
  const int rowb = U * KP;                               // packed bytes per row per stage
  const int stage_bytes = (U * kGemmA + mats * NT * rowb + 1023) / 1024 * 1024;
  // split-K: CTA b takes K tiles [kt0, kt0 + nk) of slab b / ks (of
  // gridDim.x / ks slabs); otherwise every K tile of slab b
  const int ks = a.ks > 1 ? a.ks : 1, kg = blockIdx.x % ks, nslab = gridDim.x / ks;
  const int kt0 = kg * (a.K / kKT) / ks;
  const int nk = (kg + 1) * (a.K / kKT) / ks - kt0, nsu = (nk + U - 1) / U;
  int S = (bw.smem_avail - (int)(stg - base)) / stage_bytes;
  S = min(min(S, kGemmStages), max(nsu, 2));
  __shared__ __align__(8) uint64_t bar_ld[kGemmStages], bar_su[kGemmStages], bar_grp[2];
  if (S < 2) {  // the host sizes the shared memory for two stages of the largest tile
    if (threadIdx.x == 0) atomicExch(c.err, 1);
    return;
  }
  int lo, hi;
  if ((int)blockIdx.x / ks < nslab) gemv_slab(a.row_begin, a.row_end, blockIdx.x / ks, nslab, lo, hi);
  else lo = hi = a.row_end;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemmStages; i++) {
      mbar_init(&bar_ld[i], 1);
      mbar_init(&bar_su[i], 1);
    }
    for (int i = 0; i < 2; i++) mbar_init(&bar_grp[i], 1);
    mbar_fence_init();
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long best = 0ull;  // ARGMAX: lane's sequence best key
  // trace: per-block time stamps of the o projection (16 start, 17 first
  // copies issued, 18 first stage's MMAs issued, 23 end)
  const bool mk = a.epi == EPI_RESID && a.resid_mode == RESID_ATTN;
  if (mk) rg_bmark(c, 16);
  // stage TU of the phase (over all N tiles) uses slot TU % S (bar_ld and
  // bar_su complete once per use, use TU / S) and unpacked group TU & 1
  // (bar_grp[TU & 1] completes when the stage's MMAs are done, completion
  // TU >> 1)
  int TU0 = 0;
  for (int n0 = lo; n0 < hi; n0 += NT, TU0 += nsu) {
    const int nrows = min(NT, hi - n0);
    auto issue = [&](int su) {  // thread 0: copies of stage su (K tiles su*U ..)
      const int slot = (TU0 + su) % S;
      uint8_t *sa = stg + (size_t)slot * stage_bytes;
      const uint32_t bytes_a = (uint32_t)min(U, nk - su * U) * kGemmA;
      const uint32_t bytes_b = (uint32_t)NT * rowb;  // the whole box (past the matrix: zero-filled)
      mbar_expect_tx(&bar_ld[slot], bytes_a + mats * bytes_b);
      bulk_g2s(sa, bw.act + (size_t)(kt0 + su * U) * kGemmA, bytes_a, &bar_ld[slot]);
      tma_2d(sa + U * kGemmA, a.mapA, kt0 * KP + su * rowb, n0, &bar_ld[slot]);
      if (two) tma_2d(sa + U * kGemmA + bytes_b, a.mapB, kt0 * KP + su * rowb, n0, &bar_ld[slot]);
    };
    // the first stages' copies first: the scales below are read only by the
    // epilogue, so their load latency overlaps the copies and the MMAs
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int su = 0; su < nsu && su < S; su++) issue(su);
    }
    // scales / row sums of this N tile
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      s_scl[i] = __ldg(a.A.scale + n0 + i);
      s_rs[i] = __ldg(a.A.rowsum + n0 + i);
      // argmax: 128 * rowsum of vnni_finalize, once per column (the B half is unused)
      if (a.epi == EPI_ARGMAX) s_scl[kMaxNT + i] = __fmul_rn(128.0f, (float)s_rs[i]);
      if (two) {
        s_scl[kMaxNT + i] = __ldg(a.B.scale + n0 + i);
        s_rs[kMaxNT + i] = __ldg(a.B.rowsum + n0 + i);
      }
    }
    if (mk && n0 == lo) rg_bmark(c, 17);
    const uint32_t idesc = umma_idesc_i8(NT);
    // unpack tasks: CPR packed chunks per row, per = NT * CPR tasks per (tile, matrix)
    constexpr int CPR = QT == QT_Q4 ? KP / 16 : KP / 48;
    const int per = NT * CPR;
    const int jm0 = threadIdx.x / per, rc0 = threadIdx.x - jm0 * per;
    const int djm = kThreads / per, drc = kThreads - djm * per;
    for (int su = 0; su < nsu; su++) {
      const int TU = TU0 + su, slot = TU % S, grp = TU & 1;
      const int nt_here = min(U, nk - su * U);  // K tiles of this stage
      const uint8_t *sa = stg + (size_t)slot * stage_bytes;
      uint8_t *sg = sB0 + (size_t)grp * gbytes;
      const bool ms = mk && n0 == lo && su == 2;
      if (ms) rg_bmark(c, 19);
      mbar_wait(&bar_ld[slot], (uint32_t)(TU / S) & 1u, c.err);
      // the group's previous MMAs (stage TU - 2) are done before it is rewritten
      if (su >= 2) mbar_wait(&bar_grp[grp], (uint32_t)((TU >> 1) - 1) & 1u, c.err);
      if (ms) rg_bmark(c, 20);
      // unpack the stage's K tiles to int8 in the core-matrix layout:
      // tile j of matrix mi into sg + (j * mats + mi) * sbytes
      // task t = (tile j, matrix mi, row r, chunk) in that order; the
      // thread's (jm = j * mats + mi, rc = row * CPR + chunk) advance by
      // kThreads tasks a step without divisions
      int jm = jm0, rc = rc0;
      if (QT == QT_Q4) {
        // 16 packed bytes -> 32 int8 = two 16-byte K chunks
        for (int task = threadIdx.x; task < nt_here * mats * per; task += kThreads) {
          const int j = mats == 2 ? jm >> 1 : jm, mi = mats == 2 ? jm & 1 : 0;
          const int r = rc / CPR, c4 = rc % CPR;
          const uint8_t *pk_src = sa + U * kGemmA + (size_t)mi * NT * rowb + (size_t)j * KP;
          uint8_t *dstB = sg + (size_t)(j * mats + mi) * sbytes;
          uint4 pk = make_uint4(0, 0, 0, 0);
          if (r < nrows) pk = *(const uint4 *)(pk_src + (size_t)r * rowb + 16 * c4);
          const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
          uint32_t o[8];
#pragma unroll
          for (int jq = 0; jq < 4; jq++) {
            const uint32_t lo4 = w4[jq] & 0x0F0F0F0Fu, hi4 = (w4[jq] >> 4) & 0x0F0F0F0Fu;
            // bytes b0..b3 -> (lo0, hi0, lo1, hi1), (lo2, hi2, lo3, hi3); nibble - 8
            const uint32_t x0 = __byte_perm(lo4, hi4, 0x5140), x1 = __byte_perm(lo4, hi4, 0x7362);
            o[2 * jq] = __vsub4(x0, 0x08080808u);
            o[2 * jq + 1] = __vsub4(x1, 0x08080808u);
          }
          *(uint4 *)(dstB + cm_off(r, 32 * c4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *(uint4 *)(dstB + cm_off(r, 32 * c4 + 16)) = make_uint4(o[4], o[5], o[6], o[7]);
          jm += djm;
          rc += drc;
          if (rc >= per) {
            rc -= per;
            jm++;
          }
        }
      } else {
        // 48 packed bytes -> 64 int8 = four 16-byte K chunks
        for (int task = threadIdx.x; task < nt_here * mats * per; task += kThreads) {
          const int j = mats == 2 ? jm >> 1 : jm, mi = mats == 2 ? jm & 1 : 0;
          const int r = rc / CPR, c3 = rc % CPR;
          const uint8_t *pk_src = sa + U * kGemmA + (size_t)mi * NT * rowb + (size_t)j * KP;
          uint8_t *dstB = sg + (size_t)(j * mats + mi) * sbytes;
          uint32_t wd[12];
          if (r < nrows) {
            const uint4 *s4 = (const uint4 *)(pk_src + (size_t)r * rowb + 48 * c3);
            const uint4 x = s4[0], y = s4[1], z = s4[2];
            const uint32_t t12[12] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w, z.x, z.y, z.z, z.w};
#pragma unroll
            for (int i = 0; i < 12; i++) wd[i] = t12[i];
          } else {
#pragma unroll
            for (int i = 0; i < 12; i++) wd[i] = 0u;
          }
#pragma unroll
          for (int g = 0; g < 4; g++) {
            const uint32_t w0 = wd[3 * g], w1 = wd[3 * g + 1], w2 = wd[3 * g + 2];
            uint32_t f[4] = {q6_spread(w0 & 0xFFFFFFu), q6_spread(__funnelshift_r(w0, w1, 24) & 0xFFFFFFu),
                             q6_spread(__funnelshift_r(w1, w2, 16) & 0xFFFFFFu), q6_spread(w2 >> 8)};
#pragma unroll
            for (int i = 0; i < 4; i++) f[i] = r < nrows ? __vsub4(f[i], 0x20202020u) : 0u;
            *(uint4 *)(dstB + cm_off(r, 64 * c3 + 16 * g)) = make_uint4(f[0], f[1], f[2], f[3]);
          }
          jm += djm;
          rc += drc;
          if (rc >= per) {
            rc -= per;
            jm++;
          }
        }
      }
      if (ms) rg_bmark(c, 21);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (ms) rg_bmark(c, 22);
      if (warp == 0) {
        // MMAs of the stage's K tiles, in K order: warp 0 computes the
        // descriptors, one elected lane issues
        const bool leader = elect_one_sync();
        for (int j = 0; j < nt_here; j++)
          for (int s4 = 0; s4 < kKT / 32; s4++) {
            const uint64_t da = umma_desc(sa + (size_t)j * kGemmA + s4 * 256);
            const uint32_t acc = (su > 0 || j > 0 || s4 > 0) ? 1u : 0u;
            for (int mi = 0; mi < mats; mi++) {
              const uint64_t db = umma_desc(sg + (size_t)(j * mats + mi) * sbytes + s4 * 256);
              if (leader) umma_i8(tmem + (uint32_t)(mi * NT), da, db, idesc, acc);
            }
          }
        if (leader) {
          umma_commit(&bar_grp[grp]);
          umma_commit(&bar_su[slot]);
        }
        __syncwarp();
        if (mk && n0 == lo && su == 0) rg_bmark(c, 18);
        if (ms) rg_bmark(c, 15);
        // the previous stage's slot takes stage su - 1 + S once its MMAs are done
        if (su >= 1 && su - 1 + S < nsu) {
          const int pslot = (TU - 1) % S;
          mbar_wait(&bar_su[pslot], (uint32_t)((TU - 1) / S) & 1u, c.err);
          tc_fence_after();
          if (leader) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(su - 1 + S);
          }
          __syncwarp();
        }
      }
    }
    // the last stage's MMAs (commits complete in order: all are done)
    if (nsu > 0) {
      const int TL = TU0 + nsu - 1;
      mbar_wait(&bar_grp[TL & 1], (uint32_t)(TL >> 1) & 1u, c.err);
      tc_fence_after();
      __syncthreads();
    }
    // ---- epilogue: warps w and w+4 share TMEM lane quarter w (sequences
    // 16w .. 16w+15 in lanes 0..15), columns split between them
    {
      const int quarter = warp & 3, half = warp >> 2;
      const int m = 16 * quarter + lane;
      const bool live = lane < 16 && m < M;
      const float sx = live ? __ldcg(bw.act_sx + m) : 0.0f;
      // argmax only: lanes l and l + 16 share sequence 16 quarter + (l & 15),
      // lane l + 16 taking the upper 16 of every 32 columns
      const int ma = 16 * quarter + (lane & 15);
      const bool alive = ma < M;
      const float sxa = alive ? __ldcg(bw.act_sx + ma) : 0.0f;
      bool in_place = false;
      if (a.epi == EPI_RESID && live) {
        if (a.resid_mode == RESID_ALWAYS) {
          in_place = true;
        } else if (a.resid_mode == RESID_ATTN) {
          const int len = c.sp->seq[m].len;
          in_place = len >= 1 && len + 1 <= 6;  // model.go:4043-4062
        }
      }
      const int ncol = (NT + 15) / 16 * 8;  // columns per half, multiple of 8
      const int c_begin = half * ncol, c_end = min(min(NT, c_begin + ncol), nrows);
      const int epi = a.epi;
      const size_t ldo = (size_t)a.ldo;
      float *const outp = a.out, *const residp = a.resid, *const voutp = a.vout, *const logitsp = a.logits;
      const uint32_t tq = tmem + ((uint32_t)(32 * quarter) << 16);
      // 32 columns per load (columns < 2 NT + 32 <= kTmemCols: NT <= 256,
      // multiple of 16, and c_begin a multiple of 8 below NT / 2 + 8)
      for (int c0 = c_begin; c0 < c_end; c0 += 32) {
        uint32_t dv[32], uv[32];
        tmem_ld32_nowait(tq + (uint32_t)c0, dv);
        if (two) tmem_ld32_nowait(tq + (uint32_t)(NT + c0), uv);
        tmem_wait_ld();
        const int nj = min(32, c_end - c0);
        if (a.part) {
          // split-K: the raw dots of this K range
          if (!live) continue;
          int32_t *pp = a.part + ((size_t)kg * kMmaM + m) * ldo + n0 + c0;
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (j < nj) pp[j] = (int32_t)dv[j];
          continue;
        }
        if (epi == EPI_ARGMAX && !logitsp) {
          // vnni_finalize with the column's 128 * rowsum precomputed
          const int hi16 = lane >> 4;
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const uint32_t up = __shfl_sync(0xffffffffu, dv[16 + j], lane & 15);
            const int jj = j + 16 * hi16;
            if (alive && jj < nj) {
              const int cj = c0 + jj;
              const float d = __fsub_rn((float)(int32_t)(hi16 ? up : dv[j]), s_scl[kMaxNT + cj]);
              const unsigned long long k = argmax_key(__fmul_rn(__fmul_rn(d, sxa), s_scl[cj]), n0 + cj);
              best = k > best ? k : best;
            }
          }
          continue;
        }
        if (!live) continue;
        const size_t ob = (size_t)m * ldo + n0 + c0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          if (j >= nj) break;
          const int cj = c0 + j;
          const float v = vnni_finalize((int32_t)dv[j], s_rs[cj], sx, s_scl[cj]);
          const size_t o = ob + j;
          if (epi == EPI_STORE) {
            outp[o] = v;
          } else if (epi == EPI_RESID) {
            const float tt = __fadd_rn(__ldcg(residp + o), v);
            voutp[o] = tt;
            if (in_place) residp[o] = tt;
          } else if (epi == EPI_SWIGLU) {
            const float u = vnni_finalize((int32_t)uv[j], s_rs[kMaxNT + cj], sx, s_scl[kMaxNT + cj]);
            outp[o] = silu_mul(v, u);
          } else {
            if (logitsp) logitsp[o] = v;
            const unsigned long long k = argmax_key(v, n0 + cj);
            best = k > best ? k : best;
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (a.epi == EPI_ARGMAX) {
    const int m = 16 * (warp & 3) + lane;
    {
      // lanes l and l + 16 hold the same sequence's keys
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, 16);
      best = o > best ? o : best;
    }
    if (lane < 16 && m < M && best) atomicMax(a.argkey + m, best);
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
  if (mk) rg_bmark(c, 23);
}

// Split-K finalize of a residual GEMM (o or down projection): for every
// (sequence, row), the ks partial dots summed (exact int32), the same
// finalize and residual epilogue as EPI_RESID.
__device__ __noinline__ void phase_splitk_resid(const Ctx *cp, const BatchedW *bwp, const DMat *Ap, int ks, int rows,
                                                float *resid, float *vout, int resid_mode) {
  const Ctx &c = *cp;
  const BatchedW &bw = *bwp;
  const DMat &A = *Ap;
  const int M = c.sp->M;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < M * rows; i += gridDim.x * kThreads) {
    const int m = i / rows, row = i - m * rows;
    int32_t d = 0;  // the loads issued together; integer sums in any order are exact
#pragma unroll
    for (int g = 0; g < kDownSplits; g++)
      if (g < ks) d += __ldcg(bw.part + ((size_t)g * kMmaM + m) * rows + row);
    const float v = vnni_finalize(d, __ldg(A.rowsum + row), __ldcg(bw.act_sx + m), __ldg(A.scale + row));
    bool in_place = resid_mode == RESID_ALWAYS;
    if (resid_mode == RESID_ATTN) {
      const int len = c.sp->seq[m].len;
      in_place = len >= 1 && len + 1 <= 6;  // model.go:4043-4062
    }
    const size_t o = (size_t)m * rows + row;
    const float tt = __fadd_rn(__ldcg(resid + o), v);
    vout[o] = tt;
    if (in_place) resid[o] = tt;
  }
}

}  // namespace ocrvl
