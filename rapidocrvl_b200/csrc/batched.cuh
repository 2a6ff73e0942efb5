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
//   with two buffers per operand, so the copies and the unpacking of tile t+1
//   overlap the tensor core's work on tile t; each MMA batch commits to an
//   mbarrier that frees its buffers.  The epilogue reads D with tcgen05.ld
//   (M = 64 puts sequence r in TMEM lane 32*(r/16) + r%16) and applies the
//   same finalize and epilogue (store, residual, SwiGLU, argmax) as the
//   single-sequence kernels.
#pragma once

namespace ocrvl {

constexpr int kKT = 128;          // activations (int8 columns) per K tile
constexpr int kMmaM = 64;         // A rows (sequences) per MMA
constexpr int kMaxNT = 256;       // output rows per N tile
constexpr int kTmemCols = 512;    // TMEM columns a block allocates

// TMA descriptor of one packed weight matrix (CUtensorMap, 128 bytes).
struct __align__(64) TmapBytes {
  unsigned char b[128];
};

struct BatchedW {
  const TmapBytes *tm;  // [L * 5 + 1]: per layer qkv, o, gate, up, down; then lm_head
  uint8_t *act;         // activation image [K tiles][64 rows][kKT]
  float *act_sx;        // [kMaxSeqs] activation scale per sequence
};

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
// 2-D TMA tile copy (no multicast) of a box at (x bytes, y rows).
__device__ __forceinline__ void tma_2d(void *dst, const TmapBytes *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

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
  int epi;                       // EPI_*
  float *out;
  int ldo;
  float *resid, *vout;
  int resid_mode;
  unsigned long long *argkey;
  float *logits;
  int argmax_finish, feed;
};

// shared-memory layout of the GEMM phase (bytes)
constexpr int kGemmA = kMmaM * kKT;              // 8 KB per A buffer
constexpr int kGemmB = kMaxNT * kKT;             // 32 KB per B buffer (int8)
constexpr int kGemmStage = kMaxNT * kKT * 3 / 4; // 24 KB per packed staging buffer (Q6 worst case)
__host__ __device__ __forceinline__ size_t gemm_b_smem_bytes() {
  return 2 * (size_t)kGemmA + 2 * (size_t)kGemmB + 2 * (size_t)kGemmStage * 2 + 4 * kMaxNT * 4 + 1024;
}

template <int QT>
__device__ __noinline__ void phase_gemm_b(const Ctx *cp, const BatchedW *bwp, const GemmArgs *gp, uint32_t tmem,
                                          float *smem) {
  const Ctx &c = *cp;
  const BatchedW &bw = *bwp;
  const GemmArgs &a = *gp;
  constexpr int KP = QT == QT_Q4 ? kKT / 2 : kKT * 3 / 4;  // packed bytes per row per K tile
  const bool two = a.epi == EPI_SWIGLU;
  const int M = c.sp->M;
  uint8_t *base = (uint8_t *)smem;
  uint8_t *sA[2] = {base, base + kGemmA};
  uint8_t *sB[2][2] = {{base + 2 * kGemmA, base + 2 * kGemmA + kGemmB}, {nullptr, nullptr}};
  uint8_t *stg0 = base + 2 * kGemmA + 2 * kGemmB;
  uint8_t *sStage[2][2] = {{stg0, stg0 + kGemmStage}, {stg0 + 2 * kGemmStage, stg0 + 3 * kGemmStage}};
  float *s_scl = (float *)(stg0 + 4 * kGemmStage);  // [2][kMaxNT] scales, [2][kMaxNT] row sums
  int32_t *s_rs = (int32_t *)(s_scl + 2 * kMaxNT);
  __shared__ __align__(8) uint64_t bar_ld[2], bar_mma[2];
  __shared__ uint32_t par_ld, par_mma;
  // SwiGLU keeps both weight tiles: B of the up matrix reuses the second
  // buffer pair, so K tiles are single-buffered for it
  int lo, hi;
  gemv_slab(a.row_begin, a.row_end, blockIdx.x, gridDim.x, lo, hi);
  const int nk = a.K / kKT;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&bar_ld[i], 1);
      mbar_init(&bar_mma[i], 1);
    }
    mbar_fence_init();
    par_ld = 0;
    par_mma = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long best = 0ull;  // ARGMAX: lane's sequence best key
  for (int n0 = lo; n0 < hi; n0 += a.nt) {
    const int nrows = min(a.nt, hi - n0);
    const int NT = a.nt;
    // scales / row sums of this N tile
    for (int i = threadIdx.x; i < nrows; i += kThreads) {
      s_scl[i] = __ldg(a.A.scale + n0 + i);
      s_rs[i] = __ldg(a.A.rowsum + n0 + i);
      if (two) {
        s_scl[kMaxNT + i] = __ldg(a.B.scale + n0 + i);
        s_rs[kMaxNT + i] = __ldg(a.B.rowsum + n0 + i);
      }
    }
    const int nbuf = two ? 1 : 2;  // SwiGLU: one buffer per matrix
    auto issue = [&](int t) {     // thread 0: copies of K tile t
      const int b = t % nbuf;
      const uint32_t bytes_b = (uint32_t)a.nt * KP;  // the whole box (rows past the matrix are zero-filled)
      mbar_expect_tx(&bar_ld[b], kGemmA + (two ? 2 : 1) * bytes_b);
      bulk_g2s(sA[b], bw.act + (size_t)t * kGemmA, kGemmA, &bar_ld[b]);
      tma_2d(sStage[0][b], a.mapA, t * KP, n0, &bar_ld[b]);
      if (two) tma_2d(sStage[1][0], a.mapB, t * KP, n0, &bar_ld[b]);
    };
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int t = 0; t < nk && t < nbuf; t++) issue(t);
    }
    const uint32_t idesc = umma_idesc_i8(NT);
    for (int t = 0; t < nk; t++) {
      const int b = t % nbuf;
      // wait for the copies of tile t
      if (!mbar_wait(&bar_ld[b], (par_ld >> b) & 1u, c.err)) break;
      // unpack the packed weights to int8 in the core-matrix layout
      for (int mi = 0; mi < (two ? 2 : 1); mi++) {
        const uint8_t *stg = two ? sStage[mi][0] : sStage[0][b];
        uint8_t *dstB = two ? sB[0][mi] : sB[0][b];
        if (QT == QT_Q4) {
          // 16 packed bytes -> 32 int8 = two 16-byte K chunks
          for (int task = threadIdx.x; task < NT * (KP / 16); task += kThreads) {
            const int r = task / (KP / 16), c4 = task % (KP / 16);
            uint4 pk = make_uint4(0, 0, 0, 0);
            if (r < nrows) pk = *(const uint4 *)(stg + (size_t)r * KP + 16 * c4);
            const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const uint32_t lo4 = w4[j] & 0x0F0F0F0Fu, hi4 = (w4[j] >> 4) & 0x0F0F0F0Fu;
              // bytes b0..b3 -> (lo0, hi0, lo1, hi1), (lo2, hi2, lo3, hi3); nibble - 8
              const uint32_t x0 = __byte_perm(lo4, hi4, 0x5140), x1 = __byte_perm(lo4, hi4, 0x7362);
              o[2 * j] = __vsub4(x0, 0x08080808u);
              o[2 * j + 1] = __vsub4(x1, 0x08080808u);
            }
            *(uint4 *)(dstB + cm_off(r, 32 * c4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *(uint4 *)(dstB + cm_off(r, 32 * c4 + 16)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        } else {
          // 48 packed bytes -> 64 int8 = four 16-byte K chunks
          for (int task = threadIdx.x; task < NT * (KP / 48); task += kThreads) {
            const int r = task / (KP / 48), c3 = task % (KP / 48);
            uint32_t wd[12];
            if (r < nrows) {
              const uint4 *s4 = (const uint4 *)(stg + (size_t)r * KP + 48 * c3);
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
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (threadIdx.x == 0) {
        par_ld ^= 1u << b;
        // MMAs of this K tile
        for (int s = 0; s < kKT / 32; s++) {
          const uint64_t da = umma_desc(sA[b] + s * 256);
          const uint32_t acc = (t > 0 || s > 0) ? 1u : 0u;
          if (two) {
            umma_i8(tmem, da, umma_desc(sB[0][0] + s * 256), idesc, acc);
            umma_i8(tmem + (uint32_t)NT, da, umma_desc(sB[0][1] + s * 256), idesc, acc);
          } else {
            umma_i8(tmem, da, umma_desc(sB[0][b] + s * 256), idesc, acc);
          }
        }
        umma_commit(&bar_mma[b]);
      }
      // refill: the buffers of the previous tile (two buffers) or of this
      // tile (SwiGLU, one buffer) take tile t + 1 once their MMAs are done
      const int tb = nbuf == 2 ? t - 1 : t;
      if (tb >= 0) {
        const int bb = tb % nbuf;
        if (!mbar_wait(&bar_mma[bb], (par_mma >> bb) & 1u, c.err)) break;
        tc_fence_after();
        __syncthreads();
        if (threadIdx.x == 0) {
          par_mma ^= 1u << bb;
          if (t + 1 < nk && (nbuf == 1 || t + 1 >= nbuf)) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(t + 1);
          }
        }
      }
    }
    // the last tile's MMAs (two buffers: not waited in the loop)
    if (nbuf == 2 && nk > 0) {
      const int bb = (nk - 1) % 2;
      mbar_wait(&bar_mma[bb], (par_mma >> bb) & 1u, c.err);
      tc_fence_after();
      __syncthreads();
      if (threadIdx.x == 0) par_mma ^= 1u << bb;
      __syncthreads();
    }
    // ---- epilogue: warps w and w+4 share TMEM lane quarter w (sequences
    // 16w .. 16w+15 in lanes 0..15), columns split between them
    {
      const int quarter = warp & 3, half = warp >> 2;
      const int m = 16 * quarter + lane;
      const bool live = lane < 16 && m < M;
      const float sx = live ? __ldcg(bw.act_sx + m) : 0.0f;
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
      const int c_begin = half * ncol, c_end = min(NT, c_begin + ncol);
      for (int c0 = c_begin; c0 < c_end; c0 += 8) {
        uint32_t dv[8], uv[8];
        tmem_ld8(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, dv);
        if (two) tmem_ld8(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(NT + c0), uv);
        if (!live) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int cj = c0 + j;
          if (cj >= nrows) break;
          const int row = n0 + cj;
          const float v = vnni_finalize((int32_t)dv[j], s_rs[cj], sx, s_scl[cj]);
          const size_t o = (size_t)m * a.ldo + row;
          if (a.epi == EPI_STORE) {
            a.out[o] = v;
          } else if (a.epi == EPI_RESID) {
            const float tt = __fadd_rn(__ldcg(a.resid + o), v);
            a.vout[o] = tt;
            if (in_place) a.resid[o] = tt;
          } else if (a.epi == EPI_SWIGLU) {
            const float u = vnni_finalize((int32_t)uv[j], s_rs[kMaxNT + cj], sx, s_scl[kMaxNT + cj]);
            a.out[o] = silu_mul(v, u);
          } else {
            if (a.logits) a.logits[o] = v;
            const unsigned long long k = argmax_key(v, row);
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
}

}  // namespace ocrvl
