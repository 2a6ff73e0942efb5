// Token sampling on the device: the sampler of the reference's generation
// loop on its CPU backend (internal/model/model.go:1536-1544 with the
// candidate path of 3632-3642 and 7202-7233), applied to logits rows that
// the step kernel wrote.  One CTA of kSampleThreads per row.
//
//   SAMPLE_TOPK  (2 <= k < vocab): the k highest logits with ties to the
//                lower id, in descending order (MatVecTopK*WithWork ->
//                topKSelectWithWork, internal/tensor/topk.go:326-347), then
//                sampleCandidateScoresScratch (model.go:1929-1976, 1978-2034,
//                2036-2061, 2140-2209, 2342-2462).
//   SAMPLE_FULL  (k <= 0 or k >= vocab): sampleFullLogitsScratch with a
//                weight scratch (model.go:2215-2307): ExpScaledVec weights
//                (weighted_sum.go:314-328 -> dot_amd64.s:6886-6946),
//                CumulativeSum (cumsum.go:9-58), pickCumulativeFloat32.
//   SAMPLE_ARGMAX (temperature <= 0 or k == 1): first maximum.
//
// The RNG is fastRNG (model.go:1829-1852): one uint64 state per row, one
// draw per sampled token.  Every float operation is an explicit
// round-to-nearest intrinsic in the reference's order (no contraction).
#pragma once
#include <cstdint>

#include "decoder.cuh"  // mbarriers and bulk copies
#include "numerics.cuh"

using ocrvl::exp_fma;
using ocrvl::fast_exp;

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxTopK = 4096;
constexpr int kFullTile = 1024;          // block-chain floats a round (per CumulativeSum block)
constexpr int kFullLaneSlab = 4096;      // lane-sum floats a round (16 lanes x 256)
constexpr int kFullStages = 4;           // rounds in flight in the shared-memory ring
constexpr int kFullTileStride = kFullTile + 4;  // 16-byte aligned, the 4 chain lanes on different banks
constexpr int kFullStage = 4 * kFullTileStride + kFullLaneSlab;  // floats a ring stage
constexpr int kFullMaxVocab = 262144;    // checkpoints (vocab / 16) held in shared memory
constexpr int kTopkBins = 4096;          // top-k first digit: the top 12 bits of the order key
constexpr int kTopkCap = 8192;           // top-k candidates the in-shared-memory sort holds
constexpr int kTopkRankMax = 384;        // up to this many candidates: rank sort, else bitonic

enum { SAMPLE_ARGMAX = 0, SAMPLE_TOPK = 1, SAMPLE_FULL = 2 };

struct SampleArgs {
  const float *logits;  // [rows][ld]
  long long ld;         // row stride in floats
  int V;                // vocabulary (row length)
  int mode;             // SAMPLE_*
  int k;                // top-k
  int temp1;            // top-k: temperature == 1 (float64 compare)
  float inv;            // top-k: float32(1/temp); full: 1/float32(temp)
  unsigned long long *rng;  // [rows] fastRNG states (in/out)
  int *out;                 // [rows] sampled ids (-1: internal failure)
  int *cand_ids;            // [rows][k] or null
  float *cand_scores;       // [rows][k] or null
  float *work;              // [rows][ld] cumulative sums (SAMPLE_FULL)
};

__host__ __device__ constexpr size_t sample_smem_topk(int k) {
  return (size_t)kTopkCap * 8 + (size_t)kTopkBins * 4 + (size_t)k * 20;
}
// checkpoint floats: one every 16 logits of each block plus the blocks'
// partial ends, rounded to an even count (the mbarriers after them are 8-byte)
__host__ __device__ constexpr int sample_full_ckpts(int V) { return (V / 16 + 9) & ~1; }
// ring, checkpoints, full / empty mbarriers
__host__ __device__ constexpr size_t sample_smem_full(int V) {
  return (size_t)kFullStages * kFullStage * 4 + (size_t)sample_full_ckpts(V) * 4 + 2 * kFullStages * 8;
}
__host__ __device__ constexpr size_t sample_smem_max() {
  return sample_smem_topk(kSampleMaxTopK) > sample_smem_full(kFullMaxVocab) ? sample_smem_topk(kSampleMaxTopK)
                                                                           : sample_smem_full(kFullMaxVocab);
}

// Round-to-nearest sum in the accumulator's precision.
__device__ __forceinline__ float sum_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double sum_rn(double a, float b) { return __dadd_rn(a, (double)b); }

// Four consecutive running sums (dst 16-byte aligned).
__device__ __forceinline__ void store4(float *d, float a, float b, float c, float e) {
  *reinterpret_cast<float4 *>(d) = make_float4(a, b, c, e);
}
__device__ __forceinline__ void store4(double *d, double a, double b, double c, double e) {
  reinterpret_cast<double2 *>(d)[0] = make_double2(a, b);
  reinterpret_cast<double2 *>(d)[1] = make_double2(c, e);
}

// fastRNG.Float64 (model.go:1833-1840).
__device__ __forceinline__ double rng_float64(unsigned long long &s) {
  s += 0x9e3779b97f4a7c15ull;
  unsigned long long z = s;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  z ^= z >> 31;
  return __dmul_rn(__ull2double_rn(z >> 11), 1.0 / 9007199254740992.0);
}

// Order key: a larger key is a larger float (-0 ties with +0, as the
// reference's float comparisons have it).  NaN logits are outside the
// contract.
__device__ __forceinline__ unsigned order_key(float x) {
  unsigned u = __float_as_uint(x);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One counting pass of a radix select: bin(i) in [0, 256) or -1 (skip),
// added to hist with one shared atomic per group of lanes sharing a bin.
template <typename BinFn>
__device__ __forceinline__ void sample_count(unsigned *hist, int V, BinFn bin_of) {
  const int lane = threadIdx.x & 31;
  for (int base = threadIdx.x & ~31; base < V; base += blockDim.x) {
    const int i = base + lane;
    const int bin = i < V ? bin_of(i) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, bin >= 0 ? (unsigned)bin : 256u + lane);
    if (bin >= 0 && lane == __ffs(grp) - 1) atomicAdd(&hist[bin], (unsigned)__popc(grp));
  }
}

// Warp 0: the bin holding the need-th element counted from bin 255 down
// (desc) or from bin 0 up; out = {bin, elements before it, its count}.
__device__ __forceinline__ void sample_pick_bin(const unsigned *hist, unsigned need, bool desc, unsigned *out) {
  const int lane = threadIdx.x & 31;
  unsigned c[8], local = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int b = lane * 8 + j;
    c[j] = hist[desc ? 255 - b : b];
    local += c[j];
  }
  unsigned incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  unsigned run = incl - local;
  if (run < need && need <= incl) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if (run + c[j] >= need) {
        const int b = lane * 8 + j;
        out[0] = desc ? 255 - b : b;
        out[1] = run;
        out[2] = c[j];
        break;
      }
      run += c[j];
    }
  }
}

// sampleCandidateScoresTemp1Small / sampleCandidateScoresSmall
// (model.go:2140-2209, 1978-2034) on 2..4 sorted candidates.
__device__ int sample_small(const float *ss, const int *sid, int k, bool temp1, float inv, unsigned long long &st) {
  if (k == 2) {
    const float s0 = temp1 ? ss[0] : __fmul_rn(ss[0], inv);
    const float s1 = temp1 ? ss[1] : __fmul_rn(ss[1], inv);
    if (s0 >= s1) {
      const double w1 = (double)fast_exp(__fsub_rn(s1, s0));
      return __dmul_rn(rng_float64(st), __dadd_rn(1.0, w1)) <= 1.0 ? sid[0] : sid[1];
    }
    const double w0 = (double)fast_exp(__fsub_rn(s0, s1));
    return __dmul_rn(rng_float64(st), __dadd_rn(w0, 1.0)) <= w0 ? sid[0] : sid[1];
  }
  if (temp1) {
    const float mx = ss[0];
    float w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) w[i] = i < k ? fast_exp(__fsub_rn(ss[i], mx)) : 0.0f;
    const float tot = k == 3 ? __fadd_rn(__fadd_rn(w[0], w[1]), w[2]) : __fadd_rn(__fadd_rn(w[0], w[1]), __fadd_rn(w[2], w[3]));
    const float pick = __fmul_rn(__double2float_rn(rng_float64(st)), tot);
    float acc = w[0];
    if (pick <= acc) return sid[0];
    acc = __fadd_rn(acc, w[1]);
    if (pick <= acc) return sid[1];
    if (k == 3) return sid[2];
    acc = __fadd_rn(acc, w[2]);
    return pick <= acc ? sid[2] : sid[3];
  }
  const float mx = __fmul_rn(ss[0], inv);
  double w[4];
#pragma unroll
  for (int i = 0; i < 4; i++) w[i] = i < k ? (double)fast_exp(__fsub_rn(__fmul_rn(ss[i], inv), mx)) : 0.0;
  const double tot = k == 3 ? __dadd_rn(__dadd_rn(w[0], w[1]), w[2]) : __dadd_rn(__dadd_rn(w[0], w[1]), __dadd_rn(w[2], w[3]));
  const double pick = __dmul_rn(rng_float64(st), tot);
  double acc = w[0];
  if (pick <= acc) return sid[0];
  acc = __dadd_rn(acc, w[1]);
  if (pick <= acc) return sid[1];
  if (k == 3) return sid[2];
  acc = __dadd_rn(acc, w[2]);
  return pick <= acc ? sid[2] : sid[3];
}

// Calls f(i, x[i]) for every i < V of one row; 16-byte loads, four a
// thread in flight, when the row is 16-byte aligned.  f runs under
// divergence (no warp-synchronous intrinsics).  Each thread visits its
// indices in increasing order.  kReadOnly: x is not written during the
// kernel (read-only data path); otherwise the loads go through L2.
template <bool kReadOnly = true, typename F>
__device__ __forceinline__ void for_each_logit(const float *x, int V, F f) {
  const int tid = threadIdx.x, bd = blockDim.x;
  int i0 = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    const int V4 = V >> 2;
    int j = tid;
    for (; j + 3 * bd < V4; j += 4 * bd) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) v[u] = kReadOnly ? __ldg(x4 + j + u * bd) : __ldcg(x4 + j + u * bd);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int i = 4 * (j + u * bd);
        f(i, v[u].x);
        f(i + 1, v[u].y);
        f(i + 2, v[u].z);
        f(i + 3, v[u].w);
      }
    }
    for (; j < V4; j += bd) {
      const float4 v = kReadOnly ? __ldg(x4 + j) : __ldcg(x4 + j);
      f(4 * j, v.x);
      f(4 * j + 1, v.y);
      f(4 * j + 2, v.z);
      f(4 * j + 3, v.w);
    }
    i0 = 4 * V4;
  }
  for (int i = i0 + tid; i < V; i += bd) f(i, kReadOnly ? __ldg(x + i) : __ldcg(x + i));
}

// Block-wide exclusive scan of one value a thread (blockDim.x a multiple of
// 32, at most 1024); returns the exclusive prefix, *total the block sum.
__device__ __forceinline__ unsigned block_exclusive_scan(unsigned v, unsigned *warp_sums, unsigned *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned w = lane < nw ? warp_sums[lane] : 0u;
    unsigned wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < nw) warp_sums[lane] = wi - w;
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  const unsigned r = warp_sums[warp] + incl - v;
  *total = warp_sums[32];
  __syncthreads();
  return r;
}

// Candidate key: the order key above, the complement of the id below, so
// that a larger key is a higher score or, on equal scores, a lower id.
__device__ __forceinline__ unsigned long long cand_key(unsigned key, int i) {
  return ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

// Fast path: one 12-bit histogram pass finds the bin that holds the k-th
// largest key; every logit at or above that bin's lower edge (normally a few
// hundred beyond k) is gathered into shared memory and sorted there (a rank
// count for a few hundred, else a bitonic network).
// Returns false (nothing written) when more than kTopkCap logits qualify.
__device__ bool topk_fast(const float *x, int V, int k, unsigned char *dsm, float *ss, int *sid) {
  __shared__ unsigned warp_sums[33];
  __shared__ unsigned s_bin, s_above, s_cnt, s_n;
  unsigned long long *buf = (unsigned long long *)dsm;
  unsigned *hist = (unsigned *)(dsm + (size_t)kTopkCap * 8);
  const int tid = threadIdx.x, bd = blockDim.x;
  for (int b = tid; b < kTopkBins; b += bd) hist[b] = 0;
  if (tid == 0) s_bin = s_above = s_cnt = 0;
  __syncthreads();
  for_each_logit(x, V, [&](int, float v) { atomicAdd(&hist[order_key(v) >> 20], 1u); });
  __syncthreads();
  // bins from the top, kTopkBins / blockDim.x consecutive bins a thread
  const int per = kTopkBins / bd;
  unsigned local = 0;
  for (int j = 0; j < per; j++) local += hist[kTopkBins - 1 - (tid * per + j)];
  unsigned total;
  unsigned run = block_exclusive_scan(local, warp_sums, &total);
  if (run < (unsigned)k && (unsigned)k <= run + local) {
    for (int j = 0; j < per; j++) {
      const int b = kTopkBins - 1 - (tid * per + j);
      if (run + hist[b] >= (unsigned)k) {
        s_bin = b;
        s_above = run;
        s_cnt = hist[b];
        break;
      }
      run += hist[b];
    }
  }
  __syncthreads();
  const unsigned C = s_above + s_cnt;
  if (C > (unsigned)kTopkCap) return false;  // uniform: read after a barrier
  const unsigned lower = s_bin << 20;
  if (tid == 0) s_n = 0;
  __syncthreads();
  for_each_logit(x, V, [&](int i, float v) {
    const unsigned key = order_key(v);
    if (key >= lower) {
      const unsigned p = atomicAdd(&s_n, 1u);
      if (p < C) buf[p] = cand_key(key, i);
    }
  });
  __syncthreads();
  if (C <= (unsigned)kTopkRankMax) {
    // few candidates: each one's place is the number of larger keys (only
    // the warps that hold a candidate run the count)
    if (tid < (int)C) {
      const unsigned long long mine = buf[tid];
      int place = 0;
      for (int j = 0; j < (int)C; j++) place += buf[j] > mine;
      if (place < k) sid[place] = (int)(0xFFFFFFFFu - (unsigned)(mine & 0xFFFFFFFFull));
    }
    __syncthreads();
  } else {
    int N = 2;
    while (N < (int)C) N <<= 1;
    for (int i = C + tid; i < N; i += bd) buf[i] = 0ull;  // below every real key
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= N; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int t = tid; t < (N >> 1); t += bd) {
          const int lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
          const unsigned long long u = buf[lo], w = buf[hi];
          if ((u < w) == ((lo & size) == 0)) {
            buf[lo] = w;
            buf[hi] = u;
          }
        }
        __syncthreads();
      }
    }
    for (int c = tid; c < k; c += bd) sid[c] = (int)(0xFFFFFFFFu - (unsigned)(buf[c] & 0xFFFFFFFFull));
    __syncthreads();
  }
  for (int c = tid; c < k; c += bd) ss[c] = x[sid[c]];  // the logit's own bits (the key folds -0 into +0)
  __syncthreads();
  return true;
}

// General path: 8-bit radix select of the k-th largest key, then the k-th
// smallest id among the logits equal to it, a gather of exactly k
// candidates and a rank sort.  Returns false on a candidate count mismatch.
__device__ bool topk_radix(const float *x, int V, int k, unsigned char *dsm, float *ss, int *sid) {
  __shared__ unsigned hist[256];
  __shared__ unsigned sel[3];
  __shared__ unsigned s_cnt;
  const int tid = threadIdx.x, lane = tid & 31;
  unsigned prefix = 0, mask = 0, need = (unsigned)k, ties = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    if (tid == 0) sel[0] = sel[1] = sel[2] = 0;
    __syncthreads();
    sample_count(hist, V, [&](int i) {
      const unsigned key = order_key(x[i]);
      return (key & mask) == prefix ? (int)((key >> shift) & 255u) : -1;
    });
    __syncthreads();
    if (tid < 32) sample_pick_bin(hist, need, true, sel);
    __syncthreads();
    prefix |= sel[0] << shift;
    mask |= 0xFFu << shift;
    need -= sel[1];
    ties = sel[2];
    __syncthreads();
  }
  unsigned idcut = 0xFFFFFFFFu;
  if (ties > need) {
    unsigned ip = 0, im = 0, n2 = need;
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (((unsigned)(V - 1) >> shift) == 0u) continue;  // every id has a zero byte here
      for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
      if (tid == 0) sel[0] = sel[1] = sel[2] = 0;
      __syncthreads();
      sample_count(hist, V, [&](int i) {
        return (order_key(x[i]) == prefix && ((unsigned)i & im) == ip) ? (int)(((unsigned)i >> shift) & 255u) : -1;
      });
      __syncthreads();
      if (tid < 32) sample_pick_bin(hist, n2, false, sel);
      __syncthreads();
      ip |= sel[0] << shift;
      im |= 0xFFu << shift;
      n2 -= sel[1];
      __syncthreads();
    }
    idcut = ip;
  }
  unsigned long long *ck = (unsigned long long *)dsm;
  int *cid = (int *)(ck + k);
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  for (int base = tid & ~31; base < V; base += blockDim.x) {
    const int i = base + lane;
    unsigned key = 0;
    bool take = false;
    if (i < V) {
      key = order_key(x[i]);
      take = key > prefix || (key == prefix && (unsigned)i <= idcut);
    }
    const unsigned b = __ballot_sync(0xffffffffu, take);
    unsigned p0 = 0;
    if (lane == 0 && b) p0 = atomicAdd(&s_cnt, (unsigned)__popc(b));
    p0 = __shfl_sync(0xffffffffu, p0, 0);
    if (take) {
      const unsigned p = p0 + __popc(b & ((1u << lane) - 1u));
      if (p < (unsigned)k) {
        ck[p] = cand_key(key, i);
        cid[p] = i;
      }
    }
  }
  __syncthreads();
  if (s_cnt != (unsigned)k) return false;
  for (int c = tid; c < k; c += blockDim.x) {
    const unsigned long long me = ck[c];
    int r = 0;
    for (int j = 0; j < k; j++) r += ck[j] > me;
    sid[r] = cid[c];
    ss[r] = x[cid[c]];
  }
  __syncthreads();
  return true;
}

// acc += src[0], src[1], ... src[n-1] in order (src 16-byte aligned), each
// partial sum stored to dst[j] when kStore (dst may be src).  16-byte loads
// run four to eight ahead of the dependent adds, so the chain is bound by
// the add latency rather than by shared-memory latency.
template <bool kStore, typename T>
__device__ __forceinline__ void chain4(T &acc, const float *src, T *dst, int n) {
  const float4 *s4 = reinterpret_cast<const float4 *>(src);
  const int n4 = n >> 2;
  const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 b[4];
#pragma unroll
  for (int u = 0; u < 4; u++) b[u] = u < n4 ? s4[u] : z;
  for (int q0 = 0; q0 < n4; q0 += 4) {
    float4 nb[4];
#pragma unroll
    for (int u = 0; u < 4; u++) nb[u] = q0 + 4 + u < n4 ? s4[q0 + 4 + u] : z;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      if (q0 + u < n4) {
        const T r0 = acc = sum_rn(acc, b[u].x);
        const T r1 = acc = sum_rn(acc, b[u].y);
        const T r2 = acc = sum_rn(acc, b[u].z);
        const T r3 = acc = sum_rn(acc, b[u].w);
        if (kStore) store4(dst + 4 * (q0 + u), r0, r1, r2, r3);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) b[u] = nb[u];
  }
  for (int j = 4 * n4; j < n; j++) {
    acc = sum_rn(acc, src[j]);
    if (kStore) dst[j] = acc;
  }
}

// acc += the 4 * n4 floats of src in order, storing the running sum after
// every 16 (each whole group of four float4) to ck[0], ck[1], ...  The main
// loop has no per-element guards: the next group's loads are issued, then
// this group's 16 dependent adds run.
__device__ __forceinline__ void chain_ckpt(float &acc, const float *src, int n4, float *ck) {
  const float4 *s4 = reinterpret_cast<const float4 *>(src);
  const int nf = n4 & ~3;  // float4 in whole groups
  float4 b0, b1, b2, b3;
  if (nf > 0) {
    b0 = s4[0];
    b1 = s4[1];
    b2 = s4[2];
    b3 = s4[3];
  }
  for (int q0 = 0; q0 < nf; q0 += 4) {
    float4 n0, n1, n2, n3;
    const bool more = q0 + 4 < nf;
    if (more) {
      n0 = s4[q0 + 4];
      n1 = s4[q0 + 5];
      n2 = s4[q0 + 6];
      n3 = s4[q0 + 7];
    }
    acc = __fadd_rn(acc, b0.x); acc = __fadd_rn(acc, b0.y); acc = __fadd_rn(acc, b0.z); acc = __fadd_rn(acc, b0.w);
    acc = __fadd_rn(acc, b1.x); acc = __fadd_rn(acc, b1.y); acc = __fadd_rn(acc, b1.z); acc = __fadd_rn(acc, b1.w);
    acc = __fadd_rn(acc, b2.x); acc = __fadd_rn(acc, b2.y); acc = __fadd_rn(acc, b2.z); acc = __fadd_rn(acc, b2.w);
    acc = __fadd_rn(acc, b3.x); acc = __fadd_rn(acc, b3.y); acc = __fadd_rn(acc, b3.z); acc = __fadd_rn(acc, b3.w);
    ck[q0 >> 2] = acc;
    if (more) {
      b0 = n0;
      b1 = n1;
      b2 = n2;
      b3 = n3;
    }
  }
  for (int q = nf; q < n4; q++) {  // a partial last group (its end is the block's, stored by the caller)
    const float4 v = s4[q];
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
    acc = __fadd_rn(acc, v.z);
    acc = __fadd_rn(acc, v.w);
  }
}

// Top-k candidates and the draw for one row.  Shared memory: kTopkCap
// 8-byte candidate keys, kTopkBins counters, then the running sums (k
// doubles), ss, sid and w (k each).
__device__ void sample_topk_row(const SampleArgs &a, int row, unsigned char *dsm) {
  __shared__ int s_first;
  __shared__ float s_pickf;
  __shared__ double s_pickd;
  const float *x = a.logits + (long long)row * a.ld;
  const int V = a.V, k = a.k, tid = threadIdx.x;
  unsigned char *tail = dsm + (size_t)kTopkCap * 8 + (size_t)kTopkBins * 4;
  double *partd = (double *)tail;
  float *partf = (float *)tail;
  float *ss = (float *)(partd + k);
  int *sid = (int *)(ss + k);
  float *w = (float *)(sid + k);
  if (!topk_fast(x, V, k, dsm, ss, sid) && !topk_radix(x, V, k, dsm, ss, sid)) {
    if (tid == 0) a.out[row] = -1;
    return;
  }
  for (int c = tid; c < k; c += blockDim.x) {
    if (a.cand_ids) a.cand_ids[(long long)row * k + c] = sid[c];
    if (a.cand_scores) a.cand_scores[(long long)row * k + c] = ss[c];
  }
  const bool temp1 = a.temp1 != 0;
  if (k <= 4) {
    if (tid == 0) {
      unsigned long long st = a.rng[row];
      a.out[row] = sample_small(ss, sid, k, temp1, a.inv, st);
      a.rng[row] = st;
    }
    return;
  }
  // weights; the maximum of the sorted candidates is the first
  const float mx = temp1 ? ss[0] : __fmul_rn(ss[0], a.inv);
  for (int c = tid; c < k; c += blockDim.x)
    w[c] = temp1 ? fast_exp(__fsub_rn(ss[c], mx)) : fast_exp(__fsub_rn(__fmul_rn(ss[c], a.inv), mx));
  __syncthreads();
  // the running sums (one chain in the reference's order; the pick scan of
  // pickWeighted*Float32 compares against the same partial sums)
  if (tid == 0) {
    unsigned long long st = a.rng[row];
    if (temp1) {
      float acc = 0.0f;
      chain4<true>(acc, w, partf, k);
      s_pickf = __fmul_rn(__double2float_rn(rng_float64(st)), acc);
    } else {
      double acc = 0.0;
      chain4<true>(acc, w, partd, k);
      s_pickd = __dmul_rn(rng_float64(st), acc);
    }
    a.rng[row] = st;
    s_first = k;
  }
  __syncthreads();
  for (int c = tid; c < k; c += blockDim.x) {
    const bool hit = temp1 ? s_pickf <= partf[c] : s_pickd <= partd[c];
    if (hit) atomicMin(&s_first, c);
  }
  __syncthreads();
  if (tid == 0) a.out[row] = sid[s_first < k ? s_first : k - 1];
}

// Bounded mbarrier wait that sleeps between polls: for the warps that run
// ahead of the cumulative-sum chains, so that their polling leaves the
// shared-memory pipe to the chains.  Gives up (error word set) after about
// two seconds or, with bail (waits on other threads' arrivals, not on this
// block's own copies), once another thread has set the error word.
__device__ __forceinline__ bool wait_backoff(uint64_t *bar, uint32_t parity, int *err, bool bail) {
  const unsigned long long t0 = ocrvl::gtimer();
  for (long long i = 0; i < (1ll << 24); i++) {
    uint32_t done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done)
                 : "r"(ocrvl::smem_u32(bar)), "r"(parity)
                 : "memory");
    if (done) return true;
    __nanosleep(256);
    if ((i & 63) == 63 && (ocrvl::gtimer() - t0 > ocrvl::kMbarWaitNs || (bail && *(volatile int *)err))) break;
  }
  atomicExch(err, 1);
  return false;
}

// Full-vocabulary draw for one row (V a multiple of 16, at most
// kFullMaxVocab).  Phases:
//   (1) maximum (tensor.Max) and bias = -(max * inv);
//   (2) every weight exp(x * inv + bias) to work[] (all threads), noting any
//       weight with its sign bit set or NaN;
//   (3) the sequential sums: warp 1 lanes 0..nb-1 run the CumulativeSum
//       block chains and keep the running sum at the end of every 16-logit
//       group (checkpoints, in shared memory); warp 0 lanes 0..15 run the 16
//       lane sums of expScaledVecFMA.  The weights reach shared memory by
//       bulk copies (cp.async.bulk) into a ring of kFullStages rounds that
//       warp 2 lane 0 refills as the consumers release stages.
//   (4) the pick and pickCumulativeFloat32: with no negative or NaN weight
//       the cumulative sums never decrease, so the binary search's answer is
//       the first index whose sum reaches the pick: the first group whose end
//       does, then one group re-summed from its checkpoint.  Otherwise the
//       binary search itself runs, each probe re-summed from a checkpoint.
__device__ void sample_full_row(const SampleArgs &a, int row, unsigned char *dsm) {
  __shared__ float red[32];
  __shared__ float s_bs[4];
  __shared__ float s_sum, s_pick;
  __shared__ int s_neg, s_err, s_first;
  const float *x = a.logits + (long long)row * a.ld;
  float *wk = a.work + (long long)row * a.ld;
  const int V = a.V, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int nb = V < 4096 ? 1 : 4;
  const int bs = V < 4096 ? V : V / 4;
  const int ngrp = (bs + 15) / 16;  // checkpoint groups a block
  float *ring = (float *)dsm;
  float *ck = ring + (size_t)kFullStages * kFullStage;
  uint64_t *full = (uint64_t *)(ck + sample_full_ckpts(V));
  uint64_t *empty = full + kFullStages;

  // (1)
  if (tid == 0) {
    s_neg = 0;
    s_err = 0;
    for (int st = 0; st < kFullStages; st++) {
      ocrvl::mbar_init(&full[st], 1);
      ocrvl::mbar_init(&empty[st], 2);
    }
    ocrvl::mbar_fence_init();
  }
  float m = -INFINITY;
  for_each_logit(x, V, [&](int, float v) { m = fmaxf(m, v); });
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < nwarps ? red[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[0] = m;
  }
  __syncthreads();
  const float inv = a.inv;
  const float bias = -__fmul_rn(red[0], inv);
  auto weight = [&](float v) { return exp_fma(__fadd_rn(__fmul_rn(v, inv), bias)); };

  // (2) V % 16 == 0 and 16-byte aligned rows: whole float4 groups
  {
    bool neg = false;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *w4 = reinterpret_cast<float4 *>(wk);
    for (int q = tid; q < V / 4; q += blockDim.x) {
      const float4 v = __ldg(x4 + q);
      const float4 w = make_float4(weight(v.x), weight(v.y), weight(v.z), weight(v.w));
      neg |= (__float_as_uint(w.x) | __float_as_uint(w.y) | __float_as_uint(w.z) | __float_as_uint(w.w)) >> 31;
      neg |= isnan(w.x) || isnan(w.y) || isnan(w.z) || isnan(w.w);
      w4[q] = w;
    }
    if (__any_sync(0xffffffffu, neg) && lane == 0) s_neg = 1;
    // the bulk copies (async proxy) read what these stores wrote
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();

  // (3)
  const int rounds = (bs + kFullTile - 1) / kFullTile;
  const int lrounds = (V + kFullLaneSlab - 1) / kFullLaneSlab;
  const int R = rounds > lrounds ? rounds : lrounds;
  float acc = 0.0f;
  if (warp == 2 && lane == 0) {
    for (int r = 0; r < R; r++) {
      const int st = r % kFullStages;
      if (r >= kFullStages && !wait_backoff(&empty[st], (r / kFullStages - 1) & 1, &s_err, true)) break;
      float *dst = ring + (size_t)st * kFullStage;
      const int cl = max(0, min(kFullTile, bs - r * kFullTile));
      const int ll = max(0, min(kFullLaneSlab, V - r * kFullLaneSlab));
      ocrvl::mbar_expect_tx(&full[st], (uint32_t)(4 * (nb * cl + ll)));
      if (cl > 0)
        for (int b = 0; b < nb; b++)
          ocrvl::bulk_g2s(dst + b * kFullTileStride, wk + (size_t)b * bs + (size_t)r * kFullTile, 4u * cl, &full[st]);
      if (ll > 0) ocrvl::bulk_g2s(dst + 4 * kFullTileStride, wk + (size_t)r * kFullLaneSlab, 4u * ll, &full[st]);
    }
  } else if (warp == 0 && lane < 16) {
    for (int r = 0; r < R; r++) {
      const int st = r % kFullStages;
      if (!wait_backoff(&full[st], (r / kFullStages) & 1, &s_err, false)) break;
      const float *src = ring + (size_t)st * kFullStage + 4 * kFullTileStride + lane;
      const int n = max(0, min(kFullLaneSlab, V - r * kFullLaneSlab)) / 16;  // this lane's terms
      float nxt[8];
#pragma unroll
      for (int u = 0; u < 8; u++) nxt[u] = u < n ? src[16 * u] : 0.0f;
      for (int t0 = 0; t0 < n; t0 += 8) {
        float cur[8];
#pragma unroll
        for (int u = 0; u < 8; u++) cur[u] = nxt[u];
#pragma unroll
        for (int u = 0; u < 8; u++) nxt[u] = t0 + 8 + u < n ? src[16 * (t0 + 8 + u)] : 0.0f;
#pragma unroll
        for (int u = 0; u < 8; u++)
          if (t0 + u < n) acc = __fadd_rn(acc, cur[u]);
      }
      __syncwarp(0xffffu);
      if (lane == 0) asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(ocrvl::smem_u32(&empty[st])) : "memory");
    }
  } else if (warp == 1 && lane < nb) {
    const unsigned cmask = (1u << nb) - 1u;
    float *ckb = ck + lane * ngrp;
    for (int r = 0; r < R; r++) {
      const int st = r % kFullStages;
      if (!ocrvl::mbar_wait(&full[st], (r / kFullStages) & 1, &s_err)) break;
      const float4 *s4 = reinterpret_cast<const float4 *>(ring + (size_t)st * kFullStage + lane * kFullTileStride);
      const int n4 = max(0, min(kFullTile, bs - r * kFullTile)) / 4;
      // the running sum after every 16 logits, and at the block's end
      chain_ckpt(acc, reinterpret_cast<const float *>(s4), n4, ckb + r * (kFullTile / 16));
      if (r * kFullTile + 4 * n4 == bs && (bs & 15)) ckb[(bs - 1) >> 4] = acc;
      __syncwarp(cmask);
      if (lane == 0) asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(ocrvl::smem_u32(&empty[st])) : "memory");
    }
  }
  if (warp == 0) {  // tree16 of the 16 lane sums
    float v = acc;
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
    if (lane == 0) s_sum = v;
  } else if (warp == 1 && lane < 4) {
    s_bs[lane] = lane < nb ? acc : 0.0f;
  }
  __syncthreads();
  if (s_err) {
    if (tid == 0) a.out[row] = -1;
    return;
  }

  // (4) block offsets (cumsum.go:46-57), the pick, pickCumulativeFloat32
  const float off1 = s_bs[0];
  const float off2 = __fadd_rn(off1, s_bs[1]);
  const float off3 = __fadd_rn(off2, s_bs[2]);
  auto with_off = [&](int b, float c) { return b == 0 ? c : __fadd_rn(c, b == 1 ? off1 : b == 2 ? off2 : off3); };
  // block-local running sum at j, re-summed from the checkpoint before it
  auto cs_at = [&](int b, int j) {
    const int g = j >> 4;
    float c = g == 0 ? 0.0f : ck[b * ngrp + g - 1];
    for (int e = g * 16; e <= j; e++) c = __fadd_rn(c, __ldcg(wk + (size_t)b * bs + e));
    return c;
  };
  if (tid == 0) {
    unsigned long long stt = a.rng[row];
    s_pick = __fmul_rn(__double2float_rn(rng_float64(stt)), s_sum);
    a.rng[row] = stt;
    s_first = nb * ngrp;
  }
  __syncthreads();
  const float pick = s_pick;
  if (!s_neg) {
    for (int G = tid; G < nb * ngrp; G += blockDim.x)
      if (pick <= with_off(G / ngrp, ck[G])) atomicMin(&s_first, G);
    __syncthreads();
    if (tid == 0) {
      int res = V - 1;
      if (s_first < nb * ngrp) {
        const int b = s_first / ngrp, g = s_first % ngrp;
        float c = g == 0 ? 0.0f : ck[b * ngrp + g - 1];
        const int end = min(bs, (g + 1) * 16);
        for (int e = g * 16; e < end; e++) {
          c = __fadd_rn(c, __ldcg(wk + (size_t)b * bs + e));
          if (pick <= with_off(b, c)) {
            res = b * bs + e;
            break;
          }
        }
      }
      a.out[row] = res;
    }
  } else if (tid == 0) {
    int lo = 0, hi = V;
    while (lo < hi) {
      const int mid = (int)((unsigned)(lo + hi) >> 1);
      const int b = mid / bs;
      if (pick <= with_off(b, cs_at(b, mid - b * bs))) hi = mid;
      else lo = mid + 1;
    }
    a.out[row] = lo < V ? lo : V - 1;
  }
}

// First maximum of one row.
__device__ void sample_argmax_row(const SampleArgs &a, int row) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float *x = a.logits + (long long)row * a.ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float bv = -INFINITY;
  int bi = a.V;
  // each thread visits its indices in increasing order: its first maximum
  for_each_logit(x, a.V, [&](int i, float v) {
    if (bi == a.V || v > bv) {
      bv = v;
      bi = i;
    }
  });
  auto merge = [&](float ov, int oi) {
    if (oi < a.V && (bi == a.V || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
    }
  };
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    merge(ov, oi);
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) merge(sv[w], si[w]);
    a.out[row] = bi < a.V ? bi : 0;
  }
}

__global__ void __launch_bounds__(kSampleThreads, 1) k_sample(SampleArgs a) {
  extern __shared__ __align__(16) unsigned char sample_dsm[];
  const int row = blockIdx.x;
  if (a.mode == SAMPLE_TOPK) sample_topk_row(a, row, sample_dsm);
  else if (a.mode == SAMPLE_FULL) sample_full_row(a, row, sample_dsm);
  else sample_argmax_row(a, row);
}
