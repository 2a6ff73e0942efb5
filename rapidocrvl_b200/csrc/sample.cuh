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

#include "numerics.cuh"

using ocrvl::exp_fma;
using ocrvl::fast_exp;

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxTopK = 4096;
constexpr int kFullTile = 1024;          // block-chain floats per round
constexpr int kFullLaneSlab = 4096;      // lane-sum floats per round (16 lanes x 256)

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
  int *out;                 // [rows] sampled ids (-1: candidate count mismatch)
  int *cand_ids;            // [rows][k] or null
  float *cand_scores;       // [rows][k] or null
  float *work;              // [rows][ld] cumulative sums (SAMPLE_FULL)
};

__host__ __device__ constexpr size_t sample_smem_topk(int k) { return (size_t)k * 28 + 16; }
__host__ __device__ constexpr size_t sample_smem_full() { return 2 * (4 * (kFullTile + 1) + kFullLaneSlab) * 4; }
__host__ __device__ constexpr size_t sample_smem_max() {
  return sample_smem_topk(kSampleMaxTopK) > sample_smem_full() ? sample_smem_topk(kSampleMaxTopK) : sample_smem_full();
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

// Top-k candidates and the draw for one row.
__device__ void sample_topk_row(const SampleArgs &a, int row, unsigned char *dsm) {
  __shared__ unsigned hist[256];
  __shared__ unsigned sel[3];
  __shared__ unsigned s_cnt;
  __shared__ int s_first;
  __shared__ float s_pickf;
  __shared__ double s_pickd;
  const float *x = a.logits + (long long)row * a.ld;
  const int V = a.V, k = a.k, tid = threadIdx.x, lane = tid & 31;

  // (1) radix select of the k-th largest order key T, 8 bits a pass
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
  // (2) when more logits equal T than are needed, the need-th smallest id
  //     among them bounds the ones taken (ties go to the lower id)
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
  // (3) collect the k candidates (unordered)
  unsigned long long *ck = (unsigned long long *)dsm;
  float *cs = (float *)(ck + k);
  int *cid = (int *)(cs + k);
  float *ss = (float *)(cid + k);
  int *sid = (int *)(ss + k);
  float *w = (float *)(sid + k);
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  for (int base = tid & ~31; base < V; base += blockDim.x) {
    const int i = base + lane;
    float v = 0.0f;
    unsigned key = 0;
    bool take = false;
    if (i < V) {
      v = x[i];
      key = order_key(v);
      take = key > prefix || (key == prefix && (unsigned)i <= idcut);
    }
    const unsigned b = __ballot_sync(0xffffffffu, take);
    unsigned p0 = 0;
    if (lane == 0 && b) p0 = atomicAdd(&s_cnt, (unsigned)__popc(b));
    p0 = __shfl_sync(0xffffffffu, p0, 0);
    if (take) {
      const unsigned p = p0 + __popc(b & ((1u << lane) - 1u));
      if (p < (unsigned)k) {
        ck[p] = ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
        cs[p] = v;
        cid[p] = i;
      }
    }
  }
  __syncthreads();
  if (s_cnt != (unsigned)k) {
    if (tid == 0) a.out[row] = -1;
    return;
  }
  // (4) descending order by (score, lower id): rank of each candidate
  for (int c = tid; c < k; c += blockDim.x) {
    const unsigned long long me = ck[c];
    int r = 0;
    for (int j = 0; j < k; j++) r += ck[j] > me;
    ss[r] = cs[c];
    sid[r] = cid[c];
  }
  __syncthreads();
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
  // (5) weights; the maximum of the sorted candidates is the first
  const float mx = temp1 ? ss[0] : __fmul_rn(ss[0], a.inv);
  for (int c = tid; c < k; c += blockDim.x)
    w[c] = temp1 ? fast_exp(__fsub_rn(ss[c], mx)) : fast_exp(__fsub_rn(__fmul_rn(ss[c], a.inv), mx));
  __syncthreads();
  // (6) the running sums (one chain in the reference's order; the pick scan
  //     of pickWeighted*Float32 compares against the same partial sums)
  double *partd = (double *)ck;
  float *partf = cs;
  if (tid == 0) {
    unsigned long long st = a.rng[row];
    if (temp1) {
      float acc = 0.0f;
#pragma unroll 8
      for (int c = 0; c < k; c++) {
        acc = __fadd_rn(acc, w[c]);
        partf[c] = acc;
      }
      s_pickf = __fmul_rn(__double2float_rn(rng_float64(st)), acc);
    } else {
      double acc = 0.0;
#pragma unroll 8
      for (int c = 0; c < k; c++) {
        acc = __dadd_rn(acc, (double)w[c]);
        partd[c] = acc;
      }
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

// Full-vocabulary draw for one row (V a multiple of 16).
__device__ void sample_full_row(const SampleArgs &a, int row, unsigned char *dsm) {
  __shared__ float red[32];
  __shared__ float s_bs[4];
  __shared__ float s_sum, s_pick;
  __shared__ int s_first, s_lastfalse;
  const float *x = a.logits + (long long)row * a.ld;
  float *cdf = a.work + (long long)row * a.ld;
  const int V = a.V, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;

  // (1) maximum (tensor.Max), bias = -(max * inv)
  float m = -INFINITY;
  for (int i = tid; i < V; i += blockDim.x) m = fmaxf(m, x[i]);
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

  // (2) weights staged through shared memory, two buffers a round: 4 block
  //     sub-tiles for the CumulativeSum chains (warp 1, lanes 0..nb-1) and a
  //     16-lane slab for the 16 lane sums of expScaledVecFMA (warp 0).
  //     Warps 2.. produce the next round while warps 0-1 consume this one.
  const int nb = V < 4096 ? 1 : 4;
  const int bs = V < 4096 ? V : (V + 3) / 4;
  const int rounds = (bs + kFullTile - 1) / kFullTile;
  const int lrounds = (V + kFullLaneSlab - 1) / kFullLaneSlab;
  const int R = rounds > lrounds ? rounds : lrounds;
  float *buf = (float *)dsm;
  const int bufsz = 4 * (kFullTile + 1) + kFullLaneSlab;
  auto produce = [&](int r, float *dst) {
    const int pt = tid - 64, np = blockDim.x - 64;
    for (int e = pt; e < 4 * kFullTile; e += np) {
      const int b = e / kFullTile, j = e % kFullTile;
      const int i = b * bs + r * kFullTile + j;
      if (b < nb && r * kFullTile + j < bs && i < V)
        dst[b * (kFullTile + 1) + j] = exp_fma(__fadd_rn(__fmul_rn(x[i], inv), bias));
    }
    for (int e = pt; e < kFullLaneSlab; e += np) {
      const int i = r * kFullLaneSlab + e;
      if (i < V) dst[4 * (kFullTile + 1) + e] = exp_fma(__fadd_rn(__fmul_rn(x[i], inv), bias));
    }
  };
  if (warp >= 2) produce(0, buf);
  __syncthreads();
  float acc = 0.0f;  // warp 0: lane sum; warp 1: block chain
  for (int r = 0; r < R; r++) {
    float *cur = buf + (r & 1) * bufsz;
    if (warp >= 2) {
      if (r + 1 < R) produce(r + 1, buf + ((r + 1) & 1) * bufsz);
    } else if (warp == 0) {
      if (lane < 16) {
        const float *src = cur + 4 * (kFullTile + 1);
        const int lim = min(kFullLaneSlab, V - r * kFullLaneSlab);
#pragma unroll 8
        for (int e = lane; e < lim; e += 16) acc = __fadd_rn(acc, src[e]);
      }
    } else if (lane < nb) {
      const float *src = cur + lane * (kFullTile + 1);
      const int st = lane * bs + r * kFullTile;
      const int lim = min(kFullTile, min(bs - r * kFullTile, V - st));
#pragma unroll 8
      for (int j = 0; j < lim; j++) {
        acc = __fadd_rn(acc, src[j]);
        cdf[st + j] = acc;
      }
    }
    __syncthreads();
  }
  if (warp == 0) {  // tree16 of the 16 lane sums
    float v = acc;
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
    if (lane == 0) s_sum = v;
  } else if (warp == 1 && lane < 4) {
    s_bs[lane] = (lane < nb && lane * bs < V) ? acc : 0.0f;
  }
  __syncthreads();
  // (3) block offsets (cumsum.go:46-57), the pick, pickCumulativeFloat32
  const float off1 = s_bs[0];
  const float off2 = __fadd_rn(off1, s_bs[1]);
  const float off3 = __fadd_rn(off2, s_bs[2]);
  if (tid == 0) {
    unsigned long long st = a.rng[row];
    s_pick = __fmul_rn(__double2float_rn(rng_float64(st)), s_sum);
    a.rng[row] = st;
    s_first = V;
    s_lastfalse = -1;
  }
  __syncthreads();
  const float pick = s_pick;
  auto cdf_at = [&](int i) {
    const int b = nb == 1 ? 0 : i / bs;
    return b == 0 ? cdf[i] : __fadd_rn(cdf[i], b == 1 ? off1 : b == 2 ? off2 : off3);
  };
  int first = V, lastfalse = -1;
  for (int i = tid; i < V; i += blockDim.x) {
    if (pick <= cdf_at(i)) first = min(first, i);
    else lastfalse = max(lastfalse, i);
  }
  for (int o = 16; o; o >>= 1) {
    first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    lastfalse = max(lastfalse, __shfl_xor_sync(0xffffffffu, lastfalse, o));
  }
  if (lane == 0) {
    atomicMin(&s_first, first);
    atomicMax(&s_lastfalse, lastfalse);
  }
  __syncthreads();
  if (tid == 0) {
    int res;
    if (s_lastfalse < s_first) {
      res = s_first;  // the predicate is monotone: the binary search's answer
    } else {
      int lo = 0, hi = V;
      while (lo < hi) {
        const int mid = (int)((unsigned)(lo + hi) >> 1);
        if (pick <= cdf_at(mid)) hi = mid;
        else lo = mid + 1;
      }
      res = lo;
    }
    a.out[row] = res < V ? res : V - 1;
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
  for (int i = tid; i < a.V; i += blockDim.x)
    if (x[i] > bv || bi == a.V) { bv = x[i]; bi = i; }
  auto merge = [&](float ov, int oi) {
    if (oi < a.V && (bi == a.V || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  };
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    merge(ov, oi);
  }
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
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
