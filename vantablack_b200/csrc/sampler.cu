// sampler.cu -- token sampling on the device: Sampler.sample
// (src/runtime/sampler.zig:44-104) over logits that never leave HBM, so a
// decode step reads back one int32 per sequence instead of f32[vocab].
//
// Pipeline per row (a cluster of C 1024-thread CTAs per row, C = 8, 4 or 1
// by row count and length; each CTA owns a contiguous slice; reductions,
// histograms and prefix sums are folded across the cluster through
// distributed shared memory between cluster barriers, in rank order so every
// CTA holds the same bits; logits rewritten in place as the reference does):
//   temperature == 0     -> argmax, first index of the maximum (math.zig:190-201)
//   scale by 1/T         (sampler.zig:50-51; 1/T computed on the host in f32)
//   top-k                (:54-63) the k-th largest value found by a 4-pass radix
//                        select on order-preserving 32-bit keys (exact, equal to
//                        the value at sorted position k-1); values below it
//                        become probability 0, as -inf does through the softmax
//   softmax              (math.zig:136-150) expf, block-reduced sum, 1/sum
//   top-p                (:68-89) the nucleus cut located by a second radix walk
//                        over the probabilities' bit patterns, descending, with
//                        per-bucket sums in 2^-31 fixed point (integer adds, so
//                        the cut is the same on every run); ties at the cut
//                        value are kept in ascending index order, which is the
//                        stable sort's order; then renormalise
//   CDF walk             (:92-103) first index with u <= running sum, from a
//                        scan over contiguous per-warp chunks (coalesced loads,
//                        shuffle scans); if u is never reached, the last index
//                        with nonzero mass
//
// The uniform draw u (the reference's prng.random().float(f32), :92) is an
// argument: the caller owns the generator.  Sums are formed in a different
// order than the reference's sequential f32 loops (whose own rounding drifts
// ~3e-4 relative over a 128k vocabulary; these sums sit closer to exact), so
// probabilities agree to that level, the nucleus set agrees except for
// entries whose preceding mass is that close to top_p, and the token agrees
// unless u falls that close to a CDF boundary; argmax and the top-k threshold
// are exact.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace vtb {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_MAX_ROWS = 256;
constexpr float SMP_FX = 2147483648.0f;  // 2^31: fixed-point scale of the nucleus sums (total mass <= 1 fits u32)

struct SampleArgs {
  float inv_t;
  int greedy;
  int top_k;    // 0: off
  float top_p;  // applied when use_p
  int use_p;
  float u[SMP_MAX_ROWS];
};

// Order-preserving key of a float (larger float -> larger key); -0 folds onto
// +0 so that they compare equal, as the reference's float comparisons do.
__device__ __forceinline__ uint32_t smp_key(float f) {
  uint32_t b = __float_as_uint(f);
  if (f == 0.f) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float smp_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SmpShared {
  uint32_t cnt[256];  // this CTA's radix histogram (read by the whole cluster)
  uint32_t sum[256];
  uint32_t merged[256];  // the cluster's histogram, folded here before a pick
  float red[32];
  int redi[32];
  float pub_f;        // this CTA's contribution to a cluster reduction
  int pub_i;
  long long pub_l;
  uint32_t prefix, mask, remaining;  // radix walk state, identical in every CTA of the cluster
  unsigned long long above;
  int nocut;
  float bcast, cbf;
  int bcasti, cbi;
  long long cbl;
};

__device__ __forceinline__ float smp_block_sum(float v, SmpShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = sh.red[lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh.bcast = v;
  }
  __syncthreads();
  return sh.bcast;
}

__device__ __forceinline__ float smp_block_max(float v, SmpShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = sh.red[lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sh.bcast = v;
  }
  __syncthreads();
  return sh.bcast;
}

// Block minimum (MIN = true) or maximum of an int.
template <bool MIN>
__device__ __forceinline__ int smp_block_int(int v, SmpShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const int w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MIN ? min(v, w) : max(v, w);
  }
  if (lane == 0) sh.redi[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = sh.redi[lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const int w = __shfl_xor_sync(0xffffffffu, v, o);
      v = MIN ? min(v, w) : max(v, w);
    }
    if (lane == 0) sh.bcasti = v;
  }
  __syncthreads();
  return sh.bcasti;
}

// Cluster-wide combination of a CTA-uniform value: every CTA publishes its
// value, then each CTA folds all of them in rank order (ranks [0, upto) for a
// prefix), so every CTA gets the same bits.  Two cluster barriers: one before
// the reads, one before a slot can be rewritten.
enum SmpOp { SMP_SUM, SMP_MAX, SMP_MIN };
template <int C>
__device__ __forceinline__ void smp_csync(cg::cluster_group& cl) {
  if constexpr (C == 1) __syncthreads();
  else cl.sync();
}

template <int C, SmpOp OP, typename T>
__device__ __forceinline__ T smp_cluster(T v, T& pub, T& out, cg::cluster_group& cl, int upto = C) {
  if constexpr (C == 1) return (OP == SMP_SUM && upto == 0) ? T(0) : v;  // one CTA: nothing to fold
  if (threadIdx.x == 0) pub = v;
  cl.sync();
  if (threadIdx.x == 0) {
    T acc = OP == SMP_SUM ? T(0) : *cl.map_shared_rank(&pub, 0);
    for (int r = OP == SMP_SUM ? 0 : 1; r < upto; ++r) {
      const T o = *cl.map_shared_rank(&pub, r);
      acc = OP == SMP_SUM ? acc + o : (OP == SMP_MAX ? (o > acc ? o : acc) : (o < acc ? o : acc));
    }
    out = acc;
  }
  cl.sync();
  return out;
}

// One radix level over the cluster's merged histograms, descending.  256
// threads each fold one bin over the cluster's CTAs (integers: any order gives
// the same totals); then warp 0 of every CTA picks the highest bin at which
// the running total (COUNT: counts against sh.remaining; else sums added to
// sh.above against target) is reached and narrows prefix/mask to it; with no
// such bin it sets sh.nocut.  The caller's cluster barriers bracket it.
template <int C, bool COUNT>
__device__ __forceinline__ void smp_pick_bin(SmpShared& sh, int shift, unsigned long long target,
                                             cg::cluster_group& cl) {
  const int lane = threadIdx.x & 31;
  const uint32_t* hist = COUNT ? sh.cnt : sh.sum;
  if constexpr (C > 1) {
    if (threadIdx.x < 256) {
      uint32_t t = 0;
#pragma unroll
      for (int r = 0; r < C; ++r) t += cl.map_shared_rank(hist, r)[threadIdx.x];
      sh.merged[threadIdx.x] = t;
    }
    __syncthreads();
    hist = sh.merged;
  }
  if (threadIdx.x < 32) {
    // lane l owns bins 255-8l down to 248-8l
    unsigned long long v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = hist[255 - 8 * lane - j];
    unsigned long long s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += v[j];
    unsigned long long c = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long w = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) c += w;
    }
    const unsigned long long base = COUNT ? 0ull : sh.above;
    const unsigned long long need = COUNT ? (unsigned long long)sh.remaining : target;
    const unsigned ball = __ballot_sync(0xffffffffu, base + c >= need);
    if (ball == 0u) {
      if (lane == 0) sh.nocut = 1;
    } else if (lane == __ffs(ball) - 1) {
      unsigned long long run = c - s;  // total of the higher lanes' bins
      int j = 0;
      for (; j < 7; ++j) {
        if (base + run + v[j] >= need) break;
        run += v[j];
      }
      const int b = 255 - 8 * lane - j;
      if (COUNT) sh.remaining -= (uint32_t)run;
      else sh.above += run;
      sh.prefix |= (uint32_t)b << shift;
      sh.mask |= 255u << shift;
    }
  }
  __syncthreads();
}

template <int V>
__device__ __forceinline__ void smp_ld(const float* p, float (&x)[V]) {
  if constexpr (V == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
  } else {
    x[0] = *p;
  }
}
template <int V>
__device__ __forceinline__ void smp_st(float* p, const float (&x)[V]) {
  if constexpr (V == 4) *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  else *p = x[0];
}

// A cluster of C CTAs (C SMs) samples one row: CTA `rank` owns the
// contiguous units [u0, u1) (units of V floats; V = 4 for rows of a multiple
// of 4 floats on 16-byte boundaries, read as float4).  Index order is (rank,
// warp, step, lane, element), so the scans below walk the row in order.  The
// row keeps the raw logits until the softmax pass; 1/T and 1/sum are
// re-applied on the fly (the same f32 products each time).
template <int V, int C>
__global__ void __cluster_dims__(C, 1, 1) __launch_bounds__(SMP_THREADS, 1)
sample_kernel(float* __restrict__ logits, long long ld, int n, const __grid_constant__ SampleArgs a,
              int32_t* __restrict__ tokens) {
  __shared__ SmpShared sh;
  __shared__ float ftot[32];
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank(), row = blockIdx.x / C;
  float* L = logits + (long long)row * ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nu = n / V;
  const int u0 = (int)((long long)rank * nu / C), u1 = (int)((long long)(rank + 1) * nu / C);

  if (a.greedy) {  // argmax: largest value, first index on ties
    float bv = -INFINITY;
    int bi = n;
    for (int u = u0 + tid; u < u1; u += SMP_THREADS) {
      float x[V];
      smp_ld<V>(L + u * V, x);
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (bi == n || x[k] > bv) { bv = x[k]; bi = u * V + k; }  // ascending: this thread's first maximum
    }
    const float mc = smp_block_max(bv, sh);
    const int ic = smp_block_int<true>((bv == mc && bi < n) ? bi : n, sh);
    const float m = smp_cluster<C, SMP_MAX>(mc, sh.pub_f, sh.cbf, cl);
    const int idx = smp_cluster<C, SMP_MIN>(mc == m ? ic : n, sh.pub_i, sh.cbi, cl);
    if (rank == 0 && tid == 0) tokens[row] = idx < n ? idx : 0;
    return;
  }

  // Maximum of the scaled logits (masking keeps it, so it is the softmax's).
  const float inv_t = a.inv_t;
  float mx = -INFINITY;
  for (int u = u0 + tid; u < u1; u += SMP_THREADS) {
    float x[V];
    smp_ld<V>(L + u * V, x);
#pragma unroll
    for (int k = 0; k < V; ++k) mx = fmaxf(mx, x[k] * inv_t);
  }
  mx = smp_cluster<C, SMP_MAX>(smp_block_max(mx, sh), sh.pub_f, sh.cbf, cl);

  // top-k threshold: the k-th largest scaled value of the whole row.
  float thr = -INFINITY;
  const bool use_k = a.top_k > 0 && a.top_k < n;
  if (use_k) {
    if (tid == 0) { sh.prefix = 0u; sh.mask = 0u; sh.remaining = (uint32_t)a.top_k; sh.nocut = 0; }
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += SMP_THREADS) sh.cnt[b] = 0u;
      __syncthreads();
      const uint32_t pre = sh.prefix, msk = sh.mask;
      for (int u = u0 + tid; u < u1; u += SMP_THREADS) {
        float x[V];
        smp_ld<V>(L + u * V, x);
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const uint32_t key = smp_key(x[k] * inv_t);
          if ((key & msk) == pre) atomicAdd(&sh.cnt[(key >> shift) & 255u], 1u);
        }
      }
      smp_csync<C>(cl);  // every CTA's histogram is complete
      smp_pick_bin<C, true>(sh, shift, 0ull, cl);
      smp_csync<C>(cl);  // nobody reads a histogram any more
    }
    thr = smp_unkey(sh.prefix);
  }

  // softmax numerators (masked entries are exp(-inf) = 0 in the reference).
  float s = 0.f;
  for (int u = u0 + tid; u < u1; u += SMP_THREADS) {
    float x[V];
    smp_ld<V>(L + u * V, x);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float v = x[k] * inv_t;
      x[k] = (use_k && v < thr) ? 0.f : expf(v - mx);
      s += x[k];
    }
    smp_st<V>(L + u * V, x);
  }
  const float inv = 1.0f / smp_cluster<C, SMP_SUM>(smp_block_sum(s, sh), sh.pub_f, sh.cbf, cl);

  // Warp w owns the contiguous units [w0, w1) of this CTA's slice, walked 32
  // units (one coalesced load per lane) at a time.
  const int cw = ((u1 - u0 + SMP_THREADS - 1) / SMP_THREADS) * 32;
  const int w0 = min(u1, u0 + warp * cw), w1 = min(u1, w0 + cw);
  float renorm = 1.f;
  bool use_renorm = false;
  if (a.use_p) {  // nucleus over p = e * inv
    const unsigned long long target = (unsigned long long)ceil((double)a.top_p * (double)SMP_FX);
    if (tid == 0) { sh.prefix = 0u; sh.mask = 0u; sh.above = 0ull; sh.nocut = 0; }
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += SMP_THREADS) sh.sum[b] = 0u;
      __syncthreads();
      if (sh.nocut) break;  // identical in every CTA
      const uint32_t pre = sh.prefix, msk = sh.mask;
      for (int u = u0 + tid; u < u1; u += SMP_THREADS) {
        float x[V];
        smp_ld<V>(L + u * V, x);
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const float p = x[k] * inv;
          const uint32_t key = __float_as_uint(p);  // p >= +0: the raw bits order like the values
          if ((key & msk) == pre) atomicAdd(&sh.sum[(key >> shift) & 255u], __float2uint_rn(p * SMP_FX));
        }
      }
      smp_csync<C>(cl);
      smp_pick_bin<C, false>(sh, shift, target, cl);
      smp_csync<C>(cl);
    }
    const bool nocut = sh.nocut != 0;
    const uint32_t kstar = sh.prefix;
    // Ties at the cut value to keep: the fewest that reach the target.
    long long keep_ties = 0;
    if (!nocut) {
      const unsigned long long vfx = __float2uint_rn(__uint_as_float(kstar) * SMP_FX);
      const unsigned long long rest = target - sh.above;  // > 0 by construction
      keep_ties = vfx ? (long long)((rest + vfx - 1) / vfx) : 1;
      if (keep_ties < 1) keep_ties = 1;
    }
    // Rank of this warp's first tie among all ties of the row, in index order.
    int my_ties = 0;
    if (!nocut)
      for (int j = w0; j < w1; j += 32) {
        const int u = j + lane;
        if (u < w1) {
          float x[V];
          smp_ld<V>(L + u * V, x);
#pragma unroll
          for (int k = 0; k < V; ++k) my_ties += __float_as_uint(x[k] * inv) == kstar;
        }
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) my_ties += __shfl_xor_sync(0xffffffffu, my_ties, o);
    if (lane == 0) sh.redi[warp] = my_ties;
    __syncthreads();
    long long rank_in = 0, cta_ties = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) rank_in += sh.redi[w];
      cta_ties += sh.redi[w];
    }
    __syncthreads();
    long long tie_rank = rank_in + smp_cluster<C, SMP_SUM>(cta_ties, sh.pub_l, sh.cbl, cl, rank);
    // Keep or zero each p; the slice now holds the nucleus probabilities.
    float kept = 0.f;
    for (int j = w0; j < w1; j += 32) {
      const int u = j + lane;
      float x[V];
      int tl = 0;
      if (u < w1) {
        smp_ld<V>(L + u * V, x);
#pragma unroll
        for (int k = 0; k < V; ++k) { x[k] *= inv; tl += __float_as_uint(x[k]) == kstar; }
      }
      int ex = tl;  // ties of the lower lanes of this step
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int w = __shfl_up_sync(0xffffffffu, ex, o);
        if (lane >= o) ex += w;
      }
      const int step_ties = __shfl_sync(0xffffffffu, ex, 31);
      ex -= tl;
      if (u < w1) {
        long long r = tie_rank + ex;
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const uint32_t key = __float_as_uint(x[k]);
          bool keep = true;
          if (!nocut) {
            keep = key > kstar;
            if (key == kstar) keep = r++ < keep_ties;
          }
          if (!keep) x[k] = 0.f;
          kept += x[k];
        }
        smp_st<V>(L + u * V, x);
      }
      tie_rank += step_ties;
    }
    const float tot = smp_cluster<C, SMP_SUM>(smp_block_sum(kept, sh), sh.pub_f, sh.cbf, cl);
    if (tot > 0.f) { use_renorm = true; renorm = 1.0f / tot; }
  }

  // CDF walk: final probabilities written back, warp totals, the mass of the
  // lower CTAs and warps, then each warp scans its range until the sum reaches u.
  float cs = 0.f;
  int last = -1;
  for (int j = w0; j < w1; j += 32) {
    const int u = j + lane;
    if (u < w1) {
      float x[V];
      smp_ld<V>(L + u * V, x);
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (!a.use_p) x[k] *= inv;
        else if (use_renorm) x[k] *= renorm;
        cs += x[k];
        if (x[k] > 0.f) last = u * V + k;
      }
      smp_st<V>(L + u * V, x);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
  if (lane == 0) ftot[warp] = cs;
  __syncthreads();  // also publishes this CTA's final slice
  float cta_mass = 0.f, acc = 0.f;
  for (int w = 0; w < 32; ++w) {
    if (w == warp) acc = cta_mass;
    cta_mass += ftot[w];
  }
  acc += smp_cluster<C, SMP_SUM>(cta_mass, sh.pub_f, sh.cbf, cl, rank);
  const float ud = a.u[row];
  int cand = n;
  for (int j = w0; j < w1; j += 32) {
    const int u = j + lane;
    float x[V];
    float lt = 0.f;
    if (u < w1) {
      smp_ld<V>(L + u * V, x);
#pragma unroll
      for (int k = 0; k < V; ++k) lt += x[k];
    }
    float inc = lt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float w = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += w;
    }
    float run = acc + __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) run = acc;
    int hit = -1;
    if (u < w1) {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        run += x[k];
        if (hit < 0 && ud <= run) hit = k;
      }
    }
    const unsigned hb = __ballot_sync(0xffffffffu, hit >= 0);
    if (hb) {
      const int fl = __ffs(hb) - 1;
      cand = (j + fl) * V + __shfl_sync(0xffffffffu, hit, fl);
      break;
    }
    acc += __shfl_sync(0xffffffffu, inc, 31);
  }
  cand = smp_cluster<C, SMP_MIN>(smp_block_int<true>(cand, sh), sh.pub_i, sh.cbi, cl);
  last = smp_cluster<C, SMP_MAX>(smp_block_int<false>(last, sh), sh.pub_i, sh.cbi, cl);
  if (rank == 0 && tid == 0) tokens[row] = cand < n ? cand : (last >= 0 ? last : 0);
}

// Host side: argument checks happen in the extern "C" wrappers.
cudaError_t launch_sample(float* logits, long long ld, int rows, int n, float temperature, long long top_k,
                          float top_p, const float* u, int32_t* tokens, cudaStream_t st) {
  SampleArgs a{};
  a.greedy = temperature == 0.0f;
  a.inv_t = a.greedy ? 1.0f : 1.0f / temperature;
  a.top_k = (top_k > 0 && top_k < n) ? (int)top_k : 0;
  a.top_p = top_p;
  a.use_p = top_p > 0.0f && top_p < 1.0f;
  for (int r = 0; r < rows; ++r) a.u[r] = u ? u[r] : 0.f;
  const bool vec = n % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  // CTAs per row: as many as keep every row's cluster in one wave of the GPU
  // and give each CTA at least 12k values (below that the cluster barriers
  // cost more than the extra SMs' bandwidth returns).
  const int sms = sm_count(current_device());
  int C = 1;
  if (rows * 8 <= sms && n >= 8 * 12288) C = 8;
  else if (rows * 4 <= sms && n >= 4 * 12288) C = 4;
  const dim3 grid(rows * C);
  if (vec) {
    if (C == 8) sample_kernel<4, 8><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
    else if (C == 4) sample_kernel<4, 4><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
    else sample_kernel<4, 1><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
  } else {
    if (C == 8) sample_kernel<1, 8><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
    else if (C == 4) sample_kernel<1, 4><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
    else sample_kernel<1, 1><<<grid, SMP_THREADS, 0, st>>>(logits, ld, n, a, tokens);
  }
  return cudaGetLastError();
}

}  // namespace vtb

using namespace vtb;

static int check_sampler(const VtbCudaSamplerConfig* cfg, const float* u, int64_t rows, int64_t n) {
  if (!cfg) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null sampler config");
  if (!(cfg->temperature >= 0.0f) || !(cfg->top_p >= 0.0f))  // rejects NaN too
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "temperature and top_p must be >= 0");
  if (rows < 1 || rows > SMP_MAX_ROWS) return set_err(VTB_CUDA_ERR_INVALID_ARG, "rows must be in [1, 256]");
  if (n < 1 || n > (1 << 24)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "n must be in [1, 2^24]");
  if (cfg->temperature != 0.0f && !u) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null uniform draws");
  return VTB_CUDA_OK;
}

extern "C" {

int vtb_cuda_sample(float* logits, int64_t rows, int64_t n, int64_t ld, const VtbCudaSamplerConfig* cfg,
                    const float* u, int32_t* tokens, void* stream) {
  cudaGetLastError();
  int rc = check_sampler(cfg, u, rows, n);
  if (rc) return rc;
  if (!logits || !tokens) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null logits or tokens");
  if (ld < n) return set_err(VTB_CUDA_ERR_INVALID_ARG, "row stride ld is below n");
  return cuda_status(launch_sample(logits, ld, (int)rows, (int)n, cfg->temperature, (long long)cfg->top_k,
                                   cfg->top_p, u, tokens, (cudaStream_t)stream));
}

int vtb_cuda_state_sample(VtbCudaState* s, int32_t rows, const VtbCudaSamplerConfig* cfg, const float* u,
                          int32_t* tokens) {
  cudaGetLastError();
  if (!s || !tokens) return merr(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  const int64_t V = s->m->c.vocab_size;
  int rc = check_sampler(cfg, u, rows, V);
  if (rc) return rc;
  if (rows > s->max_rows) return merr(VTB_CUDA_ERR_INVALID_ARG, "rows exceed the state's logits rows");
  cudaSetDevice(s->m->device);
  // s->amax / s->hamax are the argmax buffers (max_rows int32, device and pinned host).
  cudaError_t e = launch_sample(s->logits, V, rows, (int)V, cfg->temperature, (long long)cfg->top_k, cfg->top_p,
                                u, s->amax, s->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(s->hamax, s->amax, (size_t)rows * 4, cudaMemcpyDeviceToHost, s->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
  if (e != cudaSuccess) return mcuda(e);
  memcpy(tokens, s->hamax, (size_t)rows * 4);
  return VTB_CUDA_OK;
}

}  // extern "C"
