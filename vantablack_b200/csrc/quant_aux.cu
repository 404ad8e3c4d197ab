// quant_aux.cu -- bit-exact dequantization, the Q8_0 activation quantizer
// and per-block int32 dots.
//
// dequant_*: one thread per weight, arithmetic in the reference's order with
// explicit round-to-nearest intrinsics (no FMA contraction), so the values
// are bit-identical to dequantBlockQ*_* (src/kernels/simd.zig:153-404).
#include "common.cuh"

namespace vtb {

__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

__device__ __forceinline__ void scale_min_k4(int s, const uint8_t* sc, unsigned& d, unsigned& m) {
  if (s < 4) {
    d = sc[s] & 63u;
    m = sc[s + 4] & 63u;
  } else {
    d = (sc[s + 4] & 15u) | ((unsigned)(sc[s - 4] >> 6) << 4);
    m = (sc[s + 4] >> 4) | ((unsigned)(sc[s] >> 6) << 4);
  }
}

// Element e (0..255) of one K-quant super-block / element of a Q8_0 block.
template <int Q>
__device__ __forceinline__ float dequant_elem(const uint8_t* blk, int e) {
  if constexpr (Q == Q8_0) {
    return __fmul_rn(h2f(ld16(blk)), (float)(int8_t)blk[2 + e]);
  } else if constexpr (Q == Q4_K || Q == Q5_K) {
    const float d = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
    const int s = e >> 5, l = e & 31;  // sub-block s, position l
    unsigned sc, mn;
    scale_min_k4(s, blk + 4, sc, mn);
    const uint8_t* qs = blk + (Q == Q4_K ? 16 : 48) + (s >> 1) * 32;
    unsigned q = (s & 1) ? (qs[l] >> 4) : (qs[l] & 15u);
    if constexpr (Q == Q5_K) q += (blk[16 + l] >> s) & 1u ? 16u : 0u;
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
  } else if constexpr (Q == TQ2_0) {  // dequantBlockTQ2_0, simd.zig:457-472
    const int g = e >> 6, l = e & 63;
    const unsigned raw = (blk[16 * g + (l & 15)] >> (2 * g)) & 3u;
    return __fmul_rn(h2f(ld16(blk + 64)), (float)((int)raw - 1));
  } else {  // Q6_K
    const float d = h2f(ld16(blk + 208));
    const int half = e >> 7, r = e & 127, n = r >> 5, l = r & 31;
    const uint8_t* ql = blk + half * 64;
    const uint8_t qh = blk[128 + half * 32 + l];
    const int8_t sc = (int8_t)blk[192 + half * 8 + (l >> 4) + 2 * n];
    unsigned lo = (n & 1) ? ql[l + 32] : ql[l];
    lo = (n & 2) ? (lo >> 4) : (lo & 15u);
    const int q = (int)(lo | (((qh >> (2 * n)) & 3u) << 4)) - 32;
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
  }
}

template <int Q>
__global__ void dequant_kernel(const uint8_t* __restrict__ w, float* __restrict__ out, long long n) {
  constexpr int EL = Fmt<Q>::elems, BB = Fmt<Q>::bytes;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = dequant_elem<Q>(w + (i / EL) * BB, (int)(i % EL));
}

// Gather-and-dequantize rows `ids[t]` of a [rows, dim] table into out[t, dim]
// (gatherEmbedding, forward.zig:738-845).
template <int Q>
__global__ void embed_kernel(const uint8_t* __restrict__ table, const int32_t* __restrict__ ids, float* __restrict__ out,
                             int dim, int n_tok) {
  VTB_TL(18);
  constexpr int EL = Fmt<Q>::elems, BB = Fmt<Q>::bytes;
  const long long rb = (long long)(dim / EL) * BB;
  const int t = blockIdx.y;
  if (t >= n_tok) return;
  const uint8_t* row = table + (long long)ids[t] * rb;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    out[(long long)t * dim + i] = dequant_elem<Q>(row + (i / EL) * BB, i % EL);
}

// Q8_0 activation quantizer, one warp per 32-block: d = max|x|/127,
// q = round-half-away(x * (1/d)) (the rule the oracle defines).
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int8_t* __restrict__ qs, float* __restrict__ d,
                                     int nblocks) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= nblocks) return;
  const float v = x[b * 32 + lane];
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float dd = __fdiv_rn(a, 127.0f);
  const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
  qs[b * 32 + lane] = (int8_t)roundf(__fmul_rn(v, id));
  if (lane == 0) d[b] = dd;
}

// dots[i, b] = sum_j w_qs[i, b, j] * xq[b, j] (int32, dot_i8 simd.zig:40-62).
__global__ void q8_0_block_dots_kernel(const uint8_t* __restrict__ w, const int8_t* __restrict__ xq,
                                       int32_t* __restrict__ dots, int m, int nb) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)m * nb) return;
  const long long row = i / nb;
  const int b = (int)(i % nb);
  const uint8_t* blk = w + row * nb * 34 + (long long)b * 34 + 2;
  int acc = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int wv = (int)((uint32_t)blk[4 * t] | ((uint32_t)blk[4 * t + 1] << 8) | ((uint32_t)blk[4 * t + 2] << 16) |
                         ((uint32_t)blk[4 * t + 3] << 24));
    const int xv = *reinterpret_cast<const int*>(xq + b * 32 + 4 * t);
    acc = __dp4a(wv, xv, acc);
  }
  dots[i] = acc;
}

static int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  return (int)(g > 148LL * 64 ? 148LL * 64 : (g < 1 ? 1 : g));
}

cudaError_t launch_dequant(int q, const void* w, float* out, long long n, cudaStream_t st) {
  const uint8_t* p = static_cast<const uint8_t*>(w);
  const int g = grid_for(n, 256);
  switch (q) {
    case Q8_0: dequant_kernel<Q8_0><<<g, 256, 0, st>>>(p, out, n); break;
    case Q4_K: dequant_kernel<Q4_K><<<g, 256, 0, st>>>(p, out, n); break;
    case Q5_K: dequant_kernel<Q5_K><<<g, 256, 0, st>>>(p, out, n); break;
    case Q6_K: dequant_kernel<Q6_K><<<g, 256, 0, st>>>(p, out, n); break;
    case TQ2_0: dequant_kernel<TQ2_0><<<g, 256, 0, st>>>(p, out, n); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_embed(int q, const void* table, const int32_t* ids, float* out, int dim, int n_tok,
                         cudaStream_t st) {
  const uint8_t* p = static_cast<const uint8_t*>(table);
  dim3 grid((dim + 255) / 256, n_tok);
  switch (q) {
    case Q8_0: embed_kernel<Q8_0><<<grid, 256, 0, st>>>(p, ids, out, dim, n_tok); break;
    case Q4_K: embed_kernel<Q4_K><<<grid, 256, 0, st>>>(p, ids, out, dim, n_tok); break;
    case Q5_K: embed_kernel<Q5_K><<<grid, 256, 0, st>>>(p, ids, out, dim, n_tok); break;
    case Q6_K: embed_kernel<Q6_K><<<grid, 256, 0, st>>>(p, ids, out, dim, n_tok); break;
    case TQ2_0: embed_kernel<TQ2_0><<<grid, 256, 0, st>>>(p, ids, out, dim, n_tok); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0(const float* x, int8_t* qs, float* d, int nblocks, cudaStream_t st) {
  quantize_q8_0_kernel<<<(nblocks + 7) / 8, 256, 0, st>>>(x, qs, d, nblocks);
  return cudaGetLastError();
}

cudaError_t launch_q8_0_block_dots(const void* w, const int8_t* xq, int32_t* dots, int m, int nb, cudaStream_t st) {
  const long long n = (long long)m * nb;
  q8_0_block_dots_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint8_t*>(w), xq, dots, m, nb);
  return cudaGetLastError();
}

}  // namespace vtb
