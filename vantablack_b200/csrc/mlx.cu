// mlx.cu -- MLX affine-quantized GEMV and dequant (src/kernels/mlx.zig; the
// Metal counterpart is matmul_mlx_q4, src/metal/bridge.m:245-291).
//
// Layout (mlx.zig:3-23): a row of k columns is k / EL little-endian u32 words,
// EL = 32 / bits values per word, low bits first (for 3, 5 and 6 bits the top
// 32 % bits bits of a word are unused); per group of G columns one scale and
// one bias, f16 or bf16; w = q * scale + bias.  Tensors come from safetensors
// shards, so their byte offsets need not be aligned: the kernels read words
// with 32-bit loads only when the weight pointer is 4-byte aligned, and
// assemble them from bytes otherwise; scales and biases are always read as
// byte pairs.
//
// GEMV (any width): one warp owns R = 4 rows; lanes stride over the rows' words (one
// coalesced 128-byte line per row per warp step).  A word's activations and
// their sum are loaded once and shared by the four rows; per row and word,
// y += scale * sum(q * x) + bias * sum(x) (the reference's per-group
// factoring, mlx.zig:186-199, applied per word).  q is turned into a float
// with the 2^23 mantissa trick (or-in the exponent, subtract 2^23: exact for
// q < 2^23) instead of an integer conversion.  4-bit rows on 16-byte
// boundaries take gemv_mlx_q4_vec_kernel (16-byte loads, 32 weights per lane
// per row).  HBM-bound: 0.5 B per 4-bit weight plus 4 B per group.
//
// Dequant: one thread per word, out = q * scale + bias as a separate multiply
// and add (no contraction), bit-exact with dequantRow (mlx.zig:62-135).
#include "common.cuh"

namespace vtb {

constexpr int MLX_WARPS = 8, MLX_ROWS = 4;

__device__ __forceinline__ float mlx_half(const uint8_t* p, long long idx, bool bf16) {
  const uint32_t b = (uint32_t)__ldg(p + 2 * idx) | ((uint32_t)__ldg(p + 2 * idx + 1) << 8);
  if (bf16) return __uint_as_float(b << 16);
  return __half2float(__ushort_as_half((unsigned short)b));
}

template <bool AL>
__device__ __forceinline__ uint32_t mlx_word(const uint8_t* p, long long idx) {
  if constexpr (AL) return __ldg(reinterpret_cast<const uint32_t*>(p) + idx);
  const uint8_t* q = p + 4 * idx;
  return (uint32_t)__ldg(q) | ((uint32_t)__ldg(q + 1) << 8) | ((uint32_t)__ldg(q + 2) << 16) |
         ((uint32_t)__ldg(q + 3) << 24);
}

__device__ __forceinline__ float mlx_qf(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

template <int BITS, bool AL>
__global__ void __launch_bounds__(MLX_WARPS * 32)
gemv_mlx_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sc, const uint8_t* __restrict__ bi,
                const float* __restrict__ x, float* __restrict__ y, int m, int k, int group, int gshift, int bf16) {
  constexpr int EL = 32 / BITS;
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  const int lane = threadIdx.x & 31;
  const int wpr = k / EL, ng = k / group;
  const long long row_bytes = (long long)wpr * 4;
  for (int r0 = (blockIdx.x * MLX_WARPS + (threadIdx.x >> 5)) * MLX_ROWS; r0 < m;
       r0 += gridDim.x * MLX_WARPS * MLX_ROWS) {
    const int nr = min(MLX_ROWS, m - r0);
    float acc[MLX_ROWS] = {0.f, 0.f, 0.f, 0.f};
    for (int wd = lane; wd < wpr; wd += 32) {
      const int col = wd * EL;
      float xv[EL];
      if constexpr (EL % 4 == 0) {
#pragma unroll
        for (int i = 0; i < EL / 4; ++i) {
          const float4 t = __ldg(reinterpret_cast<const float4*>(x + col) + i);
          xv[4 * i] = t.x; xv[4 * i + 1] = t.y; xv[4 * i + 2] = t.z; xv[4 * i + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < EL; ++i) xv[i] = __ldg(x + col + i);
      }
      float xs = 0.f;
#pragma unroll
      for (int i = 0; i < EL; ++i) xs += xv[i];
      const int g = gshift >= 0 ? (col >> gshift) : col / group;
#pragma unroll
      for (int r = 0; r < MLX_ROWS; ++r) {
        if (r < nr) {
          const long long row = r0 + r;
          const uint32_t word = mlx_word<AL>(w + row * row_bytes, wd);
          float qd = 0.f;
#pragma unroll
          for (int i = 0; i < EL; ++i) qd = fmaf(mlx_qf((word >> (i * BITS)) & MASK), xv[i], qd);
          const float s = mlx_half(sc, row * ng + g, bf16), b = mlx_half(bi, row * ng + g, bf16);
          acc[r] = fmaf(s, qd, fmaf(b, xs, acc[r]));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < MLX_ROWS; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == r && r < nr) y[r0 + r] = v;
    }
  }
}

// 4-bit rows on 16-byte boundaries with group % 32 == 0: a lane takes 32
// consecutive weights of a row (16 bytes, inside one group) for each of the
// warp's 4 rows, so a group's scale and bias are read once per 32 weights and
// the 32 activations once per 4 rows.  Weights stream through a per-warp
// MLX_STAGES-deep ring of cp.async copies (each lane copies and later reads
// only its own 16-byte slots, so the per-thread async-copy groups order
// everything).  Nibbles become floats with one byte-permute each (low and
// high nibble planes masked once per word, byte p placed under 0x4B000000),
// and the products run as packed f32x2 FMAs.
//
// x is staged once per CTA in shared memory, float4 slot i of 32-column chunk
// c stored at c*8 + (i ^ (c & 7)): a warp reading eight float4 of 32 different
// chunks then needs 4 wavefronts per load (the minimum for 512 bytes) instead
// of one per lane, which is what direct global loads of 128 contiguous bytes
// per lane cost.  The chunk sums of x are computed once there as well.
constexpr int MLX_STAGES = 3;
constexpr int MLX_RING = MLX_WARPS * MLX_STAGES * MLX_ROWS * 32 * 16;  // bytes per CTA

__device__ __forceinline__ size_t mlx_q4_smem(int k) { return ((size_t)k + k / 32 + 3) / 4 * 16 + MLX_RING; }
static size_t mlx_q4_smem_host(int k) { return ((size_t)k + k / 32 + 3) / 4 * 16 + MLX_RING; }

__device__ __forceinline__ void mlx_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void mlx_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void mlx_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <bool H2>
__device__ __forceinline__ void mlx_sb(const uint8_t* __restrict__ sc, const uint8_t* __restrict__ bi, long long gi,
                                       int bf16, float& s, float& b) {
  if constexpr (H2) {
    const uint32_t sb = __ldg(reinterpret_cast<const unsigned short*>(sc) + gi);
    const uint32_t bb = __ldg(reinterpret_cast<const unsigned short*>(bi) + gi);
    s = bf16 ? __uint_as_float(sb << 16) : __half2float(__ushort_as_half((unsigned short)sb));
    b = bf16 ? __uint_as_float(bb << 16) : __half2float(__ushort_as_half((unsigned short)bb));
  } else {
    s = mlx_half(sc, gi, bf16);
    b = mlx_half(bi, gi, bf16);
  }
}

template <bool H2>
__global__ void __launch_bounds__(MLX_WARPS * 32)
gemv_mlx_q4_vec_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sc,
                       const uint8_t* __restrict__ bi, const float* __restrict__ x, float* __restrict__ y, int m,
                       int k, int group, int gshift, int bf16) {
  extern __shared__ __align__(16) float xsm[];  // [k] swizzled x, [k / 32] chunk sums, then the weight rings
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nch = k / 32, ng = k / group;
  float4* x4 = reinterpret_cast<float4*>(xsm);
  float* csum = xsm + k;
  uint8_t* ring = reinterpret_cast<uint8_t*>(xsm) + (mlx_q4_smem(k) - MLX_RING) +
                  warp * (MLX_STAGES * MLX_ROWS * 32 * 16);
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring) + lane * 16;
  for (int q = threadIdx.x; q < k / 4; q += blockDim.x) {
    const int c = q >> 3, i = q & 7;
    x4[c * 8 + (i ^ (c & 7))] = __ldg(reinterpret_cast<const float4*>(x) + q);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < nch; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = x4[c * 8 + (i ^ (c & 7))];
      t += (v.x + v.y) + (v.z + v.w);
    }
    csum[c] = t;
  }
  __syncthreads();
  const long long row_bytes = (long long)k / 2;
  const f2 magic = pk(8388608.0f, 8388608.0f);
  const int T = lane < nch ? (nch - lane + 31) / 32 : 0;  // this lane's chunks per row
  // This warp's rows: an even share of m over all the grid's warps (the grid is
  // one wave), walked MLX_ROWS at a time.
  const long long nw = (long long)gridDim.x * MLX_WARPS, gw = (long long)blockIdx.x * MLX_WARPS + warp;
  const int row_end = (int)((gw + 1) * m / nw);
  for (int r0 = (int)(gw * m / nw); r0 < row_end; r0 += MLX_ROWS) {
    const int nr = min(MLX_ROWS, row_end - r0);
    auto issue = [&](int t) {
      const int ch = lane + 32 * t, st = t % MLX_STAGES;
#pragma unroll
      for (int r = 0; r < MLX_ROWS; ++r)
        if (r < nr)
          mlx_cp16(ring_s + (uint32_t)((st * MLX_ROWS + r) * 32 * 16),
                   w + (long long)(r0 + r) * row_bytes + (long long)ch * 16);
    };
#pragma unroll
    for (int t = 0; t < MLX_STAGES - 1; ++t) {
      if (t < T) issue(t);
      mlx_cp_commit();
    }
    float acc[MLX_ROWS] = {0.f, 0.f, 0.f, 0.f};
    for (int t = 0; t < T; ++t) {
      if (t + MLX_STAGES - 1 < T) issue(t + MLX_STAGES - 1);
      mlx_cp_commit();
      const int ch = lane + 32 * t, st = t % MLX_STAGES;
      const int g = gshift >= 0 ? ((ch * 32) >> gshift) : (ch * 32) / group;
      float s[MLX_ROWS], b[MLX_ROWS];
#pragma unroll
      for (int r = 0; r < MLX_ROWS; ++r)
        if (r < nr) mlx_sb<H2>(sc, bi, (long long)(r0 + r) * ng + g, bf16, s[r], b[r]);
      f2 xv[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = x4[ch * 8 + (i ^ (ch & 7))];
        xv[2 * i] = pk(v.x, v.y);
        xv[2 * i + 1] = pk(v.z, v.w);
      }
      const float xs = csum[ch];
      mlx_cp_wait<MLX_STAGES - 1>();  // this lane's copies of chunk t have landed
#pragma unroll
      for (int r = 0; r < MLX_ROWS; ++r) {
        if (r < nr) {
          const uint4 wv = *reinterpret_cast<const uint4*>(ring + ((st * MLX_ROWS + r) * 32 + lane) * 16);
          const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
          f2 qd = pk(0.f, 0.f);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // byte p of lo / hi = the nibble of column 2p / 2p + 1 of this word
            const uint32_t lo = wd[j] & 0x0F0F0F0Fu, hi = (wd[j] >> 4) & 0x0F0F0F0Fu;
            qd = fma2(sub2(pk(byte_magic<0>(lo), byte_magic<0>(hi)), magic), xv[4 * j + 0], qd);
            qd = fma2(sub2(pk(byte_magic<1>(lo), byte_magic<1>(hi)), magic), xv[4 * j + 1], qd);
            qd = fma2(sub2(pk(byte_magic<2>(lo), byte_magic<2>(hi)), magic), xv[4 * j + 2], qd);
            qd = fma2(sub2(pk(byte_magic<3>(lo), byte_magic<3>(hi)), magic), xv[4 * j + 3], qd);
          }
          acc[r] = fmaf(s[r], hsum(qd), fmaf(b[r], xs, acc[r]));
        }
      }
    }
    mlx_cp_wait<0>();  // nothing of this row group may still be in flight when the ring is reused
#pragma unroll
    for (int r = 0; r < MLX_ROWS; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == r && r < nr) y[r0 + r] = v;
    }
  }
}

template <int BITS, bool AL>
__global__ void __launch_bounds__(256)
dequant_mlx_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sc, const uint8_t* __restrict__ bi,
                   float* __restrict__ out, long long words, int k, int group, int bf16) {
  constexpr int EL = 32 / BITS;
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  const int wpr = k / EL, ng = k / group;
  for (long long t = blockIdx.x * 256ll + threadIdx.x; t < words; t += (long long)gridDim.x * 256) {
    const long long row = t / wpr;
    const int col = (int)(t - row * wpr) * EL, g = col / group;
    const uint32_t word = mlx_word<AL>(w, t);
    const float s = mlx_half(sc, row * ng + g, bf16), b = mlx_half(bi, row * ng + g, bf16);
    float* o = out + row * k + col;
#pragma unroll
    for (int i = 0; i < EL; ++i) o[i] = __fadd_rn(__fmul_rn((float)((word >> (i * BITS)) & MASK), s), b);
  }
}

template <int BITS>
static cudaError_t launch_mlx_bits(bool gemv, const void* w, const void* sc, const void* bi, const float* x, float* y,
                                   long long rows, int k, int group, int bf16, cudaStream_t st) {
  const bool al = (reinterpret_cast<uintptr_t>(w) & 3u) == 0;
  const auto* W = static_cast<const uint8_t*>(w);
  const auto* S = static_cast<const uint8_t*>(sc);
  const auto* B = static_cast<const uint8_t*>(bi);
  if (gemv) {
    int gshift = -1;
    if ((group & (group - 1)) == 0) gshift = __builtin_ctz((unsigned)group);
    const long long per_cta = MLX_WARPS * MLX_ROWS;
    const int grid = (int)std::min<long long>((rows + per_cta - 1) / per_cta, 148ll * 16);
    const size_t vsmem = mlx_q4_smem_host(k);
    if (BITS == 4 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && group % 32 == 0 && k % 32 == 0 &&
        vsmem <= 200 * 1024) {
      const bool h2 = ((reinterpret_cast<uintptr_t>(sc) | reinterpret_cast<uintptr_t>(bi)) & 1u) == 0;
      const int dev = current_device();
      cudaError_t e = h2 ? ensure_smem_attr<gemv_mlx_q4_vec_kernel<true>>(dev, (int)vsmem)
                         : ensure_smem_attr<gemv_mlx_q4_vec_kernel<false>>(dev, (int)vsmem);
      if (e != cudaSuccess) return e;
      const int per_sm = h2 ? ctas_per_sm<gemv_mlx_q4_vec_kernel<true>>(dev, MLX_WARPS * 32, (int)vsmem)
                            : ctas_per_sm<gemv_mlx_q4_vec_kernel<false>>(dev, MLX_WARPS * 32, (int)vsmem);
      // One wave of CTAs, each warp an even share of the rows (at least MLX_ROWS rows per warp).
      const long long need = (rows + MLX_WARPS * MLX_ROWS - 1) / (MLX_WARPS * MLX_ROWS);
      const int vgrid = (int)std::min<long long>(need, (long long)sm_count(dev) * std::max(per_sm, 1));
      if (h2) gemv_mlx_q4_vec_kernel<true><<<vgrid, MLX_WARPS * 32, vsmem, st>>>(W, S, B, x, y, (int)rows, k, group, gshift, bf16);
      else gemv_mlx_q4_vec_kernel<false><<<vgrid, MLX_WARPS * 32, vsmem, st>>>(W, S, B, x, y, (int)rows, k, group, gshift, bf16);
    } else if (al) gemv_mlx_kernel<BITS, true><<<grid, MLX_WARPS * 32, 0, st>>>(W, S, B, x, y, (int)rows, k, group, gshift, bf16);
    else gemv_mlx_kernel<BITS, false><<<grid, MLX_WARPS * 32, 0, st>>>(W, S, B, x, y, (int)rows, k, group, gshift, bf16);
  } else {
    const long long words = rows * (k / (32 / BITS));
    const int grid = (int)std::min<long long>((words + 255) / 256, 148ll * 32);
    if (al) dequant_mlx_kernel<BITS, true><<<grid, 256, 0, st>>>(W, S, B, y, words, k, group, bf16);
    else dequant_mlx_kernel<BITS, false><<<grid, 256, 0, st>>>(W, S, B, y, words, k, group, bf16);
  }
  return cudaGetLastError();
}

cudaError_t launch_mlx(bool gemv, int bits, const void* w, const void* sc, const void* bi, const float* x, float* y,
                       long long rows, int k, int group, int bf16, cudaStream_t st) {
  switch (bits) {
    case 2: return launch_mlx_bits<2>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    case 3: return launch_mlx_bits<3>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    case 4: return launch_mlx_bits<4>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    case 5: return launch_mlx_bits<5>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    case 6: return launch_mlx_bits<6>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    case 8: return launch_mlx_bits<8>(gemv, w, sc, bi, x, y, rows, k, group, bf16, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vtb

using namespace vtb;

static int check_mlx(const void* w, const void* sc, const void* bi, int64_t rows, int64_t k, int bits, int group) {
  if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8))
    return set_err(VTB_CUDA_ERR_UNSUPPORTED, "MLX bits must be 2, 3, 4, 5, 6 or 8");
  if (!w || !sc || !bi) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null MLX tensor");
  if (rows <= 0 || k <= 0 || rows > INT_MAX || k > INT_MAX) return set_err(VTB_CUDA_ERR_INVALID_ARG, "m and k must be in [1, 2^31)");
  const int el = 32 / bits;
  if (group <= 0 || k % group || group % el)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "group size must divide k and be a multiple of 32 / bits");
  return VTB_CUDA_OK;
}

extern "C" {

int vtb_cuda_gemv_mlx(const void* w, const void* scales, const void* biases, const float* x, float* y, int64_t m,
                      int64_t k, int bits, int group_size, int scale_is_bf16, void* stream) {
  cudaGetLastError();
  int rc = check_mlx(w, scales, biases, m, k, bits, group_size);
  if (rc) return rc;
  if (!x || !y || (reinterpret_cast<uintptr_t>(x) & 15u)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "x must be 16-byte aligned, y non-null");
  return cuda_status(launch_mlx(true, bits, w, scales, biases, x, y, m, (int)k, group_size, scale_is_bf16 != 0,
                                (cudaStream_t)stream));
}

int vtb_cuda_dequant_mlx(const void* w, const void* scales, const void* biases, float* out, int64_t rows, int64_t k,
                         int bits, int group_size, int scale_is_bf16, void* stream) {
  cudaGetLastError();
  int rc = check_mlx(w, scales, biases, rows, k, bits, group_size);
  if (rc) return rc;
  if (!out) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null output");
  return cuda_status(launch_mlx(false, bits, w, scales, biases, nullptr, out, rows, (int)k, group_size,
                                scale_is_bf16 != 0, (cudaStream_t)stream));
}

int vtb_cuda_matmul_mlx_q4(VtbCudaCtx* c, VtbCudaBuf* out, VtbCudaBuf* w, size_t w_off, VtbCudaBuf* s, size_t s_off,
                           VtbCudaBuf* b, size_t b_off, VtbCudaBuf* acts, size_t acts_off, size_t m, size_t k,
                           uint32_t group_size, uint32_t scale_dtype_is_bf16) {
  if (!use_ctx(c) || !out || !w || !s || !b || !acts) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null buffer");
  if (group_size == 0 || k % group_size || k % 8) return set_err(VTB_CUDA_ERR_INVALID_ARG, "group size must divide k");
  const size_t ng = k / group_size;
  if (w_off + m * (k / 2) > w->size || s_off + m * ng * 2 > s->size || b_off + m * ng * 2 > b->size ||
      acts_off + k * 4 > acts->size || out->size < m * 4)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "buffer too small for m x k");
  return vtb_cuda_gemv_mlx((const char*)w->ptr + w_off, (const char*)s->ptr + s_off, (const char*)b->ptr + b_off,
                           (const float*)((const char*)acts->ptr + acts_off), (float*)out->ptr, (int64_t)m,
                           (int64_t)k, 4, (int)group_size, (int)scale_dtype_is_bf16, c->stream);
}

}  // extern "C"
