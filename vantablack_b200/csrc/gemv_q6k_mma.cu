// gemv_q6k_mma.cu -- tensor-core decode GEMV for Q6_K: y[m] = W[m,k] . x[k]
// with f32 x and y (the reference's matmul_q6_k, src/kernels/simd.zig:366-404).
//
// Q6_K super-block (210 B / 256 weights): ql[128] low nibbles, qh[64] high
// 2-bit fields, sc[16] int8 scales of 16-weight sub-blocks, f16 d; weight
// = d * sc * (q - 32) with q = nibble | (2 bits << 4) in [0, 63].  In half n
// (128 weights), element 32i + l (i = 0..3, l = 0..31) takes its nibble from
// ql[64n + 32(i&1) + l] (low nibble for i < 2, high for i >= 2) and its high
// bits from qh[32n + l] >> 2i.
//
// Arithmetic (same scheme as the Q4_K kernel):
//  * A (u8): q assembled in registers, four weights per 32-bit word.
//  * B (s8): per 16-weight sub-block s, x scaled by 2^-e_s into [32, 64) and
//    split into four int8 limbs (x/2^e ~ sum_c L_c 254^-c).
//  * A quad = 64 consecutive weights = sub-blocks 0..3.  MMA 1 covers
//    sub-blocks 0 (k 0..15) and 1 (k 16..31), MMA 2 sub-blocks 2 and 3; B's
//    column g carries sub-block g/2, limb g&1 (and 2 + (g&1) in the second
//    pass) only on that sub-block's k range, so each int32 accumulator is an
//    exact per-(row, sub-block, limb) dot, and lane (g, t) ends up owning
//    whole sub-block t of rows g and g+8.
//  * Epilogue per (row, sub-block): y += (d*sc) * (sum q x - 32 sum x).
//
// Data movement: one 2-D TMA box per tile = 16 rows x two super-blocks (432 B
// from the 16-byte boundary at or below super-block 2c, so row pitch must be
// a multiple of 16 B: k % 2048 == 0).  Rows land 432 B apart (12 mod 32
// words: conflict-free fragment loads).  The odd super-block of a tile sits
// 2 bytes off a word boundary; its words are rebuilt with one byte-permute
// from two aligned loads.
#include "common.cuh"
#include "tma.cuh"

namespace vtb {

__device__ __forceinline__ void imma16832_q6(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int Q6M_ROWS = 16;                 // one m16 tile per warp tile
constexpr int Q6M_BOXB = 432;                // 2 x 210 B + up to 12 B lead, multiple of 16
constexpr int Q6M_STAGE = Q6M_ROWS * Q6M_BOXB;

// Shared x: xq[quad] = 256 B = [lane (g, t)][limb g&1 word | limb 2+(g&1) word]
// for sub-block 4*quad + g/2, elements 4t..4t+3; xs[sub-block] = {2^e / 254, 32 * sum x}.
__device__ __forceinline__ void build_x_q6k(const float* __restrict__ x, int K, int8_t* xq, float2* xs, int warp,
                                            int lane, int nwarps) {
  const int n4 = K / 4;  // float4 groups; 4 per sub-block, a warp covers 8 sub-blocks per pass
  for (int base = warp * 32; base < n4; base += nwarps * 32 * 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int f = base + u * nwarps * 32 + lane;
      v[u] = f < n4 ? __ldg(reinterpret_cast<const float4*>(x) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int f = base + u * nwarps * 32 + lane;
      if (base + u * nwarps * 32 >= n4) break;  // warp-uniform: n4 is a multiple of 32
      const float4 a = v[u];
      float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
      float sum = (a.x + a.y) + (a.z + a.w);
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
      }
      const int E = (int)((__float_as_uint(m) >> 23) & 0xffu);
      const int e = (E == 0) ? 0 : (E - 127 - 5);  // max|x| * 2^-e in [32, 64)
      const float sx = __uint_as_float((uint32_t)(127 + e) << 23);
      const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
      float xv[4] = {a.x * inv, a.y * inv, a.z * inv, a.w * inv};
      uint32_t lw[4];
      limbs254(xv, lw);
      const int sb = f >> 2, t = f & 3, sbl = sb & 3;
#pragma unroll
      for (int c = 0; c < 2; ++c)
        *reinterpret_cast<uint2*>(xq + (sb >> 2) * 256 + ((2 * sbl + c) * 4 + t) * 8) = make_uint2(lw[c], lw[2 + c]);
      if (t == 0) xs[sb] = make_float2(sx * (1.0f / 254.0f), 32.0f * sum);
    }
  }
}

// Word at byte offset `o` of a staged row: 4-byte aligned when !ODD, 2 mod 4 when ODD.
template <bool ODD>
__device__ __forceinline__ uint32_t ldw6(const uint8_t* p) {
  if constexpr (!ODD) {
    return *reinterpret_cast<const uint32_t*>(p);
  } else {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - 2);
    return __byte_perm(q[0], q[1], 0x5432);
  }
}

// q for four consecutive weights: nibbles (shifted down by ns) | 2-bit fields (qh >> 2i) << 4.
__device__ __forceinline__ uint32_t q6word(uint32_t ql, uint32_t qh, int ns, int i) {
  return ((ql >> ns) & 0x0F0F0F0Fu) | (((qh >> (2 * i)) << 4) & 0x30303030u);
}

template <int WARPS, int S>
__global__ void __launch_bounds__(WARPS * 32, 1)
gemv_q6k_mma_kernel(const __grid_constant__ CUtensorMap wmap, float* __restrict__ y, const float* __restrict__ x,
                    int M, int K, int ksplit, int accumulate) {
  VTB_TL(2);
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3, sbl = g >> 1;

  uint8_t* ring = smem + warp * S * Q6M_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * S * Q6M_STAGE) + warp * S;
  float* red = reinterpret_cast<float*>(smem + WARPS * S * Q6M_STAGE + WARPS * S * 8);  // [WARPS][16]
  int8_t* xq = reinterpret_cast<int8_t*>(red + WARPS * 16);
  float2* xs = reinterpret_cast<float2*>(xq + 4 * K);

  const int slots = WARPS / ksplit, slot = warp / ksplit, kpart = warp % ksplit;
  const int nb = K / 256, nch = nb / 2;  // chunk = tile = two super-blocks
  const int nunits = (M + Q6M_ROWS - 1) / Q6M_ROWS;
  const int ngroups = (nunits + slots - 1) / slots;
  const int my_groups = blockIdx.x < ngroups ? (ngroups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int my_chunks = kpart < nch ? (nch - 1 - kpart) / ksplit + 1 : 0;
  const int ntiles = my_groups * my_chunks;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto issue = [&](int tt) {  // rows past M arrive zero-filled and count toward the box bytes
    const int u = (blockIdx.x + (tt / my_chunks) * gridDim.x) * slots + slot;
    const int c = kpart + ksplit * (tt % my_chunks), st = tt % S;
    if (lane == 0) {
      mbar_expect_tx(&bars[st], (unsigned)Q6M_STAGE);
      tma_load_2d(ring + st * Q6M_STAGE, &wmap, ((420 * c) >> 4) << 2, u * Q6M_ROWS, &bars[st]);
    }
  };
  for (int tt = 0; tt < min(S, ntiles); ++tt) issue(tt);

  // Let the next kernel in the stream launch now (its own wait still orders it
  // after this grid completes): its CTAs start their weight prefetch on free SMs.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  build_x_q6k(x, K, xq, xs, warp, lane, WARPS);
  __syncthreads();

  bool ok = true;
  for (int ui = 0; ui < my_groups; ++ui) {
    const int u = (blockIdx.x + ui * gridDim.x) * slots + slot;
    const int r0 = u * Q6M_ROWS, nr = max(0, min(Q6M_ROWS, M - r0));
    float acc[2] = {0.f, 0.f};  // rows g, g+8
    for (int ci = 0; ci < my_chunks && ok; ++ci) {
      const int tt = ui * my_chunks + ci, st = tt % S;
      const int c = kpart + ksplit * ci;
      if (!mbar_wait_bounded(&bars[st], (unsigned)((tt / S) & 1))) { ok = false; break; }
      const uint8_t* tile = ring + st * Q6M_STAGE + ((420 * c) & 15);
      auto superblock = [&](auto odd_tag, int j) {
        constexpr bool ODD = decltype(odd_tag)::value;
        const uint8_t* b0 = tile + g * Q6M_BOXB + (ODD ? 210 : 0);  // row g; row g+8 at +8 rows
        const uint8_t* b1 = b0 + 8 * Q6M_BOXB;
        const float d0 = h2f(*reinterpret_cast<const uint16_t*>(b0 + 208));
        const float d1 = h2f(*reinterpret_cast<const uint16_t*>(b1 + 208));
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          uint32_t L0[4], L1[4], H0[2], H1[2];  // ql words (k 0..15, 16..31 of groups 0/1), qh words
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            L0[w] = ldw6<ODD>(b0 + 64 * n + 16 * w + 4 * t);
            L1[w] = ldw6<ODD>(b1 + 64 * n + 16 * w + 4 * t);
          }
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            H0[w] = ldw6<ODD>(b0 + 128 + 32 * n + 16 * w + 4 * t);
            H1[w] = ldw6<ODD>(b1 + 128 + 32 * n + 16 * w + 4 * t);
          }
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {  // quad qi = 2n + qq: groups i = 2qq (MMA 1), 2qq + 1 (MMA 2)
            const int qi = 2 * n + qq, ns = 4 * qq;
            const int gq = j * 4 + qi;  // quad index along K
            const uint2 bx = *reinterpret_cast<const uint2*>(xq + gq * 256 + lane * 8);
            const float2 xv = xs[gq * 4 + t];
            int D[4] = {0, 0, 0, 0}, E[4] = {0, 0, 0, 0};
#pragma unroll
            for (int mm = 0; mm < 2; ++mm) {
              const int i = 2 * qq + mm;  // group: ql words 2mm, 2mm+1 (k 0..15, 16..31)
              const uint32_t a0 = q6word(L0[2 * mm], H0[0], ns, i), a1 = q6word(L1[2 * mm], H1[0], ns, i);
              const uint32_t a2 = q6word(L0[2 * mm + 1], H0[1], ns, i), a3 = q6word(L1[2 * mm + 1], H1[1], ns, i);
              const bool lo = sbl == 2 * mm, hi = sbl == 2 * mm + 1;  // this lane's columns in MMA mm
              imma16832_q6(D, a0, a1, a2, a3, lo ? bx.x : 0u, hi ? bx.x : 0u);
              imma16832_q6(E, a0, a1, a2, a3, lo ? bx.y : 0u, hi ? bx.y : 0u);
            }
            const int sbi = 4 * qi + t;  // sub-block index within the super-block
            const float s0 = (float)(int)reinterpret_cast<const int8_t*>(b0)[192 + sbi];
            const float s1 = (float)(int)reinterpret_cast<const int8_t*>(b1)[192 + sbi];
            const float h0 = (float)(D[0] * 254 + D[1]), l0 = (float)(E[0] * 254 + E[1]);
            const float h1 = (float)(D[2] * 254 + D[3]), l1 = (float)(E[2] * 254 + E[3]);
            const float sq0 = (h0 + l0 * (1.0f / 64516.0f)) * xv.x;  // sum_k q_k x_k
            const float sq1 = (h1 + l1 * (1.0f / 64516.0f)) * xv.x;
            acc[0] += (d0 * s0) * (sq0 - xv.y);
            acc[1] += (d1 * s1) * (sq1 - xv.y);
          }
        }
      };
      superblock(std::integral_constant<bool, false>{}, 2 * c);
      superblock(std::integral_constant<bool, true>{}, 2 * c + 1);
      __syncwarp();
      if (tt + S < ntiles) issue(tt + S);
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      float v = acc[rr];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (t == 0) red[warp * 16 + 8 * rr + g] = v;
    }
    __syncthreads();
    if (kpart == 0 && lane < 16) {
      float v = 0.f;
      for (int w = 0; w < min(ksplit, nch); ++w) v += red[(warp + w) * 16 + lane];
      if (lane < nr) y[r0 + lane] = accumulate ? y[r0 + lane] + v : v;
    }
    __syncthreads();
  }
}

template <int WARPS, int S>
constexpr int q6k_mma_smem(int k) {
  return WARPS * S * Q6M_STAGE + WARPS * S * 8 + WARPS * 64 + k * 4 + (k / 16) * 8;
}

template <int WARPS, int S>
static cudaError_t launch_q6k_mma_t(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                    int accumulate, long long pitch) {
  auto kern = gemv_q6k_mma_kernel<WARPS, S>;
  const int smem = q6k_mma_smem<WARPS, S>(k);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  CUtensorMap wmap;
  const uint64_t rbytes = (uint64_t)pitch;  // row pitch, a 16-byte multiple (rows may carry zero padding)
  if (!make_tmap(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, rbytes / 4, (uint64_t)m, rbytes, Q6M_BOXB / 4, Q6M_ROWS,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const int dev = current_device();
  cudaError_t ea = ensure_smem_attr<gemv_q6k_mma_kernel<WARPS, S>>(dev, 227 * 1024);
  if (ea != cudaSuccess) return ea;
  const int sms = sm_count(dev), per_sm = ctas_per_sm<gemv_q6k_mma_kernel<WARPS, S>>(dev, WARPS * 32, smem);
  const int units = (m + Q6M_ROWS - 1) / Q6M_ROWS;
  const int nch = k / 512;
  const int cap = sms * per_sm;
  int ksplit = pick_ksplit(units, nch, WARPS, cap);
  const int groups = (units + WARPS / ksplit - 1) / (WARPS / ksplit);
  const int grid = groups < cap ? groups : cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, wmap, y, x, m, k, ksplit, accumulate);
}

// Usable when the row pitch is a 16-byte multiple (dense rows when k % 2048 == 0,
// or rows the model uploaded with zero padding), rows hold whole super-block
// pairs (k % 512 == 0) and w is 16-byte aligned.
bool q6k_mma_ok(const void* w, int k, long long pitch) {
  return k % 512 == 0 && pitch % 16 == 0 && pitch >= (long long)(k / 256) * 210 &&
         (reinterpret_cast<uintptr_t>(w) & 15) == 0 && q6k_mma_smem<8, 2>(k) <= 227 * 1024;
}

cudaError_t launch_gemv_q6k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate, long long pitch) {
  if (q6k_mma_smem<12, 2>(k) <= 227 * 1024) return launch_q6k_mma_t<12, 2>(w, x, y, m, k, st, pdl, accumulate, pitch);
  return launch_q6k_mma_t<8, 2>(w, x, y, m, k, st, pdl, accumulate, pitch);
}

}  // namespace vtb
