// gemv_mma.cu -- tensor-core decode GEMV for Q4_K: y[m] = W[m,k] . x[k]
// with f32 x and y (the reference's matmul_q4_k, src/kernels/simd.zig:245-273).
//
// Why tensor cores for a GEMV: a Q4_K weight costs 0.5625 B of HBM, so at
// ~6.5 TB/s every SM must retire ~41 weights per clock.  SIMT dequant
// (nibble -> f32, FMA) costs >2 instructions per weight and runs out of issue
// slots at ~40% of the HBM roofline.  Here the nibble bytes go to the integer
// tensor core unchanged: one AND extracts four weights.
//
// Arithmetic:
//  * A (u8): the low nibbles q (AND 0x0F0F0F0F) of sub-block 2j, or the high
//    nibbles kept in place, 16*q (AND 0xF0F0F0F0), of sub-block 2j+1.  One
//    m16n8k32 MMA covers 16 rows x one 32-weight sub-block.
//  * B (s8): per sub-block s, x is scaled by 2^-e_s so that max|x| lands in
//    [32, 64), then split into four int8 limbs x/2^e_s ~ sum_c L_c 254^-c,
//    L0 = rint(x'), L_c = rint(residual * 254) (|error| < 254^-3, about
//    2^-29 relative to the block max).
//  * Block-diagonal B: the 8 columns hold (L0, L1) -- and, in a second MMA
//    pass over the same A registers, (L2, L3) -- of 4 consecutive
//    sub-blocks; the MMA of sub-block s only has its own column pair
//    non-zero, so the int32 accumulators D[r, 2s'+c] = sum_k A[r,k] L_c[k]
//    are EXACT integer dots per (row, sub-block, limb).
//  * Epilogue per (row, sub-block): sum_k q x = 2^e sum_c D_c 254^-c (/16
//    for high nibbles), and y += (d*sc) * sum q x - (dmin*mn) * sum x -- the
//    reference's w = d1*q - m1 (simd.zig:221-243) distributed over the
//    sub-block.  fp32 accumulation; tolerance-checked (<= 1e-4).
//
// Data movement: persistent CTAs; each warp streams tiles of 32 rows x one
// super-block HBM -> shared as one 2-D TMA box (no multicast) into an S-stage
// mbarrier ring; the copies for the first S tiles are issued before
// griddepcontrol.wait, so with programmatic dependent launch they overlap the
// kernel that produces x.  A landed tile is read out at once (A fragments and
// decoded block scales into registers), which frees its stage for the next
// copy; the activation loads are issued before the first read-out so their
// L2 latency overlaps it.
#include <cstring>

#include "common.cuh"
#include "tma.cuh"

namespace vtb {

__device__ __forceinline__ void imma16832(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void imma_s8(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared layout of the activation vector, written once per CTA:
//   xq[s] : 128 bytes per sub-block s = [limb c][lane-quad t][8 bytes]; the 8
//           bytes are the B-fragment registers b0 (k = 4t..4t+3) and b1
//           (k = 16+4t..16+4t+3) of column limb c.
//   xs[s] : {2^e_s, sum_k x_k}
struct XShared {
  int8_t* xq;
  float2* xs;
};

// Converts group gi (4 sub-blocks, 128 elements; this lane holds elements
// 4*lane .. 4*lane+3 in `a`) into int8 limbs and {2^e, sum x} per sub-block.
__device__ __forceinline__ void convert_group(float4 a, int gi, int lane, XShared xsh) {
  const int sub = lane >> 3, part = lane & 7;
  float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
  float sum = (a.x + a.y) + (a.z + a.w);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  const int E = (int)((__float_as_uint(m) >> 23) & 0xffu);  // biased exponent of max|x|
  // max|x| * 2^-e in [32, 64), so L0 = rint(x') fits int8 with room; zero /
  // subnormal blocks keep e = 0 (their limbs round to 0)
  const int e = (E == 0) ? 0 : (E - 127 - 5);
  const float sx = __uint_as_float((uint32_t)(127 + e) << 23);
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  float xv[4] = {a.x * inv, a.y * inv, a.z * inv, a.w * inv};  // exact (power of two)
  uint32_t lw[4];
  limbs254(xv, lw);
  const int s = gi * 4 + sub;
  // element l = 4*part + c sits at t = part & 3, half = part >> 2, byte c
  int8_t* dst = xsh.xq + s * 128 + (part & 3) * 8 + (part >> 2) * 4;
#pragma unroll
  for (int li = 0; li < 4; ++li) *reinterpret_cast<uint32_t*>(dst + 32 * li) = lw[li];
  if (part == 0) xsh.xs[s] = make_float2(sx, sum);
}

// x (times the RMSNorm weight `nw` and `inv` when nw is given: the layer's
// rmsNorm, math.zig:11-32, fused into the GEMV that consumes it) for groups
// gi = base + u * nwarps.
__device__ __forceinline__ float4 load_group(const float* __restrict__ x, int gi, int lane, const float* __restrict__ nw,
                                             float inv) {
  float4 v = __ldg(reinterpret_cast<const float4*>(x + gi * 128) + lane);
  if (nw) {
    const float4 wv = __ldg(reinterpret_cast<const float4*>(nw + gi * 128) + lane);
    v = make_float4((v.x * wv.x) * inv, (v.y * wv.y) * inv, (v.z * wv.z) * inv, (v.w * wv.w) * inv);
  }
  return v;
}

// Each warp converts 4 sub-blocks per float4 load (8 lanes per sub-block) and
// keeps up to 8 loads in flight, so the prologue costs about one L2 round trip.
__device__ __forceinline__ void build_x_shared(const float* __restrict__ x, int K, XShared xsh, int warp, int lane,
                                               int nwarps, const float* __restrict__ nw, float inv) {
  const int n4 = K / 128;  // groups of 4 sub-blocks
  for (int base = warp; base < n4; base += nwarps * 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int gi = base + u * nwarps;
      if (gi < n4) v[u] = load_group(x, gi, lane, nw, inv);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int gi = base + u * nwarps;
      if (gi >= n4) break;
      convert_group(v[u], gi, lane, xsh);
    }
  }
}

// The tile arrives as one 2-D TMA box (32 or 16 rows x one super-block, rows
// dense at 144 B = 4 (mod 32) words, so the fragment loads are conflict-free).
// Per-row copies of a few hundred bytes capped the stream near 5 TB/s on their
// issue rate alone; one box per tile moves the same bytes with 32x fewer copy
// operations.
//
// Q5_K (176 B: d, dmin, 12 scale bytes, qh[32], qs[128]) runs the same kernel:
// its sub-block values q + 16 * (bit s of qh[l]) (simd.zig:290-319) are
// assembled per A word from the nibbles and the qh bits, and fit u8 as they are.
template <int Q, int ROWS_ = 32>
struct MmaQ4K {
  static constexpr int ROWS = ROWS_;  // 32 (two m16 MMA tiles per warp tile) or 16 (one)
  static constexpr int BB = Q == Q5_K ? 176 : 144;
  static constexpr int QS = Q == Q5_K ? 48 : 16;  // offset of qs[] in the block
  static constexpr int SLOT = BB;
  static constexpr int STAGE = ROWS * SLOT;
  static_assert(Q == Q4_K || Q == Q5_K, "Q4_K / Q5_K super-blocks");
};

// Bit s of each byte of v moved to bit 4 (the qh bit of Q5_K, worth 16).
// (sh is a constant once the loops over sub-blocks are unrolled.)
__device__ __forceinline__ uint32_t qh_bit4(uint32_t v, int sh) {
  return (sh <= 4 ? (v << (4 - sh)) : (v >> (sh - 4))) & 0x10101010u;
}

// A tile's weight-side operands, read out of shared memory before the
// activations are needed: the MMA A fragments (raw nibble words) and, per
// (sub-block group, row), the block scales d*sc (times 1/16 for the high-
// nibble sub-blocks, which the MMA sees as 16q) and dmin*mn.
template <int MT>
struct TilePrep {
  uint32_t a[2][2][MT][4];  // [group][pair in group][m-tile][a0..a3]
  uint32_t h[MT][4];        // Q5_K: qh words at the same rows / k positions
  float d1[2][2 * MT], m1[2][2 * MT];
};

template <int WARPS, int S, int Q, int ROWS>
__global__ void __launch_bounds__(WARPS * 32, 1)
gemv_q4k_mma_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ W, const float* __restrict__ x, float* __restrict__ y, int M, int K,
                    int ksplit, int accumulate, const float* __restrict__ norm_w, float eps, float* __restrict__ swi) {
  VTB_TL(1);
  using C = MmaQ4K<Q, ROWS>;
  constexpr int MT = ROWS / 16, NI = 2 * MT;  // m16 tiles; rows g + 8i this lane holds
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  uint8_t* ring = smem + warp * S * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * S * C::STAGE) + warp * S;
  float* red = reinterpret_cast<float*>(smem + WARPS * S * C::STAGE + WARPS * S * 8);  // [WARPS][32]
  XShared xsh;
  xsh.xq = reinterpret_cast<int8_t*>(red + WARPS * 32);
  xsh.xs = reinterpret_cast<float2*>(xsh.xq + 4 * K);

  // Work: ROWS-row units.  The CTA's warps form WARPS/ksplit slots; a slot's
  // ksplit warps share one unit and split its K range by super-blocks
  // (super-block c goes to part c % ksplit).  Small M uses a large ksplit so
  // every SM streams; large M uses ksplit = 1.  ksplit is a power of two.
  const int kshift = __ffs(ksplit) - 1;
  const int slots = WARPS >> kshift, slot = warp >> kshift, kpart = warp & (ksplit - 1);
  const int nch = K / 256;
  const int nunits = (M + C::ROWS - 1) / C::ROWS;
  const int ngroups = (nunits + slots - 1) >> (__ffs(slots) - 1);  // a group = `slots` consecutive units
  const int my_groups = blockIdx.x < ngroups ? (ngroups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int my_chunks = kpart < nch ? ((nch - 1 - kpart) >> kshift) + 1 : 0;
  const int ntiles = my_groups * my_chunks;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Tiles go out in order (group, chunk); rows past M arrive zero-filled and
  // count toward the box bytes.
  int iss_g = 0, iss_c = 0, iss_n = 0;
  auto issue_next = [&]() {
    if (iss_n >= ntiles) return;
    const int u = (blockIdx.x + iss_g * gridDim.x) * slots + slot;
    const int c = kpart + (iss_c << kshift), st = iss_n % S;
    if (lane == 0) {
      mbar_expect_tx(&bars[st], (unsigned)C::STAGE);
      tma_load_2d(ring + st * C::STAGE, &wmap, c * (C::BB / 4), u * C::ROWS, &bars[st]);
    }
    ++iss_n;
    if (++iss_c == my_chunks) { iss_c = 0; ++iss_g; }
  };
#pragma unroll
  for (int i = 0; i < S; ++i) issue_next();

  // Let the next kernel in the stream launch now (its own wait still orders it
  // after this grid completes): its CTAs start their weight prefetch on free SMs.
  // The x rows of at most 2 groups per warp stay in registers; the RMSNorm
  // weight (when fused) is a weight, independent of the producer of x, so it
  // is loaded before the wait.
  const int n4 = K / 128;
  const bool early_x = n4 <= 2 * WARPS;
  float4 xv0 = make_float4(0.f, 0.f, 0.f, 0.f), xv1 = xv0, nv0 = xv0, nv1 = xv0;
  if (norm_w && early_x) {
    if (warp < n4) nv0 = __ldg(reinterpret_cast<const float4*>(norm_w + warp * 128) + lane);
    if (warp + WARPS < n4) nv1 = __ldg(reinterpret_cast<const float4*>(norm_w + (warp + WARPS) * 128) + lane);
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();

  // Read tile tt's weight-side operands into registers, then hand its stage
  // back to the copy engine.
  TilePrep<MT> P;
  auto prep = [&](int tt) -> bool {
    const int st = tt % S;
    if (!mbar_wait_bounded(&bars[st], (unsigned)((tt / S) & 1))) return false;
    const uint8_t* base = ring + st * C::STAGE + g * C::SLOT;  // row g + 8i at base + 8i*SLOT
#pragma unroll
    for (int grp = 0; grp < 2; ++grp)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint8_t* r = base + 16 * mt * C::SLOT + C::QS + 32 * (2 * grp + jj) + 4 * t;
          P.a[grp][jj][mt][0] = *reinterpret_cast<const uint32_t*>(r);
          P.a[grp][jj][mt][1] = *reinterpret_cast<const uint32_t*>(r + 8 * C::SLOT);
          P.a[grp][jj][mt][2] = *reinterpret_cast<const uint32_t*>(r + 16);
          P.a[grp][jj][mt][3] = *reinterpret_cast<const uint32_t*>(r + 8 * C::SLOT + 16);
        }
    if constexpr (Q == Q5_K) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint8_t* r = base + 16 * mt * C::SLOT + 16 + 4 * t;  // qh[4t], qh[16 + 4t]
        P.h[mt][0] = *reinterpret_cast<const uint32_t*>(r);
        P.h[mt][1] = *reinterpret_cast<const uint32_t*>(r + 8 * C::SLOT);
        P.h[mt][2] = *reinterpret_cast<const uint32_t*>(r + 16);
        P.h[mt][3] = *reinterpret_cast<const uint32_t*>(r + 8 * C::SLOT + 16);
      }
    }
    // Q4_K: odd sub-blocks are high nibbles, carried in place as 16*q
    const float qscale = (Q == Q4_K && (t & 1)) ? 0.0625f : 1.0f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const uint4 hh = *reinterpret_cast<const uint4*>(base + 8 * i * C::SLOT);
      const float dd = h2f((uint16_t)(hh.x & 0xffffu)) * qscale, dm = h2f((uint16_t)(hh.x >> 16));
      const unsigned yb = (hh.y >> (8 * t)) & 0xffu, zb = (hh.z >> (8 * t)) & 0xffu, wb = (hh.w >> (8 * t)) & 0xffu;
      // q4kScaleMin (simd.zig:211-219): sub-block t (< 4) and 4 + t
      P.d1[0][i] = dd * (float)(yb & 63u);
      P.m1[0][i] = dm * (float)(zb & 63u);
      P.d1[1][i] = dd * (float)((wb & 15u) | ((yb >> 6) << 4));
      P.m1[1][i] = dm * (float)((wb >> 4) | ((zb >> 6) << 4));
    }
    // The refill is an async-proxy write into the bytes just read: order
    // every lane's reads before it.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    issue_next();  // this stage's bytes are in registers: refill it
    return true;
  };

  float inv = 1.f;
  if (early_x) {  // the activation loads fly while the first tile is read out
    if (warp < n4) xv0 = __ldg(reinterpret_cast<const float4*>(x + warp * 128) + lane);
    if (warp + WARPS < n4) xv1 = __ldg(reinterpret_cast<const float4*>(x + (warp + WARPS) * 128) + lane);
  }
  bool ok = ntiles == 0 || prep(0);
  if (norm_w) {  // sum of squares of the whole row (every CTA; x is L2-resident)
    float ss = 0.f;
    if (early_x) {  // the same float4s, in the same order, as the loop below
      ss = (xv0.x * xv0.x + xv0.y * xv0.y) + (xv0.z * xv0.z + xv0.w * xv0.w);
      ss += (xv1.x * xv1.x + xv1.y * xv1.y) + (xv1.z * xv1.z + xv1.w * xv1.w);
    } else {
      for (int i = threadIdx.x; i < K / 4; i += WARPS * 32) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x) + i);
        ss += (a.x * a.x + a.y * a.y) + (a.z * a.z + a.w * a.w);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tsum = 0.f;
    for (int w = 0; w < WARPS; ++w) tsum += red[w];
    inv = 1.0f / sqrtf(tsum / (float)K + eps);
    __syncthreads();
  }
  if (early_x) {
    if (norm_w) {  // (x * w) * inv, as load_group scales
      xv0 = make_float4((xv0.x * nv0.x) * inv, (xv0.y * nv0.y) * inv, (xv0.z * nv0.z) * inv, (xv0.w * nv0.w) * inv);
      xv1 = make_float4((xv1.x * nv1.x) * inv, (xv1.y * nv1.y) * inv, (xv1.z * nv1.z) * inv, (xv1.w * nv1.w) * inv);
    }
    if (warp < n4) convert_group(xv0, warp, lane, xsh);
    if (warp + WARPS < n4) convert_group(xv1, warp + WARPS, lane, xsh);
  } else {
    build_x_shared(x, K, xsh, warp, lane, WARPS, norm_w, inv);
  }
  __syncthreads();
  VTB_TL_MARK(0);

  const int gs = g >> 1;                  // sub-block (within a group of 4) whose B columns this lane holds
  const int boff = (g & 1) * 32 + t * 8;  // limb g&1, quad t

  for (int ui = 0; ui < my_groups; ++ui) {
    const int u = (blockIdx.x + ui * gridDim.x) * slots + slot;
    const int r0 = u * C::ROWS, nr = max(0, min(C::ROWS, M - r0));
    float acc[NI] = {};  // rows g + 8i; this lane's sub-blocks t and 4+t
    for (int ci = 0; ci < my_chunks && ok; ++ci) {
      const int tt = ui * my_chunks + ci;
      const int sb = kpart + (ci << kshift);
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int8_t* xb = xsh.xq + (sb * 8 + 4 * grp + gs) * 128 + boff;
        const uint2 bx = *reinterpret_cast<const uint2*>(xb);        // limb (g&1)
        const uint2 bz = *reinterpret_cast<const uint2*>(xb + 64);   // limb 2 + (g&1)
        int D[MT][4] = {};  // [m-tile][frag], limbs 0/1
        int E[MT][4] = {};  // limbs 2/3
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {  // nibble pair 2 grp + jj: sub-blocks 2p (low), 2p+1 (high)
          const bool mlo = gs == 2 * jj, mhi = gs == 2 * jj + 1;
          const uint32_t bl0 = mlo ? bx.x : 0u, bl1 = mlo ? bx.y : 0u;
          const uint32_t bh0 = mhi ? bx.x : 0u, bh1 = mhi ? bx.y : 0u;
          const uint32_t zl0 = mlo ? bz.x : 0u, zl1 = mlo ? bz.y : 0u;
          const uint32_t zh0 = mhi ? bz.x : 0u, zh1 = mhi ? bz.y : 0u;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint32_t* a = P.a[grp][jj][mt];
            uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
            if constexpr (Q == Q5_K) {  // q + 16 * bit (2p | 2p+1) of qh[l]
              const uint32_t* hq = P.h[mt];
              const int SL = 2 * (2 * grp + jj), SHI = SL + 1;
              l0 = (a[0] & 0x0F0F0F0Fu) | qh_bit4(hq[0], SL); l1 = (a[1] & 0x0F0F0F0Fu) | qh_bit4(hq[1], SL);
              l2 = (a[2] & 0x0F0F0F0Fu) | qh_bit4(hq[2], SL); l3 = (a[3] & 0x0F0F0F0Fu) | qh_bit4(hq[3], SL);
              h0 = ((a[0] >> 4) & 0x0F0F0F0Fu) | qh_bit4(hq[0], SHI); h1 = ((a[1] >> 4) & 0x0F0F0F0Fu) | qh_bit4(hq[1], SHI);
              h2 = ((a[2] >> 4) & 0x0F0F0F0Fu) | qh_bit4(hq[2], SHI); h3 = ((a[3] >> 4) & 0x0F0F0F0Fu) | qh_bit4(hq[3], SHI);
            } else {
              l0 = a[0] & 0x0F0F0F0Fu; l1 = a[1] & 0x0F0F0F0Fu; l2 = a[2] & 0x0F0F0F0Fu; l3 = a[3] & 0x0F0F0F0Fu;
              h0 = a[0] & 0xF0F0F0F0u; h1 = a[1] & 0xF0F0F0F0u; h2 = a[2] & 0xF0F0F0F0u; h3 = a[3] & 0xF0F0F0F0u;
            }
            imma16832(D[mt], l0, l1, l2, l3, bl0, bl1);
            imma16832(D[mt], h0, h1, h2, h3, bh0, bh1);
            imma16832(E[mt], l0, l1, l2, l3, zl0, zl1);
            imma16832(E[mt], h0, h1, h2, h3, zh0, zh1);
          }
        }
        // D[mt][0..1]: row 16mt+g, limbs (L0, L1) of sub-block s = 4 grp + t; D[mt][2..3]: row 16mt+g+8.
        const float2 xs = xsh.xs[sb * 8 + 4 * grp + t];
        const float f = xs.x * (1.0f / 254.0f);
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          const int mt = i >> 1, e = (i & 1) * 2;
          // limbs combined exactly in int32 (|D0*254 + D1| < 2^27), then converted once
          const float hi = (float)(D[mt][e] * 254 + D[mt][e + 1]);
          const float lo = (float)(E[mt][e] * 254 + E[mt][e + 1]);
          const float sq = fmaf(lo, 1.0f / 64516.0f, hi) * f;  // sum_k q_k x_k (16 q for high nibbles)
          acc[i] = fmaf(P.d1[grp][i], sq, acc[i]);
          acc[i] = fmaf(-P.m1[grp][i], xs.y, acc[i]);
        }
      }
      if (tt + 1 < ntiles && !prep(tt + 1)) ok = false;
    }
    VTB_TL_MARK(1);
    // CTA reduction of the K-split partial sums for this unit's rows.
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      float v = acc[i];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (t == 0) red[warp * 32 + 16 * (i >> 1) + 8 * (i & 1) + g] = v;
    }
    __syncthreads();
    if (kpart == 0) {  // warp-uniform
      float v = 0.f;
      const int nk = min(ksplit, nch);
      for (int w = 0; w < nk; ++w) v += red[(warp + w) * 32 + lane];
      if (swi) {
        // rows interleave as [gate 8 | up 8] blocks: lane i < 8 of each 16-row block holds
        // gate row i, lane i + 8 its up row; SwiGLU (math.zig:154-161) goes straight to h.
        const float u = __shfl_down_sync(0xffffffffu, v, 8);
        const int blk = lane >> 4, i = lane & 15;
        if (i < 8 && lane < ROWS && r0 + lane + 8 < M) {
          const float den = 1.0f + expf(-v);
          swi[r0 / 2 + 8 * blk + i] = (v / den) * u;
        }
      } else if (lane < nr && lane < ROWS) {
        y[r0 + lane] = accumulate ? y[r0 + lane] + v : v;
      }
    }
    __syncthreads();
  }
}

template <int WARPS, int S, int Q, int ROWS = 32>
constexpr int q4k_mma_smem(int k) {
  return WARPS * S * MmaQ4K<Q, ROWS>::STAGE + WARPS * S * 8 + WARPS * 128 + k * 4 + (k / 32) * 8;
}

template <int WARPS, int S, int Q, int ROWS>
static cudaError_t launch_q4k_mma_t(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                    int accumulate, const float* norm_w, float eps, float* swi) {
  using C = MmaQ4K<Q, ROWS>;
  constexpr auto kern = gemv_q4k_mma_kernel<WARPS, S, Q, ROWS>;
  const int smem = q4k_mma_smem<WARPS, S, Q, ROWS>(k);
  CUtensorMap wmap;
  // [m rows][k/256 * BB/4 u32]: one box = ROWS rows x one super-block
  const uint64_t rbytes = (uint64_t)(k / 256) * C::BB;
  if (!make_tmap(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, rbytes / 4, (uint64_t)m, rbytes, C::BB / 4, ROWS,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  const int dev = current_device();
  cudaError_t ea = ensure_smem_attr<kern>(dev, 227 * 1024);
  if (ea != cudaSuccess) return ea;
  // occupancy depends on k through the shared x buffer
  const int sms = sm_count(dev), per_sm = ctas_per_sm<kern>(dev, WARPS * 32, smem);
  const int units = (m + C::ROWS - 1) / C::ROWS;
  const int nch = k / 256;
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
  return cudaLaunchKernelEx(&cfg, kern, wmap, (const uint8_t*)w, x, y, m, k, ksplit, accumulate, norm_w, eps, swi);
}

// Critical-path cost (in 32-row tile units) of a row-tile height: rounds x
// chunks per warp from pick_ksplit; a 16-row tile costs ~0.6 of a 32-row one
// (its MMAs and epilogue halve, its activation-fragment work does not).
static double q4k_tile_cost(int m, int k, int rows, int warps, int cap) {
  const int units = (m + rows - 1) / rows, nch = k / 256;
  const int ks = pick_ksplit(units, nch, warps, cap);
  const long long slots = warps / ks, groups = (units + slots - 1) / slots;
  const long long grid = groups < cap ? groups : cap, rounds = (groups + grid - 1) / grid;
  return (double)(rounds * ((nch + ks - 1) / ks)) * (rows == 16 ? 0.6 : 1.0);
}

template <int Q>
static cudaError_t launch_kq_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                 int accumulate, const float* norm_w, float eps, float* swi) {
  // One 2-D TMA box per tile.  Matrices above 2^24 weights stream with two
  // stages per warp; smaller ones (dominated by the dependent-launch chain)
  // with one.  Very long rows (x staged in shared memory at 4.25 B per column)
  // fall back to 8 warps.  The row-tile height (32 or 16) is the one whose
  // launch balances better over the SMs.
  if (q4k_mma_smem<16, 2, Q>(k) > 227 * 1024)
    return launch_q4k_mma_t<8, 2, Q, 32>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi);
  const int sms = sm_count(current_device());
  const bool r16 = q4k_tile_cost(m, k, 16, 16, sms) < q4k_tile_cost(m, k, 32, 16, sms);
  if ((long long)m * k > (1LL << 24))
    return r16 ? launch_q4k_mma_t<16, 2, Q, 16>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi)
               : launch_q4k_mma_t<16, 2, Q, 32>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi);
  return r16 ? launch_q4k_mma_t<16, 1, Q, 16>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi)
             : launch_q4k_mma_t<16, 1, Q, 32>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi);
}

// swi non-null: W's rows are [gate 8 | up 8] blocks (m % 16 == 0) and the
// output is SwiGLU's h[m/2] in swi instead of y.
cudaError_t launch_gemv_q4k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate, const float* norm_w = nullptr, float eps = 0.f, float* swi = nullptr) {
  return launch_kq_mma<Q4_K>(w, x, y, m, k, st, pdl, accumulate, norm_w, eps, swi);
}

// Q5_K on the same kernel; rows must be 16-byte aligned (176 B super-blocks
// keep every row pitch a multiple of 16).
cudaError_t launch_gemv_q5k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate) {
  return launch_kq_mma<Q5_K>(w, x, y, m, k, st, pdl, accumulate, nullptr, 0.f, nullptr);
}

}  // namespace vtb
