// gemm_tc.cu -- prefill GEMM on the 5th-generation tensor cores:
// out[b, m] = sum_k W[m, k] * acts[b, k] for GGUF-quantized W (Q4_K, Q5_K,
// Q6_K, Q8_0) and f32 activations -- the reference's matmulBatched
// (src/runtime/prefill.zig:325-378: dequantize a row once, then B dot_f32).
//
// Per CTA: a 128-row weight tile x BN-token tile, the full K range.
//  * Warps 0-3 (producers): thread t dequantizes row t of the tile, 64 weights
//    per k-block, with the reference's exact f32 formula (bit-identical to
//    dequantToF32), converts to bf16 and stores into a 128-byte-swizzled
//    K-major shared tile (the UMMA SWIZZLE_128B canonical layout: 8-row atoms
//    of 1024 B, 16-byte chunk c of row r at chunk c ^ (r % 8)).  The same
//    threads copy the bf16 activation tile with cp.async into the same layout.
//  * Warp 4, one elected thread: tcgen05.mma.cta_group::1.kind::f16 (bf16 x
//    bf16 -> f32), D in TMEM (BN columns), 4 MMAs of K=16 per k-block;
//    tcgen05.commit releases each stage back to the producers.
//  * Epilogue (warps 0-3): tcgen05.ld 32x32b, coalesced stores of out.
// Precision modes:
//  * PASSES = 1: bf16 operands (the north star's 2e-2 bf16 tolerance).
//  * PASSES = 3: both operands split into bf16 hi + lo parts and
//    hi*hi + hi*lo + lo*hi accumulated (~16-bit products): used by the model
//    prefill so its KV cache and logits stay within fp32-class tolerance of
//    the reference (greedy token identity).
// Every wait is bounded; a timeout sets the device error word, and all warps
// still reach the TMEM dealloc.

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "tma.cuh"

namespace vtb {

constexpr int TC_BM = 128, TC_BK = 64, TC_PROD = 128;

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: 8-row atom pitch
  d |= (uint64_t)1 << 46;                     // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                     // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, unsigned src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint32_t sw128_off(int r, int chunk) {  // byte offset of 16-B chunk `chunk` of row r
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4));
}

// ---- bit-exact dequantization of 64 consecutive weights [k0, k0+64) of one row ----
__device__ __forceinline__ uint32_t ldg_u32(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }
// Explicit shared-memory loads: the staging pointers pass through integer
// alignment arithmetic, after which the compiler would emit generic loads.
__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint4 lds_u128(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
  return v;
}
// 4-byte words from a 2-byte-aligned global address
template <int NW, bool SMEM = false>
__device__ __forceinline__ void ldg_words_a2(const uint8_t* p, uint32_t* out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  const unsigned sh = (unsigned)(a & 3) * 8u;
  uint32_t w[NW + 1];
#pragma unroll
  for (int i = 0; i <= NW; ++i) w[i] = SMEM ? lds_u32(b + 4 * i) : ldg_u32(b + 4 * i);
#pragma unroll
  for (int i = 0; i < NW; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}
__device__ __forceinline__ unsigned byte_of(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xffu; }

// SMEM: `blk` points into shared memory (TMA-staged super-block), read with
// ld.shared; otherwise it is global memory, read through the read-only path.
template <bool SMEM>
__device__ __forceinline__ uint4 ld16(const uint8_t* p) {
  if constexpr (SMEM) return lds_u128(p);
  else return __ldg(reinterpret_cast<const uint4*>(p));
}

// Weights [k0, k0 + 64) of one row as 32 packed pairs v[i] = (w[2i], w[2i+1]),
// bit-identical to dequantToF32 (forward.zig:654-736).  Every format's product
// is exact in f32 (an f16 scale times a small integer), so the packed
// multiplies and the fused multiply-subtract of Q4_K/Q5_K (d1 * q - m1, the
// product exact, one rounding) equal the reference's separately rounded ops.
// Quantized values become exact floats with the 2^23 byte-magic.
template <int Q, bool SMEM = false>
__device__ __forceinline__ void dequant64(const uint8_t* row, int k0, f2* v) {
  if constexpr (Q == Q4_K || Q == Q5_K) {
    constexpr int BB = Q == Q4_K ? 144 : 176;
    const uint8_t* blk = SMEM ? row : row + (k0 >> 8) * BB;  // SMEM: `row` is the staged super-block itself
    const int j = (k0 & 255) >> 6;  // sub-block pair: sub-blocks 2j, 2j+1
    const uint4 h = ld16<SMEM>(blk);
    const float d = h2f((uint16_t)(h.x & 0xffffu)), dmin = h2f((uint16_t)(h.x >> 16));
    const uint32_t sw[3] = {h.y, h.z, h.w};
    unsigned sc[2], mn[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // q4kScaleMin (simd.zig:211-219)
      const int s = 2 * j + u;
      if (s < 4) {
        sc[u] = byte_of(sw, s) & 63u; mn[u] = byte_of(sw, s + 4) & 63u;
      } else {
        sc[u] = (byte_of(sw, s + 4) & 15u) | ((byte_of(sw, s - 4) >> 6) << 4);
        mn[u] = (byte_of(sw, s + 4) >> 4) | ((byte_of(sw, s) >> 6) << 4);
      }
    }
    const float d1 = __fmul_rn(d, (float)sc[0]), m1 = __fmul_rn(dmin, (float)mn[0]);
    const float d2 = __fmul_rn(d, (float)sc[1]), m2 = __fmul_rn(dmin, (float)mn[1]);
    const f2 D1 = pk(d1, d1), N1 = pk(-m1, -m1), D2 = pk(d2, d2), N2 = pk(-m2, -m2);
    const f2 MG = pk(-8388608.f, -8388608.f);
    const uint8_t* qs = blk + (Q == Q4_K ? 16 : 48) + 32 * j;
    uint32_t q[8];
    const uint4 qa = ld16<SMEM>(qs), qb = ld16<SMEM>(qs + 16);
    q[0] = qa.x; q[1] = qa.y; q[2] = qa.z; q[3] = qa.w; q[4] = qb.x; q[5] = qb.y; q[6] = qb.z; q[7] = qb.w;
    uint32_t qh[8];
    if constexpr (Q == Q5_K) {
      const uint4 ha = ld16<SMEM>(blk + 16), hb = ld16<SMEM>(blk + 32);
      qh[0] = ha.x; qh[1] = ha.y; qh[2] = ha.z; qh[3] = ha.w; qh[4] = hb.x; qh[5] = hb.y; qh[6] = hb.z; qh[7] = hb.w;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) {  // weights l = 4w..4w+3 (low nibbles) and 32 + l (high nibbles)
      uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = (q[w] >> 4) & 0x0F0F0F0Fu;
      if constexpr (Q == Q5_K) {
        lo |= ((qh[w] >> (2 * j)) & 0x01010101u) << 4;
        hi |= ((qh[w] >> (2 * j + 1)) & 0x01010101u) << 4;
      }
      v[2 * w] = fma2(D1, add2(pk(byte_magic<0>(lo), byte_magic<1>(lo)), MG), N1);
      v[2 * w + 1] = fma2(D1, add2(pk(byte_magic<2>(lo), byte_magic<3>(lo)), MG), N1);
      v[16 + 2 * w] = fma2(D2, add2(pk(byte_magic<0>(hi), byte_magic<1>(hi)), MG), N2);
      v[16 + 2 * w + 1] = fma2(D2, add2(pk(byte_magic<2>(hi), byte_magic<3>(hi)), MG), N2);
    }
  } else if constexpr (Q == Q6_K) {
    const uint8_t* blk = SMEM ? row : row + (k0 >> 8) * 210;
    const int half = (k0 & 255) >> 7, nb = ((k0 & 127) >> 6) * 2;  // n in {nb, nb+1}
    uint32_t ql[16], qh[8], sc[2];
    ldg_words_a2<16, SMEM>(blk + half * 64, ql);
    ldg_words_a2<8, SMEM>(blk + 128 + half * 32, qh);
    ldg_words_a2<2, SMEM>(blk + 192 + half * 8, sc);
    uint32_t dw[1];
    ldg_words_a2<1, SMEM>(blk + 208, dw);
    const float d = h2f((uint16_t)(dw[0] & 0xffffu));
    const f2 MG = pk(-8388640.f, -8388640.f);  // 2^23 + 32: field q -> q - 32
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int n = nb + u;
#pragma unroll
      for (int w = 0; w < 8; ++w) {  // weights l = 4w..4w+3 of group n
        const uint32_t b = ql[(n & 1) * 8 + w];
        const uint32_t qv = (((n & 2) ? (b >> 4) : b) & 0x0F0F0F0Fu) | (((qh[w] >> (2 * n)) << 4) & 0x30303030u);
        const float ds = __fmul_rn(d, (float)(int8_t)byte_of(sc, (w >> 2) + 2 * n));
        const f2 DS = pk(ds, ds);
        v[16 * u + 2 * w] = mul2(DS, add2(pk(byte_magic<0>(qv), byte_magic<1>(qv)), MG));
        v[16 * u + 2 * w + 1] = mul2(DS, add2(pk(byte_magic<2>(qv), byte_magic<3>(qv)), MG));
      }
    }
  } else if constexpr (Q == TQ2_0) {  // group g = (k0 & 255) >> 6 of a 66-byte block (simd.zig:457-472)
    const uint8_t* blk = row + (k0 >> 8) * 66;
    const int g = (k0 & 255) >> 6;
    uint32_t qw[4], dw[1];
    ldg_words_a2<4, SMEM>(blk + 16 * g, qw);
    ldg_words_a2<1, SMEM>(blk + 64, dw);
    const float d = h2f((uint16_t)(dw[0] & 0xffffu));
    const f2 D = pk(d, d), MG = pk(-8388609.f, -8388609.f);  // 2^23 + 1: field r -> r - 1
#pragma unroll
    for (int t = 0; t < 4; ++t) {  // weights l = 4t..4t+3, repeated at l + 16, l + 32, l + 48
      const uint32_t r = (qw[t] >> (2 * g)) & 0x03030303u;
      const f2 a = mul2(D, add2(pk(byte_magic<0>(r), byte_magic<1>(r)), MG));
      const f2 b = mul2(D, add2(pk(byte_magic<2>(r), byte_magic<3>(r)), MG));
#pragma unroll
      for (int rep = 0; rep < 4; ++rep) {
        v[8 * rep + 2 * t] = a;
        v[8 * rep + 2 * t + 1] = b;
      }
    }
  } else {  // Q8_0: two 34-byte blocks
    const f2 MG = pk(-8388736.f, -8388736.f);  // 2^23 + 128: (i8 ^ 0x80) -> i8
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint8_t* blk = row + ((k0 >> 5) + u) * 34;
      uint32_t w[9];
      ldg_words_a2<9>(blk, w);
      const float d = h2f((uint16_t)(w[0] & 0xffffu));
      const f2 D = pk(d, d);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t qv = __funnelshift_r(w[t], w[t + 1], 16) ^ 0x80808080u;
        v[16 * u + 2 * t] = mul2(D, add2(pk(byte_magic<0>(qv), byte_magic<1>(qv)), MG));
        v[16 * u + 2 * t + 1] = mul2(D, add2(pk(byte_magic<2>(qv), byte_magic<3>(qv)), MG));
      }
    }
  }
}

// Packed bf16 pair of (v.x, v.y): v.x in the low half (round to nearest even).
__device__ __forceinline__ uint32_t cvt_bf16x2(f2 v) {
  float a, b;
  unpk(v, a, b);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// The f32 values of a packed bf16 pair.
__device__ __forceinline__ f2 bf16x2_to_f2(uint32_t h) { return pk(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u)); }


// Activations f32 [B][K] -> bf16 hi [B][K] (and lo = bf16(x - hi)).
__global__ void acts_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi,
                                    __nv_bfloat16* __restrict__ lo, long long n) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// TMA_A: raw weight super-blocks arrive by 2-D TMA (Q4_K / Q5_K: 16-byte
// multiples); otherwise producers read them from global memory directly.
// Q6_K super-blocks (210 B) start on 2-byte boundaries: the box covers 240 B
// from the 16-byte boundary at or below the super-block (TMA's x alignment rule).
template <int Q>
struct TmaA {
  static constexpr int BOX = Q == Q6_K ? 240 : Fmt<Q>::bytes;  // one super-block of one row (+ lead)
  __host__ __device__ static constexpr int x0(int j) { return Q == Q6_K ? (j * 210) & ~15 : j * Fmt<Q>::bytes; }
};

template <int Q, int BN, int PASSES, int S, bool TA>
struct TcCfg {
  static constexpr int A_BYTES = TC_BM * TC_BK * 2;  // 16 KiB
  static constexpr int B_BYTES = BN * TC_BK * 2;
  static constexpr int NOPS = PASSES == 1 ? 1 : 2;    // hi only, or hi + lo
  static constexpr int STAGE = NOPS * (A_BYTES + B_BYTES);
  static constexpr int SR = 3;                          // raw weight super-block stages
  static constexpr int RAW = TA ? TC_BM * TmaA<Q>::BOX : 0;
  static constexpr int SMEM = S * STAGE + SR * RAW + 1024 /*align*/ + 512 /*barriers + tmem slot*/;
};

// Warps 0-3 dequantize (thread = tile row), warp 4 lane 0 issues MMAs,
// warp 5 lane 0 issues the TMA loads.
template <int Q, int BN, int PASSES, int S, bool TA>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapBh,
               const __grid_constant__ CUtensorMap mapBl, const uint8_t* __restrict__ W, float* __restrict__ out,
               int M, int K, int NB, long long pitch) {
  VTB_TL(5);
  using C = TcCfg<Q, BN, PASSES, S, TA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + S * C::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(raw + C::SR * C::RAW);
  uint64_t* empty = full + S;
  uint64_t* rfull = empty + S;
  uint64_t* rempty = rfull + C::SR;
  uint64_t* done = rempty + C::SR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int m0 = blockIdx.x * TC_BM, n0 = blockIdx.y * BN;
  // Split-K (gridDim.z > 1, K % 256 == 0): this CTA takes super-blocks [sb0, sb1) and
  // writes its partial tile to out + z * NB * M; a reduce kernel sums the splits.
  const int nsb = K / 256, z = blockIdx.z, ks = gridDim.z;
  const int sb0 = ks > 1 ? z * nsb / ks : 0, sb1 = ks > 1 ? (z + 1) * nsb / ks : nsb;
  const int kb0 = ks > 1 ? 4 * sb0 : 0, kb1 = ks > 1 ? 4 * sb1 : K / TC_BK;
  out += (long long)z * NB * M;
  const long long rb = pitch;  // bytes between weight rows (the dense row size, or a padded pitch)

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], TC_PROD + 1);  // every dequant thread + the TMA thread (B bytes)
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < C::SR; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], TC_PROD);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 4) {  // TMEM: BN fp32 columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 5) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      constexpr unsigned BBYTES = (unsigned)C::B_BYTES * (PASSES == 3 ? 2u : 1u);
      int jr = sb0;  // next raw weight super-block
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        const int i = kb - kb0;  // ring position
        if constexpr (TA) {  // weights run up to SR - 1 super-blocks ahead (independent of the activations)
          while (jr < sb1 && jr - sb0 <= i / 4 + C::SR - 1 && ok) {
            const int jl = jr - sb0, rs = jl % C::SR;
            if (jl >= C::SR && !mbar_wait_bounded(&rempty[rs], (unsigned)(((jl / C::SR) - 1) & 1))) { ok = false; break; }
            mbar_expect_tx(&rfull[rs], (unsigned)C::RAW);
            tma_load_2d(raw + rs * C::RAW, &mapA, TmaA<Q>::x0(jr), m0, &rfull[rs]);
            ++jr;
          }
        }
        if (i == 0) asm volatile("griddepcontrol.wait;" ::: "memory");  // activations come from the previous kernel
  VTB_TL_WAITED();
        const int s = i % S;
        if (i >= S && !mbar_wait_bounded(&empty[s], (unsigned)(((i / S) - 1) & 1))) { ok = false; break; }
        uint8_t* st = smem + s * C::STAGE;
        mbar_expect_tx(&full[s], BBYTES);
        tma_load_2d(st + C::A_BYTES, &mapBh, kb * TC_BK, n0, &full[s]);
        if constexpr (PASSES == 3) tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, &mapBl, kb * TC_BK, n0, &full[s]);
      }
    }
  } else if (warp < 4) {
    // ---------------- dequantizers (thread = tile row) ----------------
    const int r = tid;
    const bool row_ok = m0 + r < M;
    const uint8_t* wrow = W + (long long)(row_ok ? m0 + r : 0) * rb;
    for (int kb = kb0; kb < kb1 && ok; ++kb) {
      const int i = kb - kb0, s = i % S, j = kb >> 2, jl = j - sb0;
      if constexpr (TA) {
        if ((kb & 3) == 0 && !mbar_wait_bounded(&rfull[jl % C::SR], (unsigned)((jl / C::SR) & 1))) { ok = false; break; }
      }
      if (i >= S && !mbar_wait_bounded(&empty[s], (unsigned)(((i / S) - 1) & 1))) { ok = false; break; }
      uint8_t* st = smem + s * C::STAGE;
      f2 v[32];
      if constexpr (TA) {  // this row's super-block sits at raw[j % SR] + r * BOX (out-of-range rows read as zeros)
        dequant64<Q, true>(raw + (jl % C::SR) * C::RAW + r * TmaA<Q>::BOX + (j * Fmt<Q>::bytes - TmaA<Q>::x0(j)),
                           kb * TC_BK, v);
        if ((kb & 3) == 3 || kb == kb1 - 1) mbar_arrive(&rempty[jl % C::SR]);
      } else if (row_ok) {
        dequant64<Q>(wrow, kb * TC_BK, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = pk(0.f, 0.f);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 hv;
        hv.x = cvt_bf16x2(v[4 * c]); hv.y = cvt_bf16x2(v[4 * c + 1]);
        hv.z = cvt_bf16x2(v[4 * c + 2]); hv.w = cvt_bf16x2(v[4 * c + 3]);
        *reinterpret_cast<uint4*>(st + sw128_off(r, c)) = hv;
        if constexpr (PASSES == 3) {  // lo = bf16(v - hi); v - hi is exact in f32
          uint4 lv;
          lv.x = cvt_bf16x2(sub2(v[4 * c], bf16x2_to_f2(hv.x)));
          lv.y = cvt_bf16x2(sub2(v[4 * c + 1], bf16x2_to_f2(hv.y)));
          lv.z = cvt_bf16x2(sub2(v[4 * c + 2], bf16x2_to_f2(hv.z)));
          lv.w = cvt_bf16x2(sub2(v[4 * c + 3], bf16x2_to_f2(hv.w)));
          *reinterpret_cast<uint4*>(st + C::A_BYTES + C::B_BYTES + sw128_off(r, c)) = lv;
        }
      }
      fence_async_smem();  // generic-proxy smem writes -> visible to the tensor core
      mbar_arrive(&full[s]);
    }
  } else if (lane == 0) {
    // ---------------- MMA issuer (warp 4) ----------------
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
    for (int kb = kb0; kb < kb1 && ok; ++kb) {
      const int i = kb - kb0, s = i % S;
      if (!mbar_wait_bounded(&full[s], (unsigned)((i / S) & 1))) { ok = false; break; }
      tc_fence_after();
      const uint32_t a_hi = smem_u32(smem + s * C::STAGE), b_hi = a_hi + C::A_BYTES;
      const uint32_t a_lo = b_hi + C::B_BYTES, b_lo = a_lo + C::A_BYTES;
#pragma unroll
      for (int kk = 0; kk < TC_BK / 16; ++kk) {  // K = 16 per MMA: +32 B within the swizzled row
        const int acc = (i | kk) != 0;
        mma_bf16(tmem, sw128_desc(a_hi + 32 * kk), sw128_desc(b_hi + 32 * kk), idesc, acc);
        if constexpr (PASSES == 3) {
          mma_bf16(tmem, sw128_desc(a_hi + 32 * kk), sw128_desc(b_lo + 32 * kk), idesc, 1);
          mma_bf16(tmem, sw128_desc(a_lo + 32 * kk), sw128_desc(b_hi + 32 * kk), idesc, 1);
        }
      }
      mma_commit(&empty[s]);
    }
    mma_commit(done);
  }
  __syncwarp();

  // ---------------- epilogue (warps 0-3: TMEM lanes 32w..32w+31 = tile rows) ----------------
  if (warp < 4) {
    if (ok && mbar_wait_bounded(done, 0u)) {
      tc_fence_after();
      const int row = m0 + 32 * warp + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
              "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
              "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < M) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (n0 + c0 + jj < NB) out[(long long)(n0 + c0 + jj) * M + row] = __uint_as_float(v[jj]);
        }
      }
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(BN));
  }
}

template <int Q, int BN, int PASSES, int S, bool TA>
static cudaError_t launch_gemm_tc_t(const void* w, const __nv_bfloat16* xh, const __nv_bfloat16* xl, float* out, int m,
                                    int k, int nb, int ks, cudaStream_t st, long long pitch) {
  using C = TcCfg<Q, BN, PASSES, S, TA>;
  auto kern = gemm_tc_kernel<Q, BN, PASSES, S, TA>;
  cudaError_t ea = ensure_smem_attr<gemm_tc_kernel<Q, BN, PASSES, S, TA>>(current_device(), C::SMEM);
  if (ea != cudaSuccess) return ea;
  CUtensorMap mA, mBh, mBl;
  memset(&mA, 0, sizeof mA);
  const uint64_t rbytes = (uint64_t)pitch;
  if (TA &&
      !make_tmap(&mA, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, rbytes, (uint64_t)m, rbytes, TmaA<Q>::BOX, TC_BM,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (!make_tmap(&mBh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xh, (uint64_t)k, (uint64_t)nb, (uint64_t)k * 2, TC_BK, BN,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (PASSES == 3) {
    if (!make_tmap(&mBl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xl, (uint64_t)k, (uint64_t)nb, (uint64_t)k * 2, TC_BK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else {
    mBl = mBh;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((m + TC_BM - 1) / TC_BM, (nb + BN - 1) / BN, ks);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute a[1];
  a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = a;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mA, mBh, mBl, (const uint8_t*)w, out, m, k, nb, pitch);
}

// Largest stage count (<= SMAX) whose shared memory fits the 227 KiB per-CTA limit.
template <int Q, int BN, int PASSES, bool TA, int SMAX>
constexpr int fit_stages() {
  if constexpr (SMAX <= 1) return 1;
  else if constexpr (TcCfg<Q, BN, PASSES, SMAX, TA>::SMEM <= 227 * 1024) return SMAX;
  else return fit_stages<Q, BN, PASSES, TA, SMAX - 1>();
}

template <int Q, int BN, int PASSES, bool TA>
static cudaError_t launch_fit(const void* w, const __nv_bfloat16* xh, const __nv_bfloat16* xl, float* out, int m, int k,
                              int nb, int ks, cudaStream_t st, long long pitch) {
  constexpr int S = fit_stages<Q, BN, PASSES, TA, 5>();
  static_assert(TcCfg<Q, BN, PASSES, S, TA>::SMEM <= 227 * 1024, "GEMM tile does not fit in shared memory");
  return launch_gemm_tc_t<Q, BN, PASSES, S, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
}

template <int Q, bool TA>
static cudaError_t launch_gemm_tc_qt(const void* w, const __nv_bfloat16* xh, const __nv_bfloat16* xl, float* out, int m,
                                     int k, int nb, bool precise, int ks, cudaStream_t st, long long pitch) {
  if (precise) {  // hi + lo tiles: twice the shared memory per stage
    if (nb <= 64) return launch_fit<Q, 64, 3, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
    if (nb <= 128) return launch_fit<Q, 128, 3, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
    if constexpr (TcCfg<Q, 256, 3, 2, TA>::SMEM <= 227 * 1024)
      return launch_fit<Q, 256, 3, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
    else
      return launch_fit<Q, 128, 3, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
  }
  if (nb <= 64) return launch_fit<Q, 64, 1, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
  if (nb <= 128) return launch_fit<Q, 128, 1, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
  return launch_fit<Q, 256, 1, TA>(w, xh, xl, out, m, k, nb, ks, st, pitch);
}

template <int Q>
static cudaError_t launch_gemm_tc_q(const void* w, const __nv_bfloat16* xh, const __nv_bfloat16* xl, float* out, int m,
                                    int k, int nb, bool precise, int ks, cudaStream_t st, long long pitch) {
  // TMA weight staging needs 16-byte row pitches (all K-quant configs with k % 2048 == 0 qualify)
  if constexpr (Q == Q8_0 || Q == TQ2_0) {  // blocks off 16-byte boundaries: producers read global memory
    return launch_gemm_tc_qt<Q, false>(w, xh, xl, out, m, k, nb, precise, ks, st, pitch);
  } else {
    if (pitch % 16 == 0) return launch_gemm_tc_qt<Q, true>(w, xh, xl, out, m, k, nb, precise, ks, st, pitch);
    return launch_gemm_tc_qt<Q, false>(w, xh, xl, out, m, k, nb, precise, ks, st, pitch);
  }
}

// out[i] = sum over splits z of part[z][i], in split order (deterministic).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ out, long long n, int ks) {
  VTB_TL(6);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float v = part[i];
    for (int z = 1; z < ks; ++z) v += part[(long long)z * n + i];
    out[i] = v;
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// out[nb][m] = acts[nb][k] . W^T.  `ws` is bf16 scratch of nb*k*(precise ? 2 : 1) elements.
// `part` (optional, `part_elems` floats): when the (M/128) x (B/BN) tile grid
// leaves most SMs idle (small batches), K is split across up to 8 CTAs per
// tile, each writing a partial tile there; splitk_reduce_kernel sums them.
// `pitch`: bytes between consecutive weight rows (0 = the dense row size).
cudaError_t launch_gemm_tc(int q, const void* w, const float* acts, float* out, int m, int k, int nb, bool precise,
                           void* ws, cudaStream_t st, float* part = nullptr, size_t part_elems = 0, long long pitch = 0) {
  if (pitch == 0) pitch = host_row_bytes(q, k);
  __nv_bfloat16* xh = static_cast<__nv_bfloat16*>(ws);
  __nv_bfloat16* xl = precise ? xh + (size_t)nb * k : nullptr;
  const long long n = (long long)nb * k;
  cudaLaunchConfig_t cfg = {};
  const long long blocks = (n + 255) / 256;
  cfg.gridDim = dim3((unsigned)(blocks < 148LL * 16 ? blocks : 148LL * 16));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute a[1];
  a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = a;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, acts_to_bf16_kernel, acts, xh, xl, n);
  if (e != cudaSuccess) return e;
  int ks = 1;
  if (part && k % 256 == 0) {
    const int bn = nb <= 64 ? 64 : nb <= 128 ? 128 : 256;
    const long long tiles = (long long)((m + TC_BM - 1) / TC_BM) * ((nb + bn - 1) / bn);
    while (ks < 8 && ks * 2 <= k / 256 && tiles * ks * 2 <= 148 && (size_t)ks * 2 * nb * m <= part_elems) ks *= 2;
  }
  float* dst = ks > 1 ? part : out;
  switch (q) {
    case Q4_K: e = launch_gemm_tc_q<Q4_K>(w, xh, xl, dst, m, k, nb, precise, ks, st, pitch); break;
    case Q5_K: e = launch_gemm_tc_q<Q5_K>(w, xh, xl, dst, m, k, nb, precise, ks, st, pitch); break;
    case Q6_K: e = launch_gemm_tc_q<Q6_K>(w, xh, xl, dst, m, k, nb, precise, ks, st, pitch); break;
    case Q8_0: e = launch_gemm_tc_q<Q8_0>(w, xh, xl, dst, m, k, nb, precise, ks, st, pitch); break;
    case TQ2_0: e = launch_gemm_tc_q<TQ2_0>(w, xh, xl, dst, m, k, nb, precise, ks, st, pitch); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || ks == 1) return e;
  const long long on = (long long)nb * m;
  cfg.gridDim = dim3((unsigned)std::min<long long>((on + 255) / 256, 148LL * 8));
  return cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, (const float*)part, out, on, ks);
}

}  // namespace vtb
