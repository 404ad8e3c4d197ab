// gemv.cu -- SIMT decode GEMV y[m] = W[m,k] . x[k] for GGUF Q5_K / Q8_0 /
// TQ2_0 weights, Q6_K rows that are not 16-byte multiples, and the Q8_0 x Q8_0
// path, with f32 activations (the reference's matmul_q*_* in
// src/kernels/simd.zig:159-434, dispatched by forward.zig:552-627).  Q4_K and
// TMA-compatible Q6_K run on the integer tensor cores (gemv_mma.cu,
// gemv_q6k_mma.cu); launch_gemv dispatches Q6_K itself.
//
// Design (B200):
//  * Persistent CTAs of WARPS warps; each warp owns a stream of tiles.  A
//    tile is R weight rows x one chunk of CH blocks (CH = 8 super-blocks =
//    2048 columns for the K-quants, 32 blocks = 1024 columns for Q8_0).
//  * Weight bytes move HBM -> shared memory with 1-D bulk copies
//    (cp.async.bulk, no multicast) into an S-stage per-warp ring guarded by
//    mbarriers; the copies for the next S tiles are always in flight.
//  * Lane l of the warp dequantizes 64 weights (32 for Q8_0) of each row of
//    the tile straight from shared memory: quantized values become exact floats with
//    a byte-permute against the 0x4B000000 magic, and the products go
//    through packed f32x2 FMAs.  Sub-block scales are applied once per
//    sub-block: sum_l (d1*q_l - m1)*x_l = d1*sum_l q_l*x_l - m1*sum_l x_l.
//  * The lane's x slice lives in registers and is reused by all R rows.
//  * Programmatic dependent launch: weight copies for the first S tiles are
//    issued before griddepcontrol.wait, so a GEMV queued behind another
//    kernel streams its weights while the producer of x is still running.
//
// Results are fp32-accumulated; summation order differs from the
// reference's (it is tolerance-checked, max rel err <= 1e-4).
#include "common.cuh"

namespace vtb {


template <int Q> struct GemvCfg;
template <> struct GemvCfg<Q5_K> { static constexpr int CH = 8; };
template <> struct GemvCfg<Q6_K> { static constexpr int CH = 8; };
template <> struct GemvCfg<Q8_0> { static constexpr int CH = 32; };
template <> struct GemvCfg<TQ2_0> { static constexpr int CH = 8; };

template <int Q>
struct Slot {
  static constexpr int CH = GemvCfg<Q>::CH;
  static constexpr int BYTES = ((CH * Fmt<Q>::bytes + 16) + 15) / 16 * 16;  // room for a 15 B lead
};

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Read NW 32-bit words starting at a 2-byte-aligned shared address.
template <int NW>
__device__ __forceinline__ void lds_words_a2(const uint8_t* p, uint32_t* out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  uint32_t w[NW + 1];
#pragma unroll
  for (int i = 0; i <= NW; ++i) w[i] = lds32(base + 4 * i);
  const unsigned sh = (unsigned)(a & 3) * 8u;
#pragma unroll
  for (int i = 0; i < NW; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

__device__ __forceinline__ float4 ldx4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Lane's x slice for one chunk, as 32 packed pairs (64 floats) plus the
// sums the min/bias terms need.
struct XSlice {
  f2 v[32];
  float s0, s1;  // Q5_K: sums of the low / high 32
};

// ---------------- per-format lane kernels ----------------
// Each returns this lane's contribution to one row's dot for the chunk.

// Q4_K-style blocks (the Q5_K path): lane -> block b = lane>>2, sub-block pair j = lane&3
// (simd.zig:221-243).
__device__ __forceinline__ void load_x_kq(const float* x, int col0, XSlice& xs) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 a = ldx4(x + col0 + 4 * i);
    xs.v[2 * i] = pk(a.x, a.y);
    xs.v[2 * i + 1] = pk(a.z, a.w);
    s0 += (a.x + a.y) + (a.z + a.w);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 a = ldx4(x + col0 + 32 + 4 * i);
    xs.v[16 + 2 * i] = pk(a.x, a.y);
    xs.v[16 + 2 * i + 1] = pk(a.z, a.w);
    s1 += (a.x + a.y) + (a.z + a.w);
  }
  xs.s0 = s0;
  xs.s1 = s1;
}

__device__ __forceinline__ void kq_scale_min(uint4 h, int j, float& d1, float& m1, float& d2, float& m2) {
  const float d = h2f((uint16_t)(h.x & 0xffffu));
  const float dmin = h2f((uint16_t)(h.x >> 16));
  const unsigned i = 2u * (unsigned)(j & 1);
  const unsigned ya = (h.y >> (8 * i)) & 0xffu, za = (h.z >> (8 * i)) & 0xffu, wa = (h.w >> (8 * i)) & 0xffu;
  const unsigned yb = (h.y >> (8 * i + 8)) & 0xffu, zb = (h.z >> (8 * i + 8)) & 0xffu, wb = (h.w >> (8 * i + 8)) & 0xffu;
  unsigned sa, ma, sb, mb;
  if (j < 2) {  // q4kScaleMin, s < 4
    sa = ya & 63u; ma = za & 63u; sb = yb & 63u; mb = zb & 63u;
  } else {      // s >= 4
    sa = (wa & 15u) | ((ya >> 6) << 4); ma = (wa >> 4) | ((za >> 6) << 4);
    sb = (wb & 15u) | ((yb >> 6) << 4); mb = (wb >> 4) | ((zb >> 6) << 4);
  }
  d1 = d * (float)sa; m1 = dmin * (float)ma;
  d2 = d * (float)sb; m2 = dmin * (float)mb;
}

// Q5_K (simd.zig:290-319): the Q4_K nibble layout plus bit 2j / 2j+1 of qh[l] worth 16.
__device__ __forceinline__ float lane_dot_q5k(const uint8_t* blk, int j, const XSlice& xs) {
  const uint4 h = *reinterpret_cast<const uint4*>(blk);
  const uint4 ha = *reinterpret_cast<const uint4*>(blk + 16);
  const uint4 hb = *reinterpret_cast<const uint4*>(blk + 32);
  const uint4 qa = *reinterpret_cast<const uint4*>(blk + 48 + 32 * j);
  const uint4 qb = *reinterpret_cast<const uint4*>(blk + 64 + 32 * j);
  float d1, m1, d2, m2;
  kq_scale_min(h, j, d1, m1, d2, m2);
  const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
  const unsigned s0 = 2u * (unsigned)j, s1 = s0 + 1u;
  const f2 mg = pk(-8388608.f, -8388608.f);
  f2 a0 = pk(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t lo = (qw[w] & 0x0F0F0F0Fu) | (((hw[w] >> s0) & 0x01010101u) << 4);
    const uint32_t hi = ((qw[w] >> 4) & 0x0F0F0F0Fu) | (((hw[w] >> s1) & 0x01010101u) << 4);
    f2 l01 = add2(pk(byte_magic<0>(lo), byte_magic<1>(lo)), mg);
    f2 l23 = add2(pk(byte_magic<2>(lo), byte_magic<3>(lo)), mg);
    f2 h01 = add2(pk(byte_magic<0>(hi), byte_magic<1>(hi)), mg);
    f2 h23 = add2(pk(byte_magic<2>(hi), byte_magic<3>(hi)), mg);
    a0 = fma2(l01, xs.v[2 * w], a0);
    a1 = fma2(l23, xs.v[2 * w + 1], a1);
    b0 = fma2(h01, xs.v[16 + 2 * w], b0);
    b1 = fma2(h23, xs.v[16 + 2 * w + 1], b1);
  }
  return (d1 * hsum(add2(a0, a1)) - m1 * xs.s0) + (d2 * hsum(add2(b0, b1)) - m2 * xs.s1);
}

// Q6_K (simd.zig:366-404): lane -> block b = lane>>2, half = j>>1,
// l in [16*(j&1), +16).  Its 64 weights sit at half*128 + l + 32n, n=0..3.
__device__ __forceinline__ void load_x_q6k(const float* x, int col0, int j, XSlice& xs) {
  const int base = col0 + (j >> 1) * 128 + (j & 1) * 16;
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 a = ldx4(x + base + 32 * n + 4 * i);
      xs.v[8 * n + 2 * i] = pk(a.x, a.y);
      xs.v[8 * n + 2 * i + 1] = pk(a.z, a.w);
    }
  xs.s0 = xs.s1 = 0.f;
}

__device__ __forceinline__ float lane_dot_q6k(const uint8_t* blk, int j, const XSlice& xs) {
  const int half = j >> 1, lr = (j & 1) * 16;
  uint32_t A[4], Bw[4], H[4], S[2];
  lds_words_a2<4>(blk + half * 64 + lr, A);
  lds_words_a2<4>(blk + half * 64 + 32 + lr, Bw);
  lds_words_a2<4>(blk + 128 + half * 32 + lr, H);
  lds_words_a2<2>(blk + 192 + half * 8, S);  // sc[half*8 .. +8)
  const float d = h2f((uint16_t)(*reinterpret_cast<const uint16_t*>(blk + 208)));
  const int is = j & 1;
  // sc[is + 2n] for n = 0..3, as i8
  const uint32_t sw = (is ? (S[0] >> 8) | (S[1] << 24) : S[0]);  // bytes is, is+1, .. of sc[0..3]
  const uint32_t sw2 = (is ? (S[1] >> 8) : S[1]);
  const float sc0 = (float)(int8_t)(sw & 0xff), sc1 = (float)(int8_t)((sw >> 16) & 0xff);
  const float sc2 = (float)(int8_t)(sw2 & 0xff), sc3 = (float)(int8_t)((sw2 >> 16) & 0xff);
  const f2 mg = pk(-8388640.f, -8388640.f);  // 2^23 + 32
  f2 acc[4][2];
#pragma unroll
  for (int n = 0; n < 4; ++n) acc[n][0] = acc[n][1] = pk(0.f, 0.f);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t qv[4];
    qv[0] = (A[t] & 0x0F0F0F0Fu) | ((H[t] << 4) & 0x30303030u);
    qv[1] = (Bw[t] & 0x0F0F0F0Fu) | ((H[t] << 2) & 0x30303030u);
    qv[2] = ((A[t] >> 4) & 0x0F0F0F0Fu) | (H[t] & 0x30303030u);
    qv[3] = ((Bw[t] >> 4) & 0x0F0F0F0Fu) | ((H[t] >> 2) & 0x30303030u);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      f2 p01 = add2(pk(byte_magic<0>(qv[n]), byte_magic<1>(qv[n])), mg);
      f2 p23 = add2(pk(byte_magic<2>(qv[n]), byte_magic<3>(qv[n])), mg);
      acc[n][0] = fma2(p01, xs.v[8 * n + 2 * t], acc[n][0]);
      acc[n][1] = fma2(p23, xs.v[8 * n + 2 * t + 1], acc[n][1]);
    }
  }
  return d * (((sc0 * hsum(add2(acc[0][0], acc[0][1])) + sc1 * hsum(add2(acc[1][0], acc[1][1]))) +
               sc2 * hsum(add2(acc[2][0], acc[2][1]))) + sc3 * hsum(add2(acc[3][0], acc[3][1])));
}

// TQ2_0 (simd.zig:436-498, the reference's layout): lane -> block b = lane>>2,
// group j = lane&3 (weights 64j..64j+63).  Weight 64j + l takes the 2-bit field
// at bits 2j of qs[16j + l % 16], so weights l, l+16, l+32, l+48 of the group
// share one value: the lane folds its 64 activations into 16 sums.
__device__ __forceinline__ void load_x_tq2(const float* x, int col0, XSlice& xs) {
  float4 a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = ldx4(x + col0 + 4 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // fold l, l+16, l+32, l+48 (l = 4i..4i+3)
    const float4 p = a[i], q = a[4 + i], r = a[8 + i], s = a[12 + i];
    xs.v[2 * i] = pk((p.x + q.x) + (r.x + s.x), (p.y + q.y) + (r.y + s.y));
    xs.v[2 * i + 1] = pk((p.z + q.z) + (r.z + s.z), (p.w + q.w) + (r.w + s.w));
  }
  xs.s0 = xs.s1 = 0.f;
}

__device__ __forceinline__ float lane_dot_tq2(const uint8_t* blk, int j, const XSlice& xs) {
  uint32_t q[4], dw[1];
  lds_words_a2<4>(blk + 16 * j, q);
  lds_words_a2<1>(blk + 64, dw);
  const float d = h2f((uint16_t)(dw[0] & 0xffffu));
  const f2 mg = pk(-8388609.f, -8388609.f);  // 2^23 + 1: raw field -> raw - 1
  f2 a0 = pk(0.f, 0.f), a1 = a0;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t r = (q[t] >> (2 * j)) & 0x03030303u;
    a0 = fma2(add2(pk(byte_magic<0>(r), byte_magic<1>(r)), mg), xs.v[2 * t], a0);
    a1 = fma2(add2(pk(byte_magic<2>(r), byte_magic<3>(r)), mg), xs.v[2 * t + 1], a1);
  }
  return d * hsum(add2(a0, a1));
}

// Q8_0 (simd.zig:159-190): lane -> one 32-weight block.
__device__ __forceinline__ void load_x_q80(const float* x, int col0, XSlice& xs) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 a = ldx4(x + col0 + 4 * i);
    xs.v[2 * i] = pk(a.x, a.y);
    xs.v[2 * i + 1] = pk(a.z, a.w);
  }
  xs.s0 = xs.s1 = 0.f;
}

__device__ __forceinline__ float lane_dot_q80(const uint8_t* blk, const XSlice& xs) {
  uint32_t w[9];
  lds_words_a2<9>(blk, w);  // d (2 B) + 32 qs + 2 B of the next block
  const float d = h2f((uint16_t)(w[0] & 0xffffu));
  const f2 mg = pk(-8388736.f, -8388736.f);  // 2^23 + 128
  f2 a0 = pk(0.f, 0.f), a1 = a0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t q = __funnelshift_r(w[t], w[t + 1], 16) ^ 0x80808080u;  // i8 -> u8 = q + 128
    a0 = fma2(add2(pk(byte_magic<0>(q), byte_magic<1>(q)), mg), xs.v[2 * t], a0);
    a1 = fma2(add2(pk(byte_magic<2>(q), byte_magic<3>(q)), mg), xs.v[2 * t + 1], a1);
  }
  return d * hsum(add2(a0, a1));
}

// Q8_0 x Q8_0: x pre-quantized to i8 per 32-block (quantize_q8_0_kernel);
// the block dot is an exact int32 sum (dot_i8, simd.zig:40-62) and the row
// sums (d_w * d_x) * float(dot) over blocks.
struct XQSlice {
  int4 q[2];
  float d;
};

__device__ __forceinline__ float lane_dot_q80_i8(const uint8_t* blk, const XQSlice& xq) {
  uint32_t w[9];
  lds_words_a2<9>(blk, w);
  const float d = h2f((uint16_t)(w[0] & 0xffffu));
  const int xw[8] = {xq.q[0].x, xq.q[0].y, xq.q[0].z, xq.q[0].w, xq.q[1].x, xq.q[1].y, xq.q[1].z, xq.q[1].w};
  int dot = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) dot = __dp4a((int)__funnelshift_r(w[t], w[t + 1], 16), xw[t], dot);
  return (d * xq.d) * (float)dot;
}

// ---------------- the persistent pipelined kernel ----------------
// XQ: activations are Q8_0-quantized (xv = i8[K], dx = f32[K/32]) instead
// of f32 (xv = f32[K]).
template <int Q, int R, int S, int WARPS, bool XQ>
__global__ void __launch_bounds__(WARPS * 32)
gemv_kernel(const uint8_t* __restrict__ W, const void* __restrict__ xv, const float* __restrict__ dx,
            float* __restrict__ y, int M, int K, int accumulate, long long pitch) {
  VTB_TL(4);
  const float* x = static_cast<const float*>(xv);
  constexpr int CH = GemvCfg<Q>::CH, BB = Fmt<Q>::bytes, EL = Fmt<Q>::elems;
  constexpr int SLOT = Slot<Q>::BYTES, STAGE = R * SLOT;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * S * STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * S * STAGE) + warp * S;

  const int nb = K / EL, nch = (nb + CH - 1) / CH;
  const long long rb = pitch;  // bytes between rows
  const int ngroups = (M + R - 1) / R;
  const int gw = blockIdx.x * WARPS + warp, NW = gridDim.x * WARPS;
  const int my_groups = gw < ngroups ? (ngroups - 1 - gw) / NW + 1 : 0;
  const int ntiles = my_groups * nch;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto issue = [&](int t) {  // lane 0 only
    const int g = gw + (t / nch) * NW, c = t % nch, st = t % S;
    const int b0 = c * CH, nblk = min(CH, nb - b0);
    const int r0 = g * R, nr = min(R, M - r0);
    unsigned total = 0;
    unsigned sizes[R];
    const uint8_t* srcs[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sizes[r] = 0;
      if (r < nr) {
        const uint8_t* src = W + (long long)(r0 + r) * rb + (long long)b0 * BB;
        const uint8_t* al = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
        const unsigned lead = (unsigned)(src - al);
        sizes[r] = (lead + (unsigned)(nblk * BB) + 15u) & ~15u;
        srcs[r] = al;
        total += sizes[r];
      }
    }
    mbar_expect_tx(&bars[st], total);
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (sizes[r]) bulk_g2s(ring + st * STAGE + r * SLOT, srcs[r], sizes[r], &bars[st]);
  };

  if (lane == 0)
    for (int t = 0; t < min(S, ntiles); ++t) issue(t);

  // x is produced by the previous kernel in the stream: wait for it only now.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  asm volatile("griddepcontrol.launch_dependents;");

  XSlice xs;
  XQSlice xqs;
  int x_chunk = -1;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  const int bl = (Q == Q8_0) ? lane : (lane >> 2);
  const int j = lane & 3;

  for (int t = 0; t < ntiles; ++t) {
    const int g = gw + (t / nch) * NW, c = t % nch, st = t % S;
    const int b0 = c * CH, nblk = min(CH, nb - b0);
    const int r0 = g * R, nr = min(R, M - r0);
    const bool active = bl < nblk;
    if (c != x_chunk) {
      if (active) {
        if constexpr (XQ) {
          const int4* p = reinterpret_cast<const int4*>(static_cast<const int8_t*>(xv) + (b0 + bl) * 32);
          xqs.q[0] = __ldg(p);
          xqs.q[1] = __ldg(p + 1);
          xqs.d = __ldg(dx + b0 + bl);
        } else if constexpr (Q == Q8_0) load_x_q80(x, (b0 + bl) * 32, xs);
        else if constexpr (Q == Q6_K) load_x_q6k(x, (b0 + bl) * 256, j, xs);
        else if constexpr (Q == TQ2_0) load_x_tq2(x, (b0 + bl) * 256 + 64 * j, xs);
        else load_x_kq(x, (b0 + bl) * 256 + 64 * j, xs);
      }
      x_chunk = c;
    }
    if (!mbar_wait_bounded(&bars[st], (unsigned)((t / S) & 1))) {
      // Gave up (error word set).  Do not leave the CTA while copies into its
      // shared memory may still land: drain every stage issued so far with a
      // short bounded wait, compute nothing more, then return.
      for (int u = t + 1; u < min(t + S, ntiles); ++u) mbar_wait_bounded(&bars[u % S], (unsigned)((u / S) & 1), 1u << 16);
      return;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nr && active) {
        const uint8_t* src = W + (long long)(r0 + r) * rb + (long long)b0 * BB;
        const unsigned lead = (unsigned)(reinterpret_cast<uintptr_t>(src) & 15u);
        const uint8_t* blk = ring + st * STAGE + r * SLOT + lead + bl * BB;
        float v;
        if constexpr (Q == Q5_K) v = lane_dot_q5k(blk, j, xs);
        else if constexpr (Q == Q6_K) v = lane_dot_q6k(blk, j, xs);
        else if constexpr (Q == TQ2_0) v = lane_dot_tq2(blk, j, xs);
        else if constexpr (XQ) v = lane_dot_q80_i8(blk, xqs);
        else v = lane_dot_q80(blk, xs);
        acc[r] += v;
      }
    }
    __syncwarp();
    if (lane == 0 && t + S < ntiles) issue(t + S);
    if (c == nch - 1) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float s = warp_sum(acc[r]);
        if (lane == r && r < nr) y[r0 + r] = accumulate ? y[r0 + r] + s : s;
        acc[r] = 0.f;
      }
    }
  }
}

// ---------------- host launcher ----------------
template <int Q, int R, int S, int WARPS, bool XQ = false>
static cudaError_t launch_gemv_t(const void* w, const void* x, const float* dx, float* y, int m, int k,
                                 cudaStream_t st, bool pdl, int accumulate = 0, long long pitch = 0) {
  if (pitch == 0) pitch = host_row_bytes(Q, k);
  auto kern = gemv_kernel<Q, R, S, WARPS, XQ>;
  constexpr int smem = WARPS * S * R * Slot<Q>::BYTES + WARPS * S * 8;
  const int dev = current_device();
  cudaError_t e = ensure_smem_attr<gemv_kernel<Q, R, S, WARPS, XQ>>(dev, smem);
  if (e != cudaSuccess) return e;
  const int sms = sm_count(dev), max_ctas_per_sm = ctas_per_sm<gemv_kernel<Q, R, S, WARPS, XQ>>(dev, WARPS * 32, smem);
  const int ngroups = (m + R - 1) / R;
  int grid = (ngroups + WARPS - 1) / WARPS;
  grid = grid < sms * max_ctas_per_sm ? grid : sms * max_ctas_per_sm;
  if (grid < 1) grid = 1;
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
  return cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)w, x, dx, y, m, k, accumulate, pitch);
}

cudaError_t launch_gemv_q8_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                               int accumulate);
static bool q8_mma_ok(const void* w, int k);
cudaError_t launch_gemv_q5k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate);

// `pitch`: bytes between consecutive weight rows (0 = the dense row size).
cudaError_t launch_gemv_pitched(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st,
                                bool pdl, int accumulate, long long pitch) {
  if (pitch == 0) pitch = host_row_bytes(q, k);
  switch (q) {
    case Q5_K:  // integer tensor cores on dense, 16-byte aligned rows
      if (pitch == host_row_bytes(Q5_K, k) && (reinterpret_cast<uintptr_t>(w) & 15u) == 0)
        return launch_gemv_q5k_mma(w, x, y, m, k, st, pdl, accumulate);
      return launch_gemv_t<Q5_K, 4, 4, 4>(w, x, nullptr, y, m, k, st, pdl, accumulate, pitch);
    case Q6_K:  // integer tensor cores when rows sit on 16-byte pitches
      if (q6k_mma_ok(w, k, pitch)) return launch_gemv_q6k_mma(w, x, y, m, k, st, pdl, accumulate, pitch);
      return launch_gemv_t<Q6_K, 4, 4, 4>(w, x, nullptr, y, m, k, st, pdl, accumulate, pitch);
    case Q8_0:  // integer tensor cores when rows sit on 16-byte pitches
      if (pitch == host_row_bytes(Q8_0, k) && q8_mma_ok(w, k)) return launch_gemv_q8_mma(w, x, y, m, k, st, pdl, accumulate);
      return launch_gemv_t<Q8_0, 4, 4, 4>(w, x, nullptr, y, m, k, st, pdl, accumulate, pitch);
    case TQ2_0: return launch_gemv_t<TQ2_0, 4, 4, 4>(w, x, nullptr, y, m, k, st, pdl, accumulate, pitch);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                        int accumulate) {
  return launch_gemv_pitched(q, w, x, y, m, k, st, pdl, accumulate, 0);
}

cudaError_t launch_gemv_q8_0_q8_0(const void* w, const int8_t* xq, const float* dx, float* y, int m, int k,
                                  cudaStream_t st, bool pdl, int accumulate) {
  return launch_gemv_t<Q8_0, 4, 4, 4, true>(w, xq, dx, y, m, k, st, pdl, accumulate);
}

cudaError_t launch_quantize_q8_0(const float* x, int8_t* qs, float* d, int nblocks, cudaStream_t st);
cudaError_t launch_gemv_q8q8_mma(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m, int k,
                                 cudaStream_t st, bool pdl, int accumulate);

// Q8_0 x Q8_0 from f32 x: x is quantized per 32-block into xq / dx (k int8 and
// k/32 scales) and the GEMV takes the int8 dots.  On 16-byte row pitches one
// tensor-core kernel does both (every CTA quantizes x itself; CTA 0 stores
// xq / dx); otherwise the quantizer runs first and the SIMT GEMV reads xq / dx.
cudaError_t launch_gemv_q8_0_q8_0_x(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m, int k,
                                    cudaStream_t st, bool pdl, int accumulate) {
  if (q8_mma_ok(w, k)) return launch_gemv_q8q8_mma(w, x, xq, dx, y, m, k, st, pdl, accumulate);
  cudaError_t e = launch_quantize_q8_0(x, xq, dx, k / 32, st);
  if (e != cudaSuccess) return e;
  return launch_gemv_t<Q8_0, 4, 4, 4, true>(w, xq, dx, y, m, k, st, pdl, accumulate);
}

}  // namespace vtb
