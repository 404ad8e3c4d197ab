// gemv_q8_mma.cu -- tensor-core decode GEMV for Q8_0 with f32 activations:
// y[m] = W[m,k] . x[k] (the reference's matmul_q8_0, src/kernels/simd.zig:159-190).
//
// Q8_0 blocks are 34 B per 32 weights (f16 d, then 32 int8 qs).  The qs bytes
// are the A operand of mma.m16n8k32.s8.s8 as they are -- no unpacking at all --
// and x goes in as the same four int8 limbs per 32-element block as in the
// Q4_K GEMV (gemv_mma.cu: x / 2^e ~ sum_c L_c 254^-c, block-diagonal B, two
// MMA passes for limbs (L0, L1) and (L2, L3)), so the int32 accumulators are
// exact dots per (row, block, limb).  Epilogue per (row, block):
// y += d * 2^e * sum_c D_c 254^-c -- the reference's total += d * block_dot,
// with fp32-class accuracy (tolerance-checked, <= 1e-4).
//
// Tiles are 16 rows x 8 blocks (272 B per row, one 2-D TMA box, rows 68 words
// = 4 (mod 32) apart, so fragment loads are conflict-free); even blocks start
// 2 bytes off a word boundary, and their qs words are rebuilt from two aligned
// loads with one byte permute.  Rows must sit on a 16-byte pitch, i.e.
// k % 256 == 0.  A landed tile is read out into registers at once (A words
// and the block scales), which frees its stage for the next copy.
//
// XQ = true is the Q8_0 x Q8_0 form (dot_i8, simd.zig:40-62): every CTA
// quantizes x per 32-block with the rule of vtb_cuda_quantize_q8_0 (CTA 0
// also stores the result in the caller's scratch), B holds one int8 column
// per block of the chunk, one MMA per (16 rows, block) gives the exact int32
// block dots, and y += (d_w * d_x) * dot.
namespace vtb {

constexpr int Q8M_ROWS = 16;
constexpr int Q8M_RB = 272;  // 8 blocks x 34 B
constexpr int Q8M_STAGE = Q8M_ROWS * Q8M_RB;

// Quantizes group gi of x (4 blocks of 32; this lane holds elements
// 4*lane .. 4*lane+3) to Q8_0 with the rule of vtb_cuda_quantize_q8_0
// (d = amax / 127, q = round(x * (1 / d)), IEEE division and rounding), into
// the B-fragment layout: block b at b*32 bytes, lane quad t's 8 bytes =
// k 4t..4t+3 | 16+4t..16+4t+3.  CTA 0 also writes qs and d to xq_out / dx_out.
__device__ __forceinline__ void quantize_group_q8(float4 a, int gi, int lane, int8_t* xq, float* dxs,
                                                  int8_t* __restrict__ xq_out, float* __restrict__ dx_out) {
  const int part = lane & 7, b = gi * 4 + (lane >> 3);
  float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float dd = __fdiv_rn(m, 127.0f);
  const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
  const uint32_t q0 = (uint32_t)(int)roundf(__fmul_rn(a.x, id)) & 0xffu;
  const uint32_t q1 = (uint32_t)(int)roundf(__fmul_rn(a.y, id)) & 0xffu;
  const uint32_t q2 = (uint32_t)(int)roundf(__fmul_rn(a.z, id)) & 0xffu;
  const uint32_t q3 = (uint32_t)(int)roundf(__fmul_rn(a.w, id)) & 0xffu;
  const uint32_t wq = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
  *reinterpret_cast<uint32_t*>(xq + b * 32 + (part & 3) * 8 + (part >> 2) * 4) = wq;
  if (part == 0) dxs[b] = dd;
  if (blockIdx.x == 0 && xq_out) {
    *reinterpret_cast<uint32_t*>(xq_out + b * 32 + 4 * part) = wq;
    if (part == 0) dx_out[b] = dd;
  }
}

template <int WARPS, int S, bool XQ>
__global__ void __launch_bounds__(WARPS * 32, 1)
gemv_q8_mma_kernel(const __grid_constant__ CUtensorMap wmap, const float* __restrict__ x, int8_t* __restrict__ xqg,
                   float* __restrict__ dxg, float* __restrict__ y, int M, int K, int ksplit, int accumulate) {
  VTB_TL(3);
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  uint8_t* ring = smem + warp * S * Q8M_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * S * Q8M_STAGE) + warp * S;
  float* red = reinterpret_cast<float*>(smem + WARPS * S * Q8M_STAGE + WARPS * S * 8);  // [WARPS][32]
  XShared xsh;
  xsh.xq = reinterpret_cast<int8_t*>(red + WARPS * 32);
  xsh.xs = reinterpret_cast<float2*>(xsh.xq + 4 * K);
  float* dxs = reinterpret_cast<float*>(xsh.xq + K);  // XQ: d_x per block after the k quants

  // Work split as in the Q4_K GEMV: 16-row units, ksplit (a power of two)
  // warps of a slot share a unit and split its K range by 256-weight chunks.
  const int kshift = __ffs(ksplit) - 1;
  const int slots = WARPS >> kshift, slot = warp >> kshift, kpart = warp & (ksplit - 1);
  const int nch = K / 256;
  const int nunits = (M + Q8M_ROWS - 1) / Q8M_ROWS;
  const int ngroups = (nunits + slots - 1) >> (__ffs(slots) - 1);
  const int my_groups = blockIdx.x < ngroups ? (ngroups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int my_chunks = kpart < nch ? ((nch - 1 - kpart) >> kshift) + 1 : 0;
  const int ntiles = my_groups * my_chunks;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  int iss_g = 0, iss_c = 0, iss_n = 0;
  auto issue_next = [&]() {
    if (iss_n >= ntiles) return;
    const int u = (blockIdx.x + iss_g * gridDim.x) * slots + slot;
    const int c = kpart + (iss_c << kshift), st = iss_n % S;
    if (lane == 0) {  // rows past M arrive zero-filled and count toward the box bytes
      mbar_expect_tx(&bars[st], (unsigned)Q8M_STAGE);
      tma_load_2d(ring + st * Q8M_STAGE, &wmap, c * (Q8M_RB / 4), u * Q8M_ROWS, &bars[st]);
    }
    ++iss_n;
    if (++iss_c == my_chunks) { iss_c = 0; ++iss_g; }
  };
#pragma unroll
  for (int i = 0; i < S; ++i) issue_next();

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();

  // A words of the 8 blocks (rows g, g+8; k = 4t.. and 16+4t..) and the
  // scales d of this lane's blocks t and 4+t for both rows.
  uint32_t A[8][4];
  float dsc[2][2];
  auto prep = [&](int tt) -> bool {
    const int st = tt % S;
    if (!mbar_wait_bounded(&bars[st], (unsigned)((tt / S) & 1))) return false;
    const uint8_t* r0 = ring + st * Q8M_STAGE + g * Q8M_RB;
    const uint8_t* r1 = r0 + 8 * Q8M_RB;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int o = 34 * b + 2 + 4 * t;  // qs[4t] of block b
      if (b & 1) {                       // 34b + 2 = 0 (mod 4): aligned
        A[b][0] = *reinterpret_cast<const uint32_t*>(r0 + o);
        A[b][1] = *reinterpret_cast<const uint32_t*>(r1 + o);
        A[b][2] = *reinterpret_cast<const uint32_t*>(r0 + o + 16);
        A[b][3] = *reinterpret_cast<const uint32_t*>(r1 + o + 16);
      } else {  // 2 (mod 4): bytes 2..3 of one aligned word and 0..1 of the next
        const uint32_t* p0 = reinterpret_cast<const uint32_t*>(r0 + o - 2);
        const uint32_t* p1 = reinterpret_cast<const uint32_t*>(r1 + o - 2);
        A[b][0] = __byte_perm(p0[0], p0[1], 0x5432);
        A[b][1] = __byte_perm(p1[0], p1[1], 0x5432);
        A[b][2] = __byte_perm(p0[4], p0[5], 0x5432);
        A[b][3] = __byte_perm(p1[4], p1[5], 0x5432);
      }
    }
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      const int b = XQ ? 2 * t + grp : 4 * grp + t;  // XQ: blocks 2t, 2t+1 (accumulator columns)
      dsc[grp][0] = h2f(*reinterpret_cast<const uint16_t*>(r0 + 34 * b));
      dsc[grp][1] = h2f(*reinterpret_cast<const uint16_t*>(r1 + 34 * b));
    }
    // The refill is an async-proxy write into the bytes just read: order
    // every lane's reads before it.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    issue_next();  // this stage's bytes are in registers: refill it
    return true;
  };

  bool ok;
  const int n4 = K / 128;
  const bool early_x = n4 <= 2 * WARPS;
  float4 xv0 = make_float4(0.f, 0.f, 0.f, 0.f), xv1 = xv0;
  if (early_x) {  // the activation loads fly while the first tile is read out
    if (warp < n4) xv0 = load_group(x, warp, lane, nullptr, 1.f);
    if (warp + WARPS < n4) xv1 = load_group(x, warp + WARPS, lane, nullptr, 1.f);
  }
  ok = ntiles == 0 || prep(0);
  if constexpr (XQ) {
    if (early_x) {
      if (warp < n4) quantize_group_q8(xv0, warp, lane, xsh.xq, dxs, xqg, dxg);
      if (warp + WARPS < n4) quantize_group_q8(xv1, warp + WARPS, lane, xsh.xq, dxs, xqg, dxg);
    } else {
      for (int gi = warp; gi < n4; gi += WARPS)
        quantize_group_q8(load_group(x, gi, lane, nullptr, 1.f), gi, lane, xsh.xq, dxs, xqg, dxg);
    }
  } else {
    if (early_x) {
      if (warp < n4) convert_group(xv0, warp, lane, xsh);
      if (warp + WARPS < n4) convert_group(xv1, warp + WARPS, lane, xsh);
    } else {
      build_x_shared(x, K, xsh, warp, lane, WARPS, nullptr, 1.f);
    }
  }
  __syncthreads();

  const int gs = g >> 1;                  // block (within a group of 4) whose B columns this lane holds
  const int boff = (g & 1) * 32 + t * 8;  // limb g&1, quad t

  for (int ui = 0; ui < my_groups; ++ui) {
    const int u = (blockIdx.x + ui * gridDim.x) * slots + slot;
    const int rbase = u * Q8M_ROWS, nr = max(0, min(Q8M_ROWS, M - rbase));
    float acc[2] = {0.f, 0.f};  // rows g, g+8
    for (int ci = 0; ci < my_chunks && ok; ++ci) {
      const int tt = ui * my_chunks + ci;
      const int cb = (kpart + (ci << kshift)) * 8;  // first block of the chunk
      if constexpr (XQ) {
        // column g = block cb + g; this lane's accumulators are blocks cb + 2t, cb + 2t + 1
        const uint2 bc = *reinterpret_cast<const uint2*>(xsh.xq + (cb + g) * 32 + 8 * t);
        int D[4] = {0, 0, 0, 0};
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const bool on = g == b;
          imma_s8(D, A[b][0], A[b][1], A[b][2], A[b][3], on ? bc.x : 0u, on ? bc.y : 0u);
        }
        const float dx0 = dxs[cb + 2 * t], dx1 = dxs[cb + 2 * t + 1];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          acc[i] = fmaf(dsc[0][i] * dx0, (float)D[2 * i], acc[i]);
          acc[i] = fmaf(dsc[1][i] * dx1, (float)D[2 * i + 1], acc[i]);
        }
      } else {
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int8_t* xb = xsh.xq + (cb + 4 * grp + gs) * 128 + boff;
        const uint2 bx = *reinterpret_cast<const uint2*>(xb);       // limb (g&1)
        const uint2 bz = *reinterpret_cast<const uint2*>(xb + 64);  // limb 2 + (g&1)
        int D[4] = {0, 0, 0, 0}, E[4] = {0, 0, 0, 0};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const bool on = gs == jj;
          const uint32_t* a = A[4 * grp + jj];
          imma_s8(D, a[0], a[1], a[2], a[3], on ? bx.x : 0u, on ? bx.y : 0u);
          imma_s8(E, a[0], a[1], a[2], a[3], on ? bz.x : 0u, on ? bz.y : 0u);
        }
        // D[0..1]: row g, limbs (L0, L1) of block 4 grp + t; D[2..3]: row g + 8.
        const float2 xs = xsh.xs[cb + 4 * grp + t];
        const float f = xs.x * (1.0f / 254.0f);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float hi = (float)(D[2 * i] * 254 + D[2 * i + 1]);
          const float lo = (float)(E[2 * i] * 254 + E[2 * i + 1]);
          acc[i] = fmaf(dsc[grp][i], fmaf(lo, 1.0f / 64516.0f, hi) * f, acc[i]);
        }
      }
      }
      if (tt + 1 < ntiles && !prep(tt + 1)) ok = false;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float v = acc[i];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (t == 0) red[warp * 32 + 8 * i + g] = v;
    }
    __syncthreads();
    if (kpart == 0 && lane < nr) {
      float v = 0.f;
      const int nk = min(ksplit, nch);
      for (int w = 0; w < nk; ++w) v += red[(warp + w) * 32 + lane];
      y[rbase + lane] = accumulate ? y[rbase + lane] + v : v;
    }
    __syncthreads();
  }
}

template <int WARPS, int S>
constexpr int q8_mma_smem(int k) {
  return WARPS * S * Q8M_STAGE + WARPS * S * 8 + WARPS * 128 + k * 4 + (k / 32) * 8;
}

// Rows must be 16-byte aligned and on a 16-byte pitch (k % 256 == 0) for the TMA boxes.
static bool q8_mma_ok(const void* w, int k) {
  return (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && k % 256 == 0 && q8_mma_smem<16, 1>(k) <= 227 * 1024;
}

template <int WARPS, int S, bool XQ>
static cudaError_t launch_q8_mma_t(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m,
                                   int k, cudaStream_t st, bool pdl, int accumulate) {
  constexpr auto kern = gemv_q8_mma_kernel<WARPS, S, XQ>;
  const int smem = q8_mma_smem<WARPS, S>(k);
  const uint64_t rbytes = (uint64_t)(k / 32) * 34;
  CUtensorMap wmap;
  if (!make_tmap(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, rbytes / 4, (uint64_t)m, rbytes, Q8M_RB / 4, Q8M_ROWS,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const int dev = current_device();
  cudaError_t ea = ensure_smem_attr<kern>(dev, smem);
  if (ea != cudaSuccess) return ea;
  const int sms = sm_count(dev), per_sm = ctas_per_sm<kern>(dev, WARPS * 32, smem);
  const int units = (m + Q8M_ROWS - 1) / Q8M_ROWS, nch = k / 256, cap = sms * per_sm;
  const int ksplit = pick_ksplit(units, nch, WARPS, cap);
  const int groups = (units + WARPS / ksplit - 1) / (WARPS / ksplit);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups < cap ? groups : cap);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, wmap, x, xq, dx, y, m, k, ksplit, accumulate);
}

// Two stages per warp for matrices above 2^24 weights when they fit, else one.
cudaError_t launch_gemv_q8_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                               int accumulate) {
  if ((long long)m * k > (1LL << 24) && q8_mma_smem<16, 2>(k) <= 227 * 1024)
    return launch_q8_mma_t<16, 2, false>(w, x, nullptr, nullptr, y, m, k, st, pdl, accumulate);
  return launch_q8_mma_t<16, 1, false>(w, x, nullptr, nullptr, y, m, k, st, pdl, accumulate);
}

// Q8_0 x Q8_0 in one launch: x (f32) is quantized inside the GEMV; the
// quantized x (k int8) and its scales (k/32) are also written to xq / dx.
cudaError_t launch_gemv_q8q8_mma(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m, int k,
                                 cudaStream_t st, bool pdl, int accumulate) {
  if ((long long)m * k > (1LL << 24) && q8_mma_smem<16, 2>(k) <= 227 * 1024)
    return launch_q8_mma_t<16, 2, true>(w, x, xq, dx, y, m, k, st, pdl, accumulate);
  return launch_q8_mma_t<16, 1, true>(w, x, xq, dx, y, m, k, st, pdl, accumulate);
}

}  // namespace vtb
