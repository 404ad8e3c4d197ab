// common.cuh -- shared device helpers for the vantablack B200 backend.
//
// Block formats (ggml, as restated by the reference at src/kernels/simd.zig):
//   Q8_0  34 B / 32 weights : f16 d | i8 qs[32]
//   Q4_K 144 B / 256        : f16 d | f16 dmin | u8 scales[12] | u8 qs[128]
//   Q5_K 176 B / 256        : f16 d | f16 dmin | u8 scales[12] | u8 qh[32] | u8 qs[128]
//   Q6_K 210 B / 256        : u8 ql[128] | u8 qh[64] | i8 sc[16] | f16 d
//   TQ2_0 66 B / 256        : u8 qs[64] (2-bit fields) | f16 d   (the reference's layout,
//                             src/kernels/simd.zig:436-472)
#pragma once
#include <atomic>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace vtb {

// Type ids are the reference's GgmlType values (src/core/parser.zig:31-64); TQ2_0 is 32 there.
enum Quant : int { F32 = 0, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, TQ2_0 = 32 };

template <int Q> struct Fmt;
template <> struct Fmt<Q8_0> { static constexpr int bytes = 34, elems = 32; };
template <> struct Fmt<Q4_K> { static constexpr int bytes = 144, elems = 256; };
template <> struct Fmt<Q5_K> { static constexpr int bytes = 176, elems = 256; };
template <> struct Fmt<Q6_K> { static constexpr int bytes = 210, elems = 256; };
template <> struct Fmt<TQ2_0> { static constexpr int bytes = 66, elems = 256; };

// ---- per-device launch facts ----
// Kernel attributes (the dynamic shared-memory opt-in) and occupancy are per
// device: a process that drives several GPUs must set them on each.  Caches
// are lock-free (races only repeat an idempotent query).
constexpr int VTB_MAX_DEVICES = 64;
inline int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d >= 0 && d < VTB_MAX_DEVICES ? d : 0;
}
inline int sm_count(int dev) {
  static std::atomic<int> cache[VTB_MAX_DEVICES];
  int v = cache[dev].load(std::memory_order_relaxed);
  if (!v) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (v < 1) v = 1;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}
// K-split of a persistent GEMV with `units` row units of `nch` K chunks each,
// `warps` warps per CTA and `cap` resident CTAs: the divisor d of `warps`
// (d <= nch) that minimises the per-warp critical path, rounds x ceil(nch/d),
// where `warps/d` units share a CTA and rounds = ceil(groups / grid).  Ties go
// to the larger grid (more SMs streaming), then to the smaller d.
inline int pick_ksplit(int units, int nch, int warps, int cap) {
  int best = 1;
  long long best_cost = -1, best_grid = 0;
  for (int d = 1; d <= warps && d <= nch; ++d) {
    if (warps % d) continue;
    const long long slots = warps / d, groups = (units + slots - 1) / slots;
    const long long grid = groups < cap ? groups : cap, rounds = (groups + grid - 1) / grid;
    const long long cost = rounds * ((nch + d - 1) / d);
    if (best_cost < 0 || cost < best_cost || (cost == best_cost && grid > best_grid)) {
      best = d;
      best_cost = cost;
      best_grid = grid;
    }
  }
  return best;
}

// Opt kernel KERN in to `bytes` of dynamic shared memory on device `dev` (once per size increase).
template <auto KERN>
cudaError_t ensure_smem_attr(int dev, int bytes) {
  static std::atomic<int> set[VTB_MAX_DEVICES];
  if (set[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(KERN, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) set[dev].store(bytes, std::memory_order_release);
  return e;
}
// Resident CTAs per SM of KERN at (threads, smem) on device `dev`; the last answer is cached per device.
template <auto KERN>
int ctas_per_sm(int dev, int threads, int smem) {
  static std::atomic<long long> cache[VTB_MAX_DEVICES];  // (smem << 16) | ctas
  const long long c = cache[dev].load(std::memory_order_relaxed);
  if (c && (c >> 16) == smem) return (int)(c & 0xffff);
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, KERN, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  if (n < 1) n = 1;
  cache[dev].store(((long long)smem << 16) | n, std::memory_order_relaxed);
  return n;
}

inline int64_t host_row_bytes(int q, int64_t k) {
  switch (q) {
    case F32: return 4 * k;
    case Q8_0: return (k / 32) * 34;
    case Q4_K: return (k / 256) * 144;
    case Q5_K: return (k / 256) * 176;
    case Q6_K: return (k / 256) * 210;
    case TQ2_0: return (k / 256) * 66;
    default: return -1;
  }
}
template <int Q>
__host__ __device__ __forceinline__ long long host_row_bytes_dev(long long k) {
  return (k / Fmt<Q>::elems) * Fmt<Q>::bytes;
}
inline int host_block_elems(int q) { return q == Q8_0 ? 32 : (q == F32 ? 1 : 256); }
inline bool host_quant_ok(int q) { return q == Q8_0 || q == Q4_K || q == Q5_K || q == Q6_K || q == TQ2_0; }

// Device-side error word.  Kernels that give up a bounded wait OR a code in
// here and return; the host reads it with vtb_cuda_check_device_error().
enum DevErr : unsigned { DEV_ERR_MBAR_TIMEOUT = 1u, DEV_ERR_BAD_ARG = 2u, DEV_ERR_PEER_TIMEOUT = 4u };
__device__ unsigned g_dev_error = 0;  // one definition: the library is a single translation unit

__device__ __forceinline__ void flag_error(unsigned code) { atomicOr(&g_dev_error, code); }

// Optional launch timeline (a development build with -DVTB_TIMELINE): block
// (0,0,0) of each instrumented kernel records its kernel id, SM, entry time,
// the time its griddepcontrol.wait returned and its exit time (globaltimer
// ns) into a ring read back by vtb_cuda_timeline.  Compiled out otherwise.
#ifdef VTB_TIMELINE
constexpr unsigned kTlRing = 16384;
__device__ unsigned long long g_tl[8 * kTlRing];
__device__ unsigned g_tl_n;
__device__ __forceinline__ unsigned long long tl_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
struct TlRec {
  unsigned long long t0 = 0, t1 = 0, mk[4] = {0, 0, 0, 0};
  int id;
  bool on;
  __device__ explicit TlRec(int i) : id(i) {
    on = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0;
    if (on) t0 = tl_now();
  }
  __device__ void waited() {
    if (on) t1 = tl_now();
  }
  __device__ void mark(int k) {
    if (on) mk[k] = tl_now();
  }
  __device__ ~TlRec() {
    if (!on) return;
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    const unsigned i = atomicAdd(&g_tl_n, 1u) % kTlRing;
    g_tl[8 * i] = (unsigned long long)id | ((unsigned long long)sm << 32);
    g_tl[8 * i + 1] = t0;
    g_tl[8 * i + 2] = t1 ? t1 : t0;
    g_tl[8 * i + 3] = tl_now();
    for (int k = 0; k < 4; ++k) g_tl[8 * i + 4 + k] = mk[k];
  }
};
#define VTB_TL(id) TlRec vtb_tl_rec_(id)
#define VTB_TL_WAITED() vtb_tl_rec_.waited()
#define VTB_TL_MARK(k) vtb_tl_rec_.mark(k)
#else
#define VTB_TL_MARK(k)
#define VTB_TL(id)
#define VTB_TL_WAITED()
#endif

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// ---- packed f32x2 arithmetic (sm_100a) ----
struct f2 { unsigned long long v; };
__device__ __forceinline__ f2 pk(float a, float b) {
  f2 r; asm("mov.b64 %0, {%1,%2};" : "=l"(r.v) : "f"(a), "f"(b)); return r;
}
__device__ __forceinline__ void unpk(f2 r, float& a, float& b) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(r.v));
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r; asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v)); return r;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r; asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v)); return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 r; asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v)); return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 r; asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v)); return r;
}
__device__ __forceinline__ float hsum(f2 a) { float x, y; unpk(a, x, y); return x + y; }

// Byte k of `v` as the float 2^23 + byte (exact): PRMT against 0x4B000000.
template <int K>
__device__ __forceinline__ float byte_magic(uint32_t v) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, K | (4 << 4) | (5 << 8) | (7 << 12)));
}

// ---- mbarrier + bulk copy (TMA, non-multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~max_iter polls (each try_wait itself
// suspends for a hardware-chosen time), flags DEV_ERR_MBAR_TIMEOUT.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, unsigned max_iter = 1u << 22) {
  for (unsigned i = 0; i < max_iter; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  flag_error(DEV_ERR_MBAR_TIMEOUT);
  return false;
}
// 1-D bulk copy global -> shared (both 16 B aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Four int8 limbs of four activations r (|r| < 2^22) in base 254, as the
// integer tensor-core GEMVs feed them: lw[c] packs limb c of elements 0..3
// (byte i = element i), with L_0 = rint(r) and L_c = rint((r_{c-1} -
// L_{c-1}) * 254).  t = r + 1.5*2^23 rounds to the nearest integer (ties to
// even, as rintf) and leaves L's two's-complement byte in t's low byte;
// -254 L = fma(t, -254, 254 * 1.5*2^23) is exact, and fma(r, 254, -254 L)
// rounds (r - L) * 254 once, exactly as the subtract-then-multiply does.
__device__ __forceinline__ void limbs254(float xv[4], uint32_t lw[4]) {
  constexpr float kMagic = 12582912.0f, kMagic254 = 12582912.0f * 254.0f;
#pragma unroll
  for (int li = 0; li < 4; ++li) {
    float tq[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) tq[c] = xv[c] + kMagic;
    const uint32_t lo = __byte_perm(__float_as_uint(tq[0]), __float_as_uint(tq[1]), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(tq[2]), __float_as_uint(tq[3]), 0x0040);
    lw[li] = __byte_perm(lo, hi, 0x5410);
    if (li < 3) {
#pragma unroll
      for (int c = 0; c < 4; ++c) xv[c] = fmaf(xv[c], 254.f, fmaf(tq[c], -254.f, kMagic254));
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace vtb
