// model.cu -- the Llama forward loop on the GPU: the CUDA counterpart of the
// reference's CPU backend (src/runtime/backend_cpu.zig layerStep/finalStep)
// and Metal segment (src/runtime/forward.zig:419-520), behind the vtable
// seam of src/runtime/backend.zig:67-97.
//
// Device state per VtbCudaState:
//   x[rows][dim]        residual stream (forward.zig State.x)
//   xb[rows][dim]       normed activations
//   qkv[rows][qd+2kvd]  fused Q|K|V projection output
//   att[rows][qd]       attention output
//   gu[rows][2*ffn]     fused gate|up output, h[rows][ffn] = swiglu
//   logits[rows][vocab], argmax[rows]
//   kv cache: K and V, f32, [seq][layer][max_seq][n_kv_heads*head_dim]
//             (kv_cache.zig:20-73 layout, one slab per sequence)
// Row r of a step is token `tok[r]` of sequence `seq[r]` at position
// `pos[r]`: a decode step has one row per sequence, a prefill step has one
// row per prompt token of one sequence (prefill.zig:111-232 semantics).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/vtb_cuda.h"
#include "common.cuh"

namespace vtb {

cudaError_t launch_gemv(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                        int accumulate);
cudaError_t launch_gemv_pitched(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st,
                                bool pdl, int accumulate, long long pitch);
cudaError_t launch_gemv_q4k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate, const float* norm_w, float eps, float* swi);
cudaError_t launch_embed(int q, const void* table, const int32_t* ids, float* out, int dim, int n_tok,
                         cudaStream_t st);
cudaError_t launch_gemm_tc(int q, const void* w, const float* acts, float* out, int m, int k, int nb, bool precise,
                           void* ws, cudaStream_t st, float* part, size_t part_elems, long long pitch);

// Prefill steps with at least this many rows run their projections as one
// tensor-core GEMM (precise mode) instead of one GEMV per row.
constexpr int GEMM_MIN_ROWS = 8;

// x += t (addInto, math.zig:178-187) for the GEMM path's residual adds.
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ t, long long n) {
  VTB_TL(7);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    x[i] += t[i];
}

cudaError_t launch_gemv_q8_0_q8_0(const void* w, const int8_t* xq, const float* dx, float* y, int m, int k,
                                  cudaStream_t st, bool pdl, int accumulate);
cudaError_t launch_quantize_q8_0(const float* x, int8_t* qs, float* d, int nblocks, cudaStream_t st);
cudaError_t launch_gemv_q8_0_q8_0_x(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m, int k,
                                    cudaStream_t st, bool pdl, int accumulate);


// `pitch`: bytes between weight rows (0 = dense; only Q6_K rows are ever padded).
static cudaError_t gemv_any(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st,
                            int accumulate, long long pitch = 0) {
  if (q == Q4_K) return launch_gemv_q4k_mma(w, x, y, m, k, st, true, accumulate, nullptr, 0.f, nullptr);
  return launch_gemv_pitched(q, w, x, y, m, k, st, true, accumulate, pitch);
}

// ---------------- kernels ----------------

// rmsNorm (math.zig:11-32): out = (x * w) * (1 / sqrt(mean(x^2) + eps)), one
// CTA per row.  With `res`, the row is first updated x += res (the residual
// add of addInto, math.zig:178-187, fused; used after a tensor-parallel
// all-reduce).
__global__ void rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ res, const float* __restrict__ w,
                               float* __restrict__ out, int n, float eps) {
  VTB_TL(8);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  const int r = blockIdx.x;
  float* xr = x + (long long)r * n;
  const float* rr = res ? res + (long long)r * n : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xr[i];
    if (rr) {
      v += rr[i];
      xr[i] = v;
    }
    ss += v * v;
  }
  __shared__ float part[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) part[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(part[0] / (float)n + eps);
  float* o = out + (long long)r * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = (xr[i] * w[i]) * inv;
}

// ---- tensor-parallel all-reduce over NVLink peer memory ----
// Each rank's row-parallel projection (O, down) writes its partial into a
// double-buffered slot of an IPC-shared block; tp_signal_kernel then raises
// this rank's epoch flag in every peer's block; the consumer,
// rmsnorm_tp_kernel, waits (bounded) for all peers' flags and sums the
// partials straight out of peer memory, fused with the residual add and the
// RMSNorm that follows the collective in the layer.  Every rank sums in rank
// order, so all ranks hold bit-identical residuals.  Slot e % 2 is rewritten
// only after every peer's flag for e + 1 was seen, which a peer raises after
// its consumer of e has run: no overwrite while a peer still reads.
constexpr int TP_MAX = 8;
struct PeerPtrs {
  float* p[TP_MAX];  // each rank's shared block (this rank's own included)
};
// Shared block: [2][max_rows * dim] partial slots | flags[TP_MAX] | epoch.
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Raise this rank's flag to the next epoch in every peer's block (one thread;
// called after griddepcontrol.wait, i.e. once this rank's partial is complete).
__device__ __forceinline__ void tp_raise_flag(const PeerPtrs& peers, int world, int me, long long flag_off) {
  unsigned* mine = reinterpret_cast<unsigned*>(peers.p[me] + flag_off);
  const unsigned e = mine[TP_MAX] + 1;  // epoch: one per all-reduce, identical on every rank
  mine[TP_MAX] = e;
  __threadfence_system();
  for (int r = 0; r < world; ++r)
    if (r != me) st_release_sys(reinterpret_cast<unsigned*>(peers.p[r] + flag_off) + me, e);
}

__global__ void tp_signal_kernel(PeerPtrs peers, int world, int me, long long flag_off) {
  VTB_TL(9);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the partial of this rank is complete
  VTB_TL_WAITED();
  if (threadIdx.x == 0) tp_raise_flag(peers, world, me, flag_off);
}

// x[r] += sum over ranks of slot[r] (peer loads), then out = RMSNorm(x) as rmsnorm_kernel.
// n % 4 == 0 always holds: model creation requires dim = n_heads * head_dim with
// head_dim % 8 == 0, so the float4 loop below covers every element.
__global__ void __launch_bounds__(1024) rmsnorm_tp_kernel(float* __restrict__ x, PeerPtrs peers, int world, int me, long long slot_off,
                                  long long flag_off, const float* __restrict__ w, float* __restrict__ out, int n,
                                  float eps, int signal) {
  VTB_TL(10);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  if (threadIdx.x == 0) {
    if (signal) tp_raise_flag(peers, world, me, flag_off);  // single-CTA launch: publish, then wait
    const unsigned* flags = reinterpret_cast<const unsigned*>(peers.p[me] + flag_off);
    const unsigned e = flags[TP_MAX];
    for (int r = 0; r < world; ++r) {
      if (r == me) continue;
      unsigned it = 0;
      while ((int)(ld_acquire_sys(flags + r) - e) < 0) {  // bounded: a missing peer flags an error, never hangs
        if (++it > (1u << 24)) {
          flag_error(DEV_ERR_PEER_TIMEOUT);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  const int r = blockIdx.x;
  float* xr = x + (long long)r * n;
  float ss = 0.f;
  // One 16-byte load per rank per thread, all issued before any is used: the
  // remote reads cost one NVLink round trip, not one per element.  (.cv: a
  // slot's previous contents may sit in this SM's L1.)
  for (int i4 = threadIdx.x; i4 < n / 4; i4 += blockDim.x) {
    float4 pv[TP_MAX];
#pragma unroll
    for (int q = 0; q < TP_MAX; ++q)
      if (q < world) pv[q] = __ldcv(reinterpret_cast<const float4*>(peers.p[q] + slot_off + (long long)r * n) + i4);
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < TP_MAX; ++q)
      if (q < world) {
        sum.x += pv[q].x; sum.y += pv[q].y; sum.z += pv[q].z; sum.w += pv[q].w;
      }
    float4 v = reinterpret_cast<float4*>(xr)[i4];
    v.x += sum.x; v.y += sum.y; v.z += sum.z; v.w += sum.w;
    reinterpret_cast<float4*>(xr)[i4] = v;
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  __shared__ float part[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) part[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(part[0] / (float)n + eps);
  float* o = out + (long long)r * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = (xr[i] * w[i]) * inv;
}

// rope (math.zig:88-104, interleaved pairs) on the row's Q and K heads, then
// the KV-cache write of K and V at the row's position (forward.zig:268-269).
struct RowInfo {
  const int32_t* seq;
  const int32_t* pos;
};

__global__ void rope_kv_kernel(float* __restrict__ qkv, float* __restrict__ kc, float* __restrict__ vc, RowInfo ri,
                               int layer, int n_layers, int max_seq, int n_heads, int n_kv, int hd,
                               const float* __restrict__ rope) {
  VTB_TL(11);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  const int r = blockIdx.x;
  const int qd = n_heads * hd, kvd = n_kv * hd, stride = qd + 2 * kvd;
  float* q = qkv + (long long)r * stride;
  float* k = q + qd;
  const float* v = k + kvd;
  const int pos = ri.pos[r], seq = ri.seq[r];
  const long long slot = (((long long)seq * n_layers + layer) * max_seq + pos) * kvd;
  const int half = hd / 2;
  const float2* cs = reinterpret_cast<const float2*>(rope + (long long)pos * hd);
  for (int p = threadIdx.x; p < (n_heads + n_kv) * half; p += blockDim.x) {
    const int h = p / half, i = 2 * (p % half);
    const float2 t = cs[i / 2];
    const float c = t.x, s = t.y;
    float* ptr = h < n_heads ? q + h * hd + i : k + (h - n_heads) * hd + i;
    const float x0 = ptr[0], x1 = ptr[1];
    const float a = x0 * c, b = x1 * s, pp = x0 * s, qq = x1 * c;
    const float y0 = a - b, y1 = pp + qq;
    if (h < n_heads) {
      ptr[0] = y0;
      ptr[1] = y1;
    } else {
      kc[slot + (h - n_heads) * hd + i] = y0;
      kc[slot + (h - n_heads) * hd + i + 1] = y1;
    }
  }
  for (int i = threadIdx.x; i < kvd; i += blockDim.x) vc[slot + i] = v[i];
}

// Decode/causal attention (cpuAttention forward.zig:187-228, attentionCausal
// prefill.zig:237-287): row r attends positions [0, pos[r]] of its sequence.
// Split-K ("flash decode"): CTA (kv_head, row, split) handles positions
// [split*CHUNK, ...) for the GQA group of q heads that share the kv head,
// and writes a partial (max, sum, acc[hd]) per q head; attn_combine merges.
constexpr int ATT_CHUNK = 64;  // prefill attention: positions per staged K/V chunk
constexpr int DEC_CHUNK = 64;  // decode attention: positions per split
constexpr int ATT_THREADS = 128;
constexpr int ATT_GMAX = 8;  // GQA group sizes up to 8 keep their accumulators in registers

constexpr int ATT_PAD = 8;  // floats of padding per staged K/V row: the score pass reads conflict-free
constexpr int ATT_TPP = ATT_THREADS / DEC_CHUNK;  // score pass: threads per position
static_assert(ATT_TPP * DEC_CHUNK == ATT_THREADS && (ATT_TPP & (ATT_TPP - 1)) == 0 && ATT_TPP <= 32,
              "score pass: a power-of-two number of threads per position");

// Shared-memory floats of one attention CTA: q [G][hd], scores [G][CHUNK] (reused
// as the PV reduction [slices][G][hd]), staged K and V [CHUNK][hd + PAD].
__host__ __device__ inline int attn_smem_floats(int G, int hd) {
  const int slices = ATT_THREADS / hd > 0 ? ATT_THREADS / hd : 1;
  const int scf = G * DEC_CHUNK > slices * G * hd ? G * DEC_CHUNK : slices * G * hd;
  return G * hd + scf + 2 * DEC_CHUNK * (hd + ATT_PAD);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// One CTA per (kv head, row, split slot): partial softmax-attention of the G
// query heads sharing the kv head (attention math of forward.zig's layer loop,
// split flash-decoding style over DEC_CHUNK-position chunks; the splits merge in
// attn_combine_kernel).  The grid holds about one wave: a CTA walks the row's
// live splits sp, sp + gridDim.z, ...  Each split's K and V rows go to shared
// memory in one round of 16-byte async copies, so a CTA waits on DRAM once per
// split instead of once per position.
template <int GT>  // GT: compile-time group size, or 0 for the generic path
__global__ void __launch_bounds__(ATT_THREADS)
attn_partial_kernel(const float* __restrict__ qkv, const float* __restrict__ kc, const float* __restrict__ vc,
                    RowInfo ri, int layer, int n_layers, int max_seq, int n_heads, int n_kv, int hd,
                    float* __restrict__ part, int nsplit, float* __restrict__ kcw, float* __restrict__ vcw,
                    const float* __restrict__ rope) {
  VTB_TL(12);
  // kcw / vcw non-null: decode step with RoPE + KV write fused in (rope_kv_kernel's
  // work): q is rotated in shared memory, and the split that holds the row's
  // position rotates its K and writes K and V to the cache and to its staged rows.
  // The cached K/V rows of earlier positions were written by earlier steps, so
  // in that case the first split's copies are issued before griddepcontrol.wait
  // and their DRAM latency overlaps the QKV projection still running.
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.x, r = blockIdx.y;
  int sp = blockIdx.z;
  const int G = GT ? GT : n_heads / n_kv;
  const int qd = n_heads * hd, kvd = n_kv * hd;
  const int pos = ri.pos[r], seq = ri.seq[r];  // host-staged before the step's first kernel
  const int len = pos + 1, nsp = (len + DEC_CHUNK - 1) / DEC_CHUNK;
  if (sp >= nsp) {  // attn_combine_kernel reads only live splits
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  const int slices = ATT_THREADS / hd > 0 ? ATT_THREADS / hd : 1;
  const int scf = G * DEC_CHUNK > slices * G * hd ? G * DEC_CHUNK : slices * G * hd;
  const int ks = hd + ATT_PAD, h4 = hd / 4;
  float* qs = sm;           // [G][hd]
  float* sc = sm + G * hd;  // [G][DEC_CHUNK]
  float* kst = sc + scf;    // [DEC_CHUNK][ks]
  float* vst = kst + DEC_CHUNK * ks;
  const long long lbase = ((long long)seq * n_layers + layer) * max_seq;
  // Stage split sp's K and V rows (all but the row this step writes itself).
  // One bulk copy per K row and per V row (hd * 4 bytes each, 16-byte aligned
  // rows), issued by warp 0 and counted on two mbarriers (K, V); the split's
  // k-th staging completes phase k & 1 of both.
  __shared__ __align__(8) uint64_t kvbar[2];
  if (threadIdx.x == 0) {
    mbar_init(&kvbar[0], 1);
    mbar_init(&kvbar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int lane0 = threadIdx.x & 31;
  auto stage = [&](int spl) {
    if (threadIdx.x >= 32) return;
    const int t0 = spl * DEC_CHUNK, n = min(len, t0 + DEC_CHUNK) - t0;
    const int own = (kcw && spl == pos / DEC_CHUNK) ? pos - t0 : -1;
    const unsigned bytes = (unsigned)((n - (own >= 0 ? 1 : 0)) * hd * 4);
    if (lane0 == 0) {
      mbar_expect_tx(&kvbar[0], bytes);
      mbar_expect_tx(&kvbar[1], bytes);
    }
    __syncwarp();
    for (int t = lane0; t < n; t += 32)
      if (t != own) {
        const long long src = (lbase + t0 + t) * kvd + kvh * hd;
        bulk_g2s(kst + t * ks, kc + src, (unsigned)(hd * 4), &kvbar[0]);
        bulk_g2s(vst + t * ks, vc + src, (unsigned)(hd * 4), &kvbar[1]);
      }
  };
  const bool early = kcw != nullptr;
  // (cos, sin) of the rotated pairs at the row's position.  With ATT_THREADS a
  // multiple of hd / 2 every pair a thread rotates (q heads and the own K row)
  // is pair threadIdx.x % (hd / 2): one load, issued before the staging copies
  // so it does not queue behind them.
  const int half = hd / 2;
  const float2* cs2 = reinterpret_cast<const float2*>(rope + (long long)pos * hd);
  const bool cs_one = ATT_THREADS % half == 0;
  float2 cs_mine = make_float2(1.f, 0.f);
  if (kcw && cs_one) cs_mine = cs2[threadIdx.x % half];
  if (early) stage(sp);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  const float inv_sqrt_hd = 1.0f / sqrtf((float)hd);
  const float* q = qkv + (long long)r * (qd + 2 * kvd) + kvh * G * hd;
  // The row's own K / V (this step's QKV output): rotated K and V go to the
  // cache and to the staged rows of the split that holds `pos`.
  auto own_row = [&](int own) {
    const float* kr = qkv + (long long)r * (qd + 2 * kvd) + qd + kvh * hd;
    const float* vr = kr + kvd;
    const long long slot = (lbase + pos) * kvd + kvh * hd;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
      const int i = 2 * p;
      const float2 t = cs_one ? cs_mine : cs2[p];
      const float c = t.x, sn = t.y;
      const float2 xk = *reinterpret_cast<const float2*>(kr + i);
      const float a = xk.x * c, b = xk.y * sn, pp = xk.x * sn, qq = xk.y * c;
      const float k0 = a - b, k1 = pp + qq;
      kcw[slot + i] = k0;
      kcw[slot + i + 1] = k1;
      kst[own * ks + i] = k0;
      kst[own * ks + i + 1] = k1;
    }
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
      const float v = vr[i];
      vcw[slot + i] = v;
      vst[own * ks + i] = v;
    }
  };
  if (kcw) {  // q with rope (math.zig:88-104) applied on the way into shared memory
    for (int p = threadIdx.x; p < G * half; p += blockDim.x) {
      const int h = p / half, i = 2 * (p % half);
      const float2 xq = *reinterpret_cast<const float2*>(q + h * hd + i);
      const float2 t = cs_one ? cs_mine : cs2[i / 2];
      const float c = t.x, sn = t.y;
      const float a = xq.x * c, b = xq.y * sn, pp = xq.x * sn, qq = xq.y * c;
      qs[h * hd + i] = a - b;
      qs[h * hd + i + 1] = pp + qq;
    }
    if (sp == pos / DEC_CHUNK) own_row(pos - sp * DEC_CHUNK);  // its loads overlap the q loads
  } else {
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = q[i];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float hm[64], hl[64];
  unsigned kvphase = 0;
  for (bool first = true; sp < nsp; sp += gridDim.z, first = false, kvphase ^= 1u) {
    const int t0 = sp * DEC_CHUNK, t1 = min(len, t0 + DEC_CHUNK), n = t1 - t0;
    float* pr = part + (((long long)r * n_heads + kvh * G) * nsplit + sp) * (hd + 2);  // head stride nsplit*(hd+2)
    const int own = (kcw && sp == pos / DEC_CHUNK) ? pos - t0 : -1;  // staged row this CTA writes itself
    if (!(first && early)) stage(sp);
    if (own >= 0 && !first) own_row(own);  // (the first split's own row went in with q)
    VTB_TL_MARK(0);
    mbar_wait_bounded(&kvbar[0], kvphase);  // K staged (V may still be in flight)
    __syncthreads();
    VTB_TL_MARK(1);
    // scores: ATT_TPP threads per position, each over every ATT_TPP-th float4 column of the staged K row
    {
      const int tt = threadIdx.x / ATT_TPP, hf = threadIdx.x % ATT_TPP;
      const float4* kr = reinterpret_cast<const float4*>(kst + tt * ks);
      const float4* q4 = reinterpret_cast<const float4*>(qs);
      if constexpr (GT > 0) {
        float acc[GT];
#pragma unroll
        for (int h = 0; h < GT; ++h) acc[h] = 0.f;
        if (tt < n) {
#pragma unroll 4
          for (int j = hf; j < h4; j += ATT_TPP) {
            const float4 kv = kr[j];
#pragma unroll
            for (int h = 0; h < GT; ++h) {
              const float4 b = q4[h * h4 + j];
              acc[h] += kv.x * b.x + kv.y * b.y + kv.z * b.z + kv.w * b.w;
            }
          }
        }
#pragma unroll
        for (int o = 1; o < ATT_TPP; o <<= 1)
#pragma unroll
          for (int h = 0; h < GT; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
        if (tt < n && hf == 0)
#pragma unroll
          for (int h = 0; h < GT; ++h) sc[h * DEC_CHUNK + tt] = acc[h] * inv_sqrt_hd;
      } else {
        for (int h = 0; h < G; ++h) {
          float a = 0.f;
          if (tt < n)
            for (int j = hf; j < h4; j += ATT_TPP) {
              const float4 kv = kr[j], b = q4[h * h4 + j];
              a += kv.x * b.x + kv.y * b.y + kv.z * b.z + kv.w * b.w;
            }
          for (int o = 1; o < ATT_TPP; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
          if (tt < n && hf == 0) sc[h * DEC_CHUNK + tt] = a * inv_sqrt_hd;
        }
      }
    }
    __syncthreads();
    // per head: local max and exp-sum
    for (int h = warp; h < G; h += ATT_THREADS / 32) {
      float m = -INFINITY;
      for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h * DEC_CHUNK + i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float e = expf(sc[h * DEC_CHUNK + i] - m);
        sc[h * DEC_CHUNK + i] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        hm[h] = m;
        hl[h] = l;
      }
    }
    mbar_wait_bounded(&kvbar[1], kvphase);  // V staged
    __syncthreads();
    VTB_TL_MARK(2);
    // acc[h][d] = sum_t p[h][t] v[t][d]: thread (slice, d) reads staged v[t][d] once for every
    // head of the group; `slices` threads share a dimension, split the positions, add through smem.
    const int dd = threadIdx.x % hd, sl = threadIdx.x / hd;
    if constexpr (GT > 0) {
      float acc[GT];
#pragma unroll
      for (int h = 0; h < GT; ++h) acc[h] = 0.f;
      if (sl < slices && dd < hd) {
#pragma unroll 4
        for (int t = sl; t < n; t += slices) {
          const float v = vst[t * ks + dd];
#pragma unroll
          for (int h = 0; h < GT; ++h) acc[h] += sc[h * DEC_CHUNK + t] * v;
        }
      }
      __syncthreads();
      float* red = sc;  // reuse the score buffer: [slices][GT][hd]
      if (sl < slices && dd < hd)
#pragma unroll
        for (int h = 0; h < GT; ++h) red[(sl * GT + h) * hd + dd] = acc[h];
      __syncthreads();
      for (int i = threadIdx.x; i < GT * hd; i += blockDim.x) {
        const int h = i / hd, d = i % hd;
        float a = 0.f;
        for (int z = 0; z < slices; ++z) a += red[(z * GT + h) * hd + d];
        float* p = pr + (long long)h * nsplit * (hd + 2);
        p[2 + d] = a;
        if (d == 0) {
          p[0] = hm[h];
          p[1] = hl[h];
        }
      }
    } else {
      for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int h = i / hd, d = i % hd;
        const float* ph = sc + h * DEC_CHUNK;
        float a = 0.f;
        for (int t = 0; t < n; ++t) a += ph[t] * vst[t * ks + d];
        float* p = pr + (long long)h * nsplit * (hd + 2);
        p[2 + d] = a;
        if (d == 0) {
          p[0] = hm[h];
          p[1] = hl[h];
        }
      }
    }
    VTB_TL_MARK(3);
    // the next split reuses the staging and score buffers: the bulk copies (async
    // proxy) may overwrite what was just read only after every thread's reads
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  }
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < nw; ++w) v = is_max ? fmaxf(v, red[w]) : v + red[w];
  return v;
}

// Merge the live splits of each (row, q head):
// out = sum_s acc_s e^{m_s - M} / sum_s l_s e^{m_s - M}.  The split weights are
// computed once into shared memory; each dimension's sum then has independent loads.
__global__ void attn_combine_kernel(const float* __restrict__ part, float* __restrict__ att, RowInfo ri, int n_heads,
                                    int hd, int nsplit) {
  VTB_TL(13);
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ float wsm[];  // [nsplit]
  __shared__ float red[32];
  const int h = blockIdx.x, r = blockIdx.y;
  const int na = min(nsplit, ri.pos[r] / DEC_CHUNK + 1);  // positions are staged before the step
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  const float* p = part + ((long long)r * n_heads + h) * nsplit * (hd + 2);
  float M = -INFINITY;
  for (int s = threadIdx.x; s < na; s += blockDim.x) M = fmaxf(M, p[s * (hd + 2)]);
  M = block_reduce(M, true, red);
  VTB_TL_MARK(0);
  float L = 0.f;
  for (int s = threadIdx.x; s < na; s += blockDim.x) {
    const float e = expf(p[s * (hd + 2)] - M);
    wsm[s] = e;
    L += p[s * (hd + 2) + 1] * e;
  }
  L = block_reduce(L, false, red);  // its barriers also publish wsm
  VTB_TL_MARK(1);
  const float invL = 1.0f / L;
  // blockDim / hd groups of threads split the splits, so each thread's loads
  // are few and all in flight at once; the groups add up in order.
  float* gsum = wsm + nsplit;  // [groups][hd]
  const int groups = max(1, (int)blockDim.x / hd), g = threadIdx.x / hd, d = threadIdx.x % hd;
  if (g < groups) {
    float a = 0.f;
#pragma unroll 8
    for (int s = g; s < na; s += groups) a += p[s * (hd + 2) + 2 + d] * wsm[s];
    gsum[g * hd + d] = a;
  }
  __syncthreads();
  for (int dd = threadIdx.x; dd < hd; dd += blockDim.x) {
    float a = 0.f;
    for (int q = 0; q < groups; ++q) a += gsum[q * hd + dd];
    att[((long long)r * n_heads + h) * hd + dd] = a * invL;
  }
}

// Prefill attention: the rows are one prompt (one sequence, consecutive or
// arbitrary positions).  One CTA per (kv head, tile of 64 query vectors =
// 64/G rows x the G query heads of the kv head) walks the K/V chunks up to the
// tile's last position with an online softmax, so each staged K/V chunk serves
// 64 query vectors instead of one (the per-row kernel re-reads the whole
// prefix for every row).  fp32 throughout; the output goes straight to `att`.
constexpr int PA_QV = 64;       // query vectors per CTA
constexpr int PA_THREADS = 256; // 16 groups of 4 query vectors x 16 lanes
template <int HD>
struct PaSmem {
  static constexpr int QS = HD + 4, KS = HD + 4, PS = PA_QV + 4;  // padded row strides (floats)
  static constexpr int FLOATS = PA_QV * QS + 2 * ATT_CHUNK * KS + ATT_CHUNK * PS + PA_QV;
};

template <int HD>
__global__ void __launch_bounds__(PA_THREADS)
attn_prefill_kernel(const float* __restrict__ qkv, const float* __restrict__ kc, const float* __restrict__ vc,
                    RowInfo ri, int rows, int layer, int n_layers, int max_seq, int n_heads, int n_kv,
                    float* __restrict__ att) {
  VTB_TL(14);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  using P = PaSmem<HD>;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                          // [64 qvec][QS]
  float* kst = qs + PA_QV * P::QS;         // [CHUNK][KS]
  float* vst = kst + ATT_CHUNK * P::KS;    // [CHUNK][KS]
  float* ps = vst + ATT_CHUNK * P::KS;     // [CHUNK][PS]: probabilities, position-major
  int* qpos = reinterpret_cast<int*>(ps + ATT_CHUNK * P::PS);  // [64] position of each query vector's row
  const int G = n_heads / n_kv, QT = PA_QV / G;
  const int kvh = blockIdx.x, row0 = blockIdx.y * QT;
  const int qd = n_heads * HD, kvd = n_kv * HD;
  const int seq = ri.seq[row0];
  const long long lbase = ((long long)seq * n_layers + layer) * max_seq;
  const float inv_sqrt_hd = 1.0f / sqrtf((float)HD);
  // q tile: vector v = (row v / G, head v % G); rows past the end get position 0 (never written)
  for (int i = threadIdx.x; i < PA_QV * (HD / 4); i += PA_THREADS) {
    const int v = i / (HD / 4), c4 = 4 * (i % (HD / 4)), rr = row0 + v / G;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rr < rows) a = *reinterpret_cast<const float4*>(qkv + (long long)rr * (qd + 2 * kvd) + (kvh * G + v % G) * HD + c4);
    *reinterpret_cast<float4*>(qs + v * P::QS + c4) = a;
  }
  int maxpos = 0;
  for (int v = threadIdx.x; v < PA_QV; v += PA_THREADS) {
    const int rr = row0 + v / G;
    qpos[v] = rr < rows ? ri.pos[rr] : 0;
  }
  __syncthreads();
  for (int v = 0; v < PA_QV; v += G) maxpos = max(maxpos, qpos[v]);
  const int nch = maxpos / ATT_CHUNK + 1;
  const int qg = threadIdx.x >> 4, pg = threadIdx.x & 15;  // query vectors 4qg..4qg+3; positions pg + 16j
  int mypos[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) mypos[i] = qpos[4 * qg + i];
  float mrun[4], lrun[4];
  constexpr int DPT = HD / 16;  // output dims per thread: dg*4 .. +4 (and +64 for HD = 128)
  float o[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mrun[i] = -INFINITY;
    lrun[i] = 0.f;
#pragma unroll
    for (int d = 0; d < DPT; ++d) o[i][d] = 0.f;
  }
  for (int ch = 0; ch < nch; ++ch) {
    const int t0 = ch * ATT_CHUNK, n = min(ATT_CHUNK, maxpos + 1 - t0);
    for (int i = threadIdx.x; i < n * (HD / 4); i += PA_THREADS) {
      const int t = i / (HD / 4), c4 = 4 * (i % (HD / 4));
      const long long src = (lbase + t0 + t) * kvd + kvh * HD + c4;
      cp_async16(kst + t * P::KS + c4, kc + src);
      cp_async16(vst + t * P::KS + c4, vc + src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // scores s[i][j] = q[4qg+i] . k[pg+16j] / sqrt(hd), causal per query row
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d4 = 0; d4 < HD / 4; ++d4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qs + (4 * qg + i) * P::QS + 4 * d4);
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(kst + (pg + 16 * j) * P::KS + 4 * d4);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          s[i][j] += qv[i].x * kv[j].x + qv[i].y * kv[j].y + qv[i].z * kv[j].z + qv[i].w * kv[j].w;
    }
    float alpha[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mc = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = t0 + pg + 16 * j;
        s[i][j] = (pg + 16 * j < n && t <= mypos[i]) ? s[i][j] * inv_sqrt_hd : -INFINITY;
        mc = fmaxf(mc, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
      const float mnew = fmaxf(mrun[i], mc);  // finite: chunk 0 holds position 0 for every row
      alpha[i] = expf(mrun[i] - mnew);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - mnew);
        ps[(pg + 16 * j) * P::PS + 4 * qg + i] = p;
        ls += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      lrun[i] = lrun[i] * alpha[i] + ls;
      mrun[i] = mnew;
    }
    __syncthreads();
    // o[i][.] = o * alpha + sum_t p[t][4qg+i] v[t][.]
    const int dg = pg;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int d = 0; d < DPT; ++d) o[i][d] *= alpha[i];
    for (int t = 0; t < n; ++t) {
      const float4 p4 = *reinterpret_cast<const float4*>(ps + t * P::PS + 4 * qg);
      const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int h = 0; h < DPT / 4; ++h) {
        const float4 v4 = *reinterpret_cast<const float4*>(vst + t * P::KS + 64 * h + 4 * dg);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[i][4 * h] += pp[i] * v4.x;
          o[i][4 * h + 1] += pp[i] * v4.y;
          o[i][4 * h + 2] += pp[i] * v4.z;
          o[i][4 * h + 3] += pp[i] * v4.w;
        }
      }
    }
    __syncthreads();  // the next chunk overwrites K, V and P
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * qg + i, rr = row0 + v / G;
    if (rr >= rows) continue;
    const float inv = 1.0f / lrun[i];
    float* out = att + (long long)rr * qd + (kvh * G + v % G) * HD;
#pragma unroll
    for (int h = 0; h < DPT / 4; ++h)
      *reinterpret_cast<float4*>(out + 64 * h + 4 * pg) =
          make_float4(o[i][4 * h] * inv, o[i][4 * h + 1] * inv, o[i][4 * h + 2] * inv, o[i][4 * h + 3] * inv);
  }
}

// swiglu (math.zig:154-161): h = (g / (1 + e^-g)) * u.  gu per row is
// [gate | up], or with `il` the fused weights' [gate 8 | up 8] row blocks.
__global__ void swiglu_kernel(const float* __restrict__ gu, float* __restrict__ h, int ffn, int rows, int il) {
  VTB_TL(15);
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  VTB_TL_WAITED();
  const long long n = (long long)rows * ffn;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / ffn, j = i % ffn;
    const long long gi = il ? 16 * (j / 8) + j % 8 : j, ui = il ? gi + 8 : ffn + j;
    const float g = gu[r * 2 * ffn + gi], u = gu[r * 2 * ffn + ui];
    const float den = 1.0f + expf(-g);
    h[i] = (g / den) * u;
  }
}

// argmax (math.zig:190-201): first index of the maximum of each row.
// argmax (math.zig:190-201): first index of the maximum of each row (NaNs never
// win; an all-NaN row gives 0).  Two passes so a 128K-entry vocabulary row is
// scanned by ARGMAX_PARTS CTAs: each writes its slice's (max, first index),
// then one warp per row keeps the largest value with the smallest index.
constexpr int ARGMAX_PARTS = 64;

__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
}

__global__ void argmax_partial_kernel(const float* __restrict__ logits, float* __restrict__ pv, int* __restrict__ pi,
                                      int n) {
  VTB_TL(16);
  const int r = blockIdx.y, b = blockIdx.x;
  const int slice = (n + ARGMAX_PARTS - 1) / ARGMAX_PARTS, i0 = b * slice, i1 = min(n, i0 + slice);
  const float* l = logits + (long long)r * n;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = l[i];
    if (v > bv) { bv = v; bi = i; }  // ascending i per thread: the first maximum is kept
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) argmax_merge(bv, bi, sv[w], si[w]);
    pv[r * ARGMAX_PARTS + b] = bv;
    pi[r * ARGMAX_PARTS + b] = bi;
  }
}

__global__ void argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int32_t* __restrict__ out) {
  VTB_TL(17);
  const int r = blockIdx.x, lane = threadIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int b = lane; b < ARGMAX_PARTS; b += 32) argmax_merge(bv, bi, pv[r * ARGMAX_PARTS + b], pi[r * ARGMAX_PARTS + b]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  if (lane == 0) out[r] = bi == 0x7fffffff ? 0 : bi;
}

// Row-concatenate rows [r0, r1) of `n_parts` tensors (fuseRowConcat, model.zig:358-378).
}  // namespace vtb

using namespace vtb;

// ---------------- runtime ----------------

namespace {

struct DevLayer {
  const uint8_t* qkv;  // fused Q|K|V rows (all three share quant and k)
  const uint8_t* q; const uint8_t* k; const uint8_t* v;  // unfused fallback
  const uint8_t* o;
  const uint8_t* gu;   // fused gate|up rows: [gate 8 | up 8] row blocks when gu_il
  bool gu_il;
  const uint8_t* gate; const uint8_t* up;
  const uint8_t* down;
  long long down_pitch;  // bytes between ffn_down rows: Q6_K rows padded to 16 bytes for the tensor-core GEMV
  const float* attn_norm;
  const float* ffn_norm;
  int q_q, q_k, q_v, q_o, q_gate, q_up, q_down;
};

}  // namespace

struct VtbCudaModel {
  VtbCudaCtx* ctx;
  int device;
  VtbCudaLlamaConfig c;
  std::vector<DevLayer> layers;
  const uint8_t* embd;
  int q_embd;
  const float* out_norm;
  const uint8_t* out_w;
  int q_out;
  void* blob = nullptr;  // one allocation for every weight
  size_t blob_bytes = 0;
  // Tensor parallelism (tp.cu): this rank's shard; world 1 = the whole model.
  VtbCudaTp* tp = nullptr;
  VtbCudaTpShard sh;
  int H, KV, F, V;  // local q heads, kv heads, ffn rows, vocab rows
  // Q8_0 projections take Q8_0-quantized activations (vtb_cuda_model_set_q8_activations);
  // copied into each state at its creation.
  bool q8_act = false;
};

struct VtbCudaState {
  VtbCudaModel* m;
  int device;  // kept here so destroy never touches the model
  cudaStream_t st;
  int n_seqs, max_rows;
  float *x, *xb, *qkv, *att, *gu, *h, *logits, *part, *tmp;
  void* ws;  // GEMM activation workspace (bf16 hi + lo); the Q8_0 activation quants of the Q8_0 x Q8_0 path
  bool q8_act = false;  // the model's option when the state was created
  float* gsplit = nullptr;  // split-K partial tiles of small-batch GEMMs
  size_t gsplit_elems = 0;
  int32_t *tok, *seq, *pos, *amax;
  float *kc, *vc;
  float* rope;              // [max_seq][head_dim]: (cos, sin) of each rotated pair at each position
  int32_t* hbuf;            // pinned host staging: tok | seq | pos (3 * max_rows)
  int32_t* hamax;           // pinned host argmax
  std::vector<int64_t> seq_pos;  // host-authoritative positions (KvCache.pos, forward.zig:161,168)
  int rows = 0;             // rows of the step in flight
  int nsplit;
  float* logits_local;      // [rows][V] LM-head slice under tensor parallelism
  bool pending = false;     // tmp holds an all-reduced partial still to be added to x
  bool sig_pending = false; // peer memory: this rank's partial is complete but its flag not yet raised
  bool decode_rows = false; // staged rows are distinct sequences (decode), not one prompt (prefill)
  int max_pos = 0;          // largest staged position (sizes prefill attention grids)
  bool one_seq = false;     // every staged row belongs to one sequence
  cudaGraphExec_t graph = nullptr;
  int graph_rows = -1;
  // tensor parallel over peer memory (rmsnorm_tp_kernel); false: NCCL all-reduce of tmp
  bool p2p = false;
  PeerPtrs peers = {};
  int tp_rank = 0;
  long long flag_off = 0;   // floats from a block's start to its flags
  int par = 0;              // slot of the next all-reduce (host count mod 2; every call does an even number)
};

// Error text goes to the same thread-local buffer as the rest of the shim
// (vtb_cuda_last_error); the library is one translation unit.
static int merr(int st, const char* msg) { return set_err(st, "%s", msg); }
static int mcuda(cudaError_t e) {
  if (e == cudaErrorUnknown && strncmp(g_last_err, "NCCL", 4) == 0) return VTB_CUDA_ERR_COMM;
  return cuda_status(e);
}

static bool q_ok(int q) { return host_quant_ok(q); }

// Map every rank's shared block (IPC handles all-gathered over NCCL).  All
// ranks agree on the outcome (NCCL min of the per-rank result), so either
// every rank uses peer memory or every rank keeps the NCCL all-reduce.
// Returns false only on an error that leaves the state unusable.
static bool tp_p2p_setup(VtbCudaState* s) {
  VtbCudaTp* tp = s->m->tp;
  const int world = tp->world, me = tp->rank;
  const size_t slot = (size_t)s->max_rows * s->m->c.dim;
  s->flag_off = (long long)(2 * slot);
  float* blk = nullptr;
  if (cudaMalloc(&blk, (2 * slot + 2 * TP_MAX) * sizeof(float)) != cudaSuccess) {
    mcuda(cudaGetLastError());
    return false;
  }
  s->peers.p[me] = blk;
  s->tp_rank = me;
  uint8_t* dh = nullptr;  // [world][sizeof handle] + one int for the agreement
  cudaIpcMemHandle_t h;
  int ok = cudaMemsetAsync(blk, 0, (2 * slot + 2 * TP_MAX) * sizeof(float), s->st) == cudaSuccess &&
           cudaIpcGetMemHandle(&h, blk) == cudaSuccess;
  cudaGetLastError();
  if (cudaMalloc(&dh, (size_t)world * sizeof h + 4) != cudaSuccess) {
    mcuda(cudaGetLastError());
    return false;
  }
  std::vector<uint8_t> hh((size_t)world * sizeof h);
  bool fine = cudaMemcpyAsync(dh + (size_t)me * sizeof h, &h, sizeof h, cudaMemcpyHostToDevice, s->st) == cudaSuccess &&
              ncclAllGather(dh + (size_t)me * sizeof h, dh, sizeof h, ncclUint8, tp->comm, s->st) == ncclSuccess &&
              cudaMemcpyAsync(hh.data(), dh, hh.size(), cudaMemcpyDeviceToHost, s->st) == cudaSuccess &&
              cudaStreamSynchronize(s->st) == cudaSuccess;
  for (int r = 0; fine && ok && r < world; ++r) {
    if (r == me) continue;
    cudaIpcMemHandle_t hr;
    memcpy(&hr, hh.data() + (size_t)r * sizeof h, sizeof h);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
    } else {
      s->peers.p[r] = static_cast<float*>(p);
    }
  }
  int* dok = reinterpret_cast<int*>(dh + (size_t)world * sizeof h);
  fine = fine && cudaMemcpyAsync(dok, &ok, 4, cudaMemcpyHostToDevice, s->st) == cudaSuccess &&
         ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, tp->comm, s->st) == ncclSuccess &&
         cudaMemcpyAsync(&ok, dok, 4, cudaMemcpyDeviceToHost, s->st) == cudaSuccess &&
         cudaStreamSynchronize(s->st) == cudaSuccess;
  cudaFree(dh);
  if (!fine) {
    merr(VTB_CUDA_ERR_COMM, "tensor parallel: peer-memory setup failed");
    return false;
  }
  s->p2p = ok != 0;
  return true;
}

static void tp_p2p_release(VtbCudaState* s) {
  const int me = s->tp_rank;  // the model may already be gone
  for (int r = 0; r < TP_MAX; ++r)
    if (s->peers.p[r] && r != me) cudaIpcCloseMemHandle(s->peers.p[r]);
  cudaFree(s->peers.p[me]);
  s->peers = PeerPtrs{};
}

extern "C" {

VtbCudaModel* vtb_cuda_model_create_tp(VtbCudaCtx* ctx, VtbCudaTp* tp, const VtbCudaLlamaConfig* cfg,
                                       const VtbCudaLayerWeights* lw, const void* token_embd, int32_t q_token_embd,
                                       const float* output_norm, const void* output_w, int32_t q_output) {
  cudaGetLastError();
  if (!ctx || !cfg || !lw || !token_embd || !output_norm || !output_w) {
    merr(VTB_CUDA_ERR_INVALID_ARG, "null argument");
    return nullptr;
  }
  const VtbCudaLlamaConfig c = *cfg;
  if (c.dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
      c.head_dim % 8 || c.n_heads * c.head_dim != c.dim || c.ffn_dim <= 0 || c.vocab_size <= 0 || c.max_seq <= 0 ||
      c.n_heads / c.n_kv_heads > 64 || attn_smem_floats(c.n_heads / c.n_kv_heads, c.head_dim) * 4 > 227 * 1024) {
    merr(VTB_CUDA_ERR_INVALID_ARG, "inconsistent Llama config");
    return nullptr;
  }
  // Every projection must have a GPU kernel; no CPU fallback
  // (modelGpuEligible, forward.zig:372-396; BackendUnsupportedQuant, backend.zig:61).
  for (int l = 0; l < c.n_layers; ++l) {
    const int qs[7] = {lw[l].q_attn_q, lw[l].q_attn_k, lw[l].q_attn_v, lw[l].q_attn_o,
                       lw[l].q_ffn_gate, lw[l].q_ffn_up, lw[l].q_ffn_down};
    for (int q : qs)
      if (!q_ok(q)) {
        merr(VTB_CUDA_ERR_UNSUPPORTED, "projection quant type has no CUDA kernel");
        return nullptr;
      }
  }
  if (!q_ok(q_token_embd) || !q_ok(q_output)) {
    merr(VTB_CUDA_ERR_UNSUPPORTED, "embedding/output quant type has no CUDA kernel");
    return nullptr;
  }
  const int d = c.dim, f = c.ffn_dim, hd = c.head_dim;
  for (int l = 0; l < c.n_layers; ++l) {
    const int ks[7] = {d, d, d, d, d, d, f};
    const int qs[7] = {lw[l].q_attn_q, lw[l].q_attn_k, lw[l].q_attn_v, lw[l].q_attn_o,
                       lw[l].q_ffn_gate, lw[l].q_ffn_up, lw[l].q_ffn_down};
    for (int i = 0; i < 7; ++i)
      if (ks[i] % host_block_elems(qs[i])) {
        merr(VTB_CUDA_ERR_INVALID_ARG, "matrix width is not a whole number of blocks");
        return nullptr;
      }
  }
  const int rank = tp ? tp->rank : 0, world = tp ? tp->world : 1;
  VtbCudaTpShard sh;
  int kblock = 32;
  for (int l = 0; l < c.n_layers; ++l)
    kblock = std::max(kblock, std::max(host_block_elems(lw[l].q_attn_o), host_block_elems(lw[l].q_ffn_down)));
  if (vtb_cuda_tp_shard_plan(&c, rank, world, kblock, &sh) != VTB_CUDA_OK) return nullptr;
  VtbCudaModel* m = new (std::nothrow) VtbCudaModel();
  if (!m) return nullptr;
  m->ctx = ctx;
  m->c = c;
  m->tp = tp;
  m->sh = sh;
  m->H = sh.heads; m->KV = sh.kv_heads; m->F = sh.ffn_rows; m->V = sh.vocab_rows;
  cudaGetDevice(&m->device);
  const int qd = m->H * hd, kvd = m->KV * hd, F = m->F, V = m->V;
  // Layout pass: offsets of every (sharded) tensor in one blob, 256-byte aligned.
  auto rbytes = [](int q, int k) { return (size_t)host_row_bytes(q, k); };
  size_t off = 0;
  auto take = [&](size_t n) { size_t o = off; off = (off + n + 255) & ~size_t(255); return o; };
  // ffn_down rows (k = this rank's F): Q6_K rows that are not 16-byte multiples are
  // padded with zeros to a 16-byte pitch when they hold whole super-block pairs,
  // which the tensor-core GEMV and the GEMM's TMA staging need.
  auto down_pitch = [&](int q, int k) -> size_t {
    const size_t rb = rbytes(q, k);
    return (q == Q6_K && k % 512 == 0 && rb % 16) ? (rb + 15) & ~size_t(15) : rb;
  };
  struct Off { size_t qkv, q, k, v, o, gu, gate, up, down, an, fn; bool fq, fg; };
  std::vector<Off> offs(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    Off& o = offs[l];
    o.fq = lw[l].q_attn_q == lw[l].q_attn_k && lw[l].q_attn_q == lw[l].q_attn_v;
    o.fg = lw[l].q_ffn_gate == lw[l].q_ffn_up;
    if (o.fq) o.qkv = take(rbytes(lw[l].q_attn_q, d) * (qd + 2 * kvd));
    else { o.q = take(rbytes(lw[l].q_attn_q, d) * qd); o.k = take(rbytes(lw[l].q_attn_k, d) * kvd); o.v = take(rbytes(lw[l].q_attn_v, d) * kvd); }
    o.o = take(rbytes(lw[l].q_attn_o, qd) * d);
    if (o.fg) o.gu = take(rbytes(lw[l].q_ffn_gate, d) * 2 * F);
    else { o.gate = take(rbytes(lw[l].q_ffn_gate, d) * F); o.up = take(rbytes(lw[l].q_ffn_up, d) * F); }
    o.down = take(down_pitch(lw[l].q_ffn_down, F) * d);
    o.an = take(4 * (size_t)d);
    o.fn = take(4 * (size_t)d);
  }
  const size_t o_embd = take(rbytes(q_token_embd, d) * c.vocab_size);
  const size_t o_onorm = take(4 * (size_t)d);
  const size_t o_out = take(rbytes(q_output, d) * V);
  m->blob_bytes = off + 256;
  if (cudaMalloc(&m->blob, m->blob_bytes) != cudaSuccess) {
    cudaGetLastError();
    merr(VTB_CUDA_ERR_OOM, "weight upload: out of device memory");
    delete m;
    return nullptr;
  }
  uint8_t* B = static_cast<uint8_t*>(m->blob);
  cudaStream_t st = (cudaStream_t)vtb_cuda_stream(ctx);
  bool ok = true;
  auto up = [&](size_t o, const void* src, size_t n) {
    ok = ok && cudaMemcpyAsync(B + o, src, n, cudaMemcpyHostToDevice, st) == cudaSuccess;
  };
  // rows [row0, row0+nrows) x columns [col0, col0+ncols) of a [*, k] tensor -> dense at blob offset o
  auto up_shard = [&](size_t o, int q, const void* src, int k, int row0, int nrows, int col0, int ncols) {
    const size_t rb = rbytes(q, k), w = rbytes(q, ncols), c0 = rbytes(q, col0);
    const uint8_t* sp = static_cast<const uint8_t*>(src) + (size_t)row0 * rb + c0;
    if (w == rb) up(o, sp, rb * nrows);
    else ok = ok && cudaMemcpy2DAsync(B + o, w, sp, rb, w, nrows, cudaMemcpyHostToDevice, st) == cudaSuccess;
  };
  m->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    const Off& o = offs[l];
    DevLayer& L = m->layers[l];
    L.q_q = lw[l].q_attn_q; L.q_k = lw[l].q_attn_k; L.q_v = lw[l].q_attn_v; L.q_o = lw[l].q_attn_o;
    L.q_gate = lw[l].q_ffn_gate; L.q_up = lw[l].q_ffn_up; L.q_down = lw[l].q_ffn_down;
    const size_t rq = rbytes(L.q_q, d), rk = rbytes(L.q_k, d);
    if (o.fq) {
      L.qkv = B + o.qkv;
      up_shard(o.qkv, L.q_q, lw[l].attn_q, d, sh.q_row0, qd, 0, d);
      up_shard(o.qkv + rq * qd, L.q_k, lw[l].attn_k, d, sh.kv_row0, kvd, 0, d);
      up_shard(o.qkv + rq * qd + rk * kvd, L.q_v, lw[l].attn_v, d, sh.kv_row0, kvd, 0, d);
      L.q = L.k = L.v = nullptr;
    } else {
      L.qkv = nullptr;
      L.q = B + o.q; L.k = B + o.k; L.v = B + o.v;
      up_shard(o.q, L.q_q, lw[l].attn_q, d, sh.q_row0, qd, 0, d);
      up_shard(o.k, L.q_k, lw[l].attn_k, d, sh.kv_row0, kvd, 0, d);
      up_shard(o.v, L.q_v, lw[l].attn_v, d, sh.kv_row0, kvd, 0, d);
    }
    L.o = B + o.o;
    up_shard(o.o, L.q_o, lw[l].attn_o, d, 0, d, sh.o_col0, sh.o_cols);
    const size_t rg = rbytes(L.q_gate, d);
    L.gu_il = false;
    if (o.fg && F % 8 == 0) {
      // gate and up rows interleaved in blocks of 8 ([gate 8 | up 8], 16 rows): a
      // row tile of the decode GEMV then holds both inputs of SwiGLU for its outputs
      L.gu = B + o.gu;
      L.gu_il = true;
      const uint8_t* gs = static_cast<const uint8_t*>(lw[l].ffn_gate) + (size_t)sh.ffn_row0 * rg;
      const uint8_t* us = static_cast<const uint8_t*>(lw[l].ffn_up) + (size_t)sh.ffn_row0 * rg;
      ok = ok && cudaMemcpy2DAsync(B + o.gu, 16 * rg, gs, 8 * rg, 8 * rg, F / 8, cudaMemcpyHostToDevice, st) == cudaSuccess;
      ok = ok && cudaMemcpy2DAsync(B + o.gu + 8 * rg, 16 * rg, us, 8 * rg, 8 * rg, F / 8, cudaMemcpyHostToDevice, st) ==
                     cudaSuccess;
      L.gate = L.up = nullptr;
    } else if (o.fg) {
      L.gu = B + o.gu;
      up_shard(o.gu, L.q_gate, lw[l].ffn_gate, d, sh.ffn_row0, F, 0, d);
      up_shard(o.gu + rg * F, L.q_up, lw[l].ffn_up, d, sh.ffn_row0, F, 0, d);
      L.gate = L.up = nullptr;
    } else {
      L.gu = nullptr;
      L.gate = B + o.gate; L.up = B + o.up;
      up_shard(o.gate, L.q_gate, lw[l].ffn_gate, d, sh.ffn_row0, F, 0, d);
      up_shard(o.up, L.q_up, lw[l].ffn_up, d, sh.ffn_row0, F, 0, d);
    }
    L.down = B + o.down;
    L.down_pitch = (long long)down_pitch(L.q_down, F);
    if ((size_t)L.down_pitch == rbytes(L.q_down, F)) {
      up_shard(o.down, L.q_down, lw[l].ffn_down, f, 0, d, sh.down_col0, sh.down_cols);
    } else {  // padded rows: zero the padding, then copy each row's shard columns to its pitch
      const size_t rb = rbytes(L.q_down, f), w = rbytes(L.q_down, F), c0 = rbytes(L.q_down, sh.down_col0);
      ok = ok && cudaMemsetAsync(B + o.down, 0, (size_t)L.down_pitch * d, st) == cudaSuccess;
      ok = ok && cudaMemcpy2DAsync(B + o.down, (size_t)L.down_pitch, static_cast<const uint8_t*>(lw[l].ffn_down) + c0,
                                   rb, w, d, cudaMemcpyHostToDevice, st) == cudaSuccess;
    }
    L.attn_norm = reinterpret_cast<const float*>(B + o.an);
    L.ffn_norm = reinterpret_cast<const float*>(B + o.fn);
    up(o.an, lw[l].attn_norm, 4 * (size_t)d);
    up(o.fn, lw[l].ffn_norm, 4 * (size_t)d);
  }
  m->embd = B + o_embd; m->q_embd = q_token_embd;
  up(o_embd, token_embd, rbytes(q_token_embd, d) * c.vocab_size);
  m->out_norm = reinterpret_cast<const float*>(B + o_onorm);
  up(o_onorm, output_norm, 4 * (size_t)d);
  m->out_w = B + o_out; m->q_out = q_output;
  up_shard(o_out, q_output, output_w, d, sh.vocab_row0, V, 0, d);
  ok = ok && cudaStreamSynchronize(st) == cudaSuccess;
  if (!ok) {
    mcuda(cudaGetLastError());
    cudaFree(m->blob);
    delete m;
    return nullptr;
  }
  return m;
}

VtbCudaModel* vtb_cuda_model_create(VtbCudaCtx* ctx, const VtbCudaLlamaConfig* cfg, const VtbCudaLayerWeights* lw,
                                    const void* token_embd, int32_t q_token_embd, const float* output_norm,
                                    const void* output_w, int32_t q_output) {
  return vtb_cuda_model_create_tp(ctx, nullptr, cfg, lw, token_embd, q_token_embd, output_norm, output_w, q_output);
}

void vtb_cuda_model_destroy(VtbCudaModel* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  cudaFree(m->blob);
  delete m;
}

size_t vtb_cuda_model_weight_bytes(VtbCudaModel* m) { return m ? m->blob_bytes : 0; }

int vtb_cuda_model_set_q8_activations(VtbCudaModel* m, int on) {
  if (!m) return merr(VTB_CUDA_ERR_INVALID_ARG, "null model");
  m->q8_act = on != 0;
  return VTB_CUDA_OK;
}

VtbCudaState* vtb_cuda_state_create(VtbCudaModel* m, int32_t n_seqs, int32_t max_rows) {
  if (!m || n_seqs <= 0 || max_rows < n_seqs || max_rows > 65535) {
    merr(VTB_CUDA_ERR_INVALID_ARG, "bad state dimensions");
    return nullptr;
  }
  cudaSetDevice(m->device);
  const VtbCudaLlamaConfig& c = m->c;
  VtbCudaState* s = new (std::nothrow) VtbCudaState();
  if (!s) return nullptr;
  s->m = m;
  s->device = m->device;
  s->q8_act = m->q8_act;
  // The state owns its stream, so it never depends on the context outliving it.
  if (cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) {
    mcuda(cudaGetLastError());
    delete s;
    return nullptr;
  }
  s->n_seqs = n_seqs;
  s->max_rows = max_rows;
  {  // attention stages K/V in shared memory: opt every instantiation in to the size this model needs
    const int asmem = attn_smem_floats(c.n_heads / c.n_kv_heads, c.head_dim) * 4;
    cudaError_t ea = cudaFuncSetAttribute(attn_partial_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
    if (!ea) ea = cudaFuncSetAttribute(attn_partial_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
    if (!ea) ea = cudaFuncSetAttribute(attn_partial_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
    if (!ea) ea = cudaFuncSetAttribute(attn_partial_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
    if (!ea) ea = cudaFuncSetAttribute(attn_partial_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
    if (!ea)
      ea = cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                PaSmem<64>::FLOATS * 4);
    if (!ea)
      ea = cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                PaSmem<128>::FLOATS * 4);
    if (ea) {
      mcuda(ea);
      cudaStreamDestroy(s->st);
      delete s;
      return nullptr;
    }
  }
  s->nsplit = (c.max_seq + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t R = max_rows, d = c.dim, hd = c.head_dim, qd = (size_t)m->H * hd, kvd = (size_t)m->KV * hd, f = m->F;
  const size_t qkvw = qd + 2 * kvd;
  const size_t kmax = d > f ? d : f;
  // split-K partials for small-batch GEMMs: splits x rows <= 512 of the widest projection
  const size_t gsplit = R >= (size_t)GEMM_MIN_ROWS ? 512 * std::max(std::max(qkvw, 2 * f), d) : 0;
  size_t fl = R * (d + d + qkvw + qd + 2 * f + f + (size_t)c.vocab_size + m->V + d + kmax) +
              R * m->H * (size_t)s->nsplit * (hd + 2) + gsplit + (size_t)c.max_seq * hd + 64;
  const size_t kvn = (size_t)n_seqs * c.n_layers * c.max_seq * kvd;
  float* base = nullptr;
  int32_t* ib = nullptr;
  if (cudaMalloc(&base, (fl + 2 * kvn) * 4 + 64) != cudaSuccess || cudaMalloc(&ib, 4 * R * 4) != cudaSuccess ||
      cudaMallocHost(&s->hbuf, 3 * R * 4) != cudaSuccess || cudaMallocHost(&s->hamax, R * 4) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(base);
    cudaFree(ib);
    merr(VTB_CUDA_ERR_OOM, "state: out of memory (KV cache)");
    delete s;
    return nullptr;
  }
  float* p = base;
  auto carve = [&](size_t n) { float* r = p; p += (n + 3) & ~size_t(3); return r; };
  s->x = carve(R * d); s->xb = carve(R * d); s->qkv = carve(R * qkvw); s->att = carve(R * qd);
  s->gu = carve(R * 2 * f); s->h = carve(R * f); s->logits = carve(R * c.vocab_size);
  s->logits_local = carve(R * m->V);
  s->part = carve(R * m->H * (size_t)s->nsplit * (hd + 2));
  s->tmp = carve(R * d);
  s->ws = carve(R * kmax);  // bf16 hi + lo = 4 bytes per activation
  s->gsplit = gsplit ? carve(gsplit) : nullptr;
  s->gsplit_elems = gsplit;
  s->kc = carve(kvn); s->vc = carve(kvn);
  s->rope = carve((size_t)c.max_seq * hd);
  s->tok = ib; s->seq = ib + R; s->pos = ib + 2 * R; s->amax = ib + 3 * R;
  cudaMemsetAsync(s->kc, 0, 2 * kvn * 4, s->st);
  // RoPE angles with the reference's float steps (math.zig:88-104): inv_freq =
  // 1 / pow(base, i / hd), theta = pos * inv_freq, cos / sin, computed once on
  // the host with the C library's float functions.
  std::vector<float> rope_h((size_t)c.max_seq * hd);
  for (int pos = 0; pos < c.max_seq; ++pos)
    for (size_t i = 0; i < hd; i += 2) {
      const float inv_freq = 1.0f / powf(c.rope_base, (float)i / (float)hd);
      const float theta = (float)pos * inv_freq;
      rope_h[(size_t)pos * hd + i] = cosf(theta);
      rope_h[(size_t)pos * hd + i + 1] = sinf(theta);
    }
  cudaMemcpyAsync(s->rope, rope_h.data(), rope_h.size() * 4, cudaMemcpyHostToDevice, s->st);
  s->seq_pos.assign(n_seqs, 0);
  if (m->tp && m->tp->world > 1 && m->tp->world <= TP_MAX && !tp_p2p_setup(s)) {
    vtb_cuda_state_destroy(s);
    return nullptr;
  }
  if (cudaStreamSynchronize(s->st) != cudaSuccess) {
    mcuda(cudaGetLastError());
    return nullptr;
  }
  return s;
}

void vtb_cuda_state_destroy(VtbCudaState* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  cudaStreamSynchronize(s->st);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  tp_p2p_release(s);
  cudaStreamDestroy(s->st);
  cudaFree(s->x);
  cudaFree(s->tok);
  cudaFreeHost(s->hbuf);
  cudaFreeHost(s->hamax);
  delete s;
}

int vtb_cuda_state_reset(VtbCudaState* s) {
  if (!s) return merr(VTB_CUDA_ERR_INVALID_ARG, "null state");
  for (auto& p : s->seq_pos) p = 0;
  return VTB_CUDA_OK;
}

int vtb_cuda_state_tp_p2p(const VtbCudaState* s) { return s && s->p2p ? 1 : 0; }

int64_t vtb_cuda_state_pos(VtbCudaState* s, int32_t seq) {
  if (!s || seq < 0 || seq >= s->n_seqs) return -1;
  return s->seq_pos[seq];
}

}  // extern "C"

// Stage the rows of a step (token, sequence, position) and embed them
// (gatherEmbedding, forward.zig:163).  Checks mirror stepWithBackend's
// (forward.zig:159-160) and prefillCpu's (prefill.zig:123-127).
static int stage_rows(VtbCudaState* s, int rows, const int32_t* tok, const int32_t* seq, const int32_t* pos) {
  const VtbCudaLlamaConfig& c = s->m->c;
  if (rows <= 0 || rows > s->max_rows) return merr(VTB_CUDA_ERR_INVALID_ARG, "too many rows for this state");
  for (int r = 0; r < rows; ++r) {
    if (tok[r] < 0 || tok[r] >= c.vocab_size) return merr(VTB_CUDA_ERR_INVALID_ARG, "token id out of range");
    if (pos[r] >= c.max_seq) return merr(VTB_CUDA_ERR_STREAM_ABORTED, "KV cache full");
    s->hbuf[r] = tok[r];
    s->hbuf[s->max_rows + r] = seq[r];
    s->hbuf[2 * s->max_rows + r] = pos[r];
  }
  s->rows = rows;
  s->pending = false;
  s->sig_pending = false;
  s->max_pos = 0;
  for (int r = 0; r < rows; ++r) s->max_pos = std::max(s->max_pos, (int)pos[r]);
  s->one_seq = true;
  for (int r = 1; r < rows; ++r) s->one_seq = s->one_seq && seq[r] == seq[0];
  s->decode_rows = true;
  for (int r = 1; r < rows && s->decode_rows; ++r)
    for (int q = 0; q < r; ++q)
      if (seq[q] == seq[r]) { s->decode_rows = false; break; }
  return VTB_CUDA_OK;
}

static cudaError_t enqueue_embed(VtbCudaState* s) {
  const int R = s->max_rows;
  cudaError_t e = cudaMemcpyAsync(s->tok, s->hbuf, 3 * R * 4, cudaMemcpyHostToDevice, s->st);
  if (e != cudaSuccess) return e;
  return launch_embed(s->m->q_embd, s->m->embd, s->tok, s->x, s->m->c.dim, s->rows, s->st);
}

// Every kernel of the forward loop releases its dependent at its first
// instruction: the dependent's own griddepcontrol.wait still orders it after
// this grid completes, so the early release only lets the next GEMV's CTAs
// start their weight prefetch while this kernel runs.
template <typename K, typename... A>
static cudaError_t pdl_launch(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// RMSNorm of the staged rows; under tensor parallelism the all-reduced partial
// waiting in tmp is added to x first (addInto fused into the norm).
static cudaError_t enqueue_norm(VtbCudaState* s, const float* w, int r0, int n) {
  const VtbCudaLlamaConfig& c = s->m->c;
  if (s->pending && s->p2p) {  // the all-reduce itself happens here, over peer memory
    s->pending = false;
    // One row (batch-1 decode, the last prefill row): the single CTA raises this
    // rank's flag itself.  Several rows: a one-thread kernel raises it first.
    const int sig = s->sig_pending && n == 1;
    if (s->sig_pending && !sig) {
      cudaError_t e = pdl_launch(tp_signal_kernel, dim3(1), dim3(32), 0, s->st, s->peers, s->m->tp->world,
                                 s->m->tp->rank, s->flag_off);
      if (e) return e;
    }
    s->sig_pending = false;
    const long long slot_off = (long long)(s->par ^ 1) * s->max_rows * c.dim + (long long)r0 * c.dim;
    return pdl_launch(rmsnorm_tp_kernel, dim3(n), dim3(1024), 0, s->st, s->x + (size_t)r0 * c.dim, s->peers,
                      s->m->tp->world, s->m->tp->rank, slot_off, s->flag_off, w, s->xb, c.dim, c.rms_eps, sig);
  }
  const float* res = s->pending ? s->tmp + (size_t)r0 * c.dim : nullptr;
  s->pending = false;
  return pdl_launch(rmsnorm_kernel, dim3(n), dim3(256), 0, s->st, s->x + (size_t)r0 * c.dim, res, w, s->xb, c.dim,
                    c.rms_eps);
}

// Destination of this rank's partial of the next all-reduce.
static float* partial_out(VtbCudaState* s) {
  return s->p2p ? s->peers.p[s->m->tp->rank] + (size_t)s->par * s->max_rows * s->m->c.dim : s->tmp;
}

static cudaError_t allreduce_tmp(VtbCudaState* s, size_t n) {
  if (s->p2p) {  // the partial is published (flag raised) and summed by the next RMSNorm
    s->par ^= 1;
    s->pending = true;
    s->sig_pending = true;
    return cudaSuccess;
  }
  const ncclResult_t r = ncclAllReduce(s->tmp, s->tmp, n, ncclFloat32, ncclSum, s->m->tp->comm, s->st);
  if (r != ncclSuccess) {
    nccl_status(r);
    return cudaErrorUnknown;
  }
  s->pending = true;
  return cudaSuccess;
}

// One row of a projection: y (+)= W . x.  Under the Q8_0 x Q8_0 option a Q8_0
// weight takes x quantized per 32-block into the state's workspace (the
// quantizer, then int32 block dots; dot_i8, simd.zig:31-62).
static cudaError_t gemv_row(VtbCudaState* s, int q, const void* w, const float* x, float* y, int m, int k, int acc,
                            long long pitch = 0) {
  if (s->q8_act && q == Q8_0) {
    int8_t* xq = static_cast<int8_t*>(s->ws);
    float* dx = reinterpret_cast<float*>(static_cast<char*>(s->ws) + (((size_t)k + 15) & ~size_t(15)));
    return launch_gemv_q8_0_q8_0_x(w, x, xq, dx, y, m, k, s->st, true, acc);
  }
  return gemv_any(q, w, x, y, m, k, s->st, acc, pitch);
}

// One transformer block for the staged rows (cpuLayerStep, forward.zig:230-288).
static cudaError_t enqueue_layer(VtbCudaState* s, int l) {
  VtbCudaModel* m = s->m;
  const VtbCudaLlamaConfig& c = m->c;
  const DevLayer& L = m->layers[l];
  const int hd = c.head_dim, H = m->H, KV = m->KV, G = H / KV;
  const int R = s->rows, d = c.dim, qd = H * hd, kvd = KV * hd, f = m->F, qkvw = qd + 2 * kvd;
  const bool tp = m->tp && m->tp->world > 1;
  cudaStream_t st = s->st;
  cudaError_t e;
  RowInfo ri{s->seq, s->pos};
  const bool gemm = R >= GEMM_MIN_ROWS;
  // RMSNorm fused into a Q4_K GEMV's activation prologue when nothing is pending in tmp.
  auto fused_norm_gemv = [&](const float* nw, int q, const uint8_t* w, float* out, int mm) -> bool {
    if (gemm || s->pending || q != Q4_K || !w) return false;
    for (int r = 0; r < R && e == cudaSuccess; ++r)
      e = launch_gemv_q4k_mma(w, s->x + (size_t)r * d, out + (size_t)r * mm, mm, d, st, true, 0, nw, c.rms_eps,
                              nullptr);
    return true;
  };
  auto proj = [&](int q, const uint8_t* w, const float* in, float* out, int mm, int k, int ld_out, int acc,
                  long long pitch = 0) -> cudaError_t {
    // out[r*ld_out + i] (+)= W . in[r]; GEMM rows need a dense out, so `acc` goes through tmp
    if (gemm && k % 64 == 0 && (acc || ld_out == mm) && !(s->q8_act && q == Q8_0)) {
      if (acc) {
        cudaError_t e2 = launch_gemm_tc(q, w, in, s->tmp, mm, k, R, true, s->ws, st, s->gsplit, s->gsplit_elems, pitch);
        if (e2) return e2;
        return pdl_launch(add_kernel, dim3(min(1184, (R * mm + 255) / 256)), dim3(256), 0, st, out,
                          (const float*)s->tmp, (long long)R * mm);
      }
      return launch_gemm_tc(q, w, in, out, mm, k, R, true, s->ws, st, s->gsplit, s->gsplit_elems, pitch);
    }
    for (int r = 0; r < R; ++r) {
      cudaError_t e2 = gemv_row(s, q, w, in + (size_t)r * k, out + (size_t)r * ld_out, mm, k, acc, pitch);
      if (e2) return e2;
    }
    return cudaSuccess;
  };
  // x += W . in for the row-parallel projections (O, down): single GPU adds
  // straight into x; tensor parallel writes the partial to tmp and all-reduces.
  auto residual = [&](int q, const uint8_t* w, const float* in, int k, long long pitch) -> cudaError_t {
    if (!tp) return proj(q, w, in, s->x, d, k, d, 1, pitch);
    cudaError_t e2 = proj(q, w, in, partial_out(s), d, k, d, 0, pitch);
    if (e2) return e2;
    return allreduce_tmp(s, (size_t)R * d);
  };
  e = cudaSuccess;
  if (fused_norm_gemv(L.attn_norm, L.q_q, L.qkv, s->qkv, qkvw)) {
    if (e) return e;
  } else if ((e = enqueue_norm(s, L.attn_norm, 0, R))) {
    return e;
  } else if (L.qkv) {
    if ((e = proj(L.q_q, L.qkv, s->xb, s->qkv, qkvw, d, qkvw, 0))) return e;
  } else {
    if ((e = proj(L.q_q, L.q, s->xb, s->qkv, qd, d, qkvw, 0))) return e;
    if ((e = proj(L.q_k, L.k, s->xb, s->qkv + qd, kvd, d, qkvw, 0))) return e;
    if ((e = proj(L.q_v, L.v, s->xb, s->qkv + qd + kvd, kvd, d, qkvw, 0))) return e;
  }
  // Decode rows are distinct sequences: each row's new K/V is read only by its
  // own attention, so RoPE + the cache write fold into the attention kernel.
  // Prefill rows of one sequence read each other's K/V: separate kernel first.
  const bool fuse_rope = s->decode_rows;
  if (!fuse_rope && (e = pdl_launch(rope_kv_kernel, dim3(R), dim3(256), 0, st, s->qkv, s->kc, s->vc, ri, l, c.n_layers,
                                    c.max_seq, H, KV, hd, (const float*)s->rope)))
    return e;
  float* kcw = fuse_rope ? s->kc : nullptr;
  float* vcw = fuse_rope ? s->vc : nullptr;
  if (!fuse_rope && s->one_seq && (hd == 64 || hd == 128) && PA_QV % G == 0) {
    // prompt rows: query-tiled attention, no split/combine pass
    const dim3 pgrid(KV, (R + PA_QV / G - 1) / (PA_QV / G));
    e = hd == 64 ? pdl_launch(attn_prefill_kernel<64>, pgrid, dim3(PA_THREADS), (size_t)PaSmem<64>::FLOATS * 4, st,
                              (const float*)s->qkv, (const float*)s->kc, (const float*)s->vc, ri, R, l, c.n_layers,
                              c.max_seq, H, KV, s->att)
                 : pdl_launch(attn_prefill_kernel<128>, pgrid, dim3(PA_THREADS), (size_t)PaSmem<128>::FLOATS * 4, st,
                              (const float*)s->qkv, (const float*)s->kc, (const float*)s->vc, ri, R, l, c.n_layers,
                              c.max_seq, H, KV, s->att);
    if (e) return e;
  } else {
    const size_t asmem = (size_t)attn_smem_floats(G, hd) * 4;
    // Decode (replayed as a graph while positions grow): about one wave of CTAs
    // (3 resident per SM at these sizes), each walking its row's live splits.
    // Prefill rows (enqueued directly): one CTA per live split of the longest row.
    const int zdec = std::max(1, 3 * 148 / (KV * R));
    const int z = s->decode_rows ? std::min(s->nsplit, zdec) : std::min(s->nsplit, s->max_pos / DEC_CHUNK + 1);
    const dim3 agrid(KV, R, z);
    switch (hd <= ATT_THREADS && hd % 16 == 0 ? G : 0) {  // register path needs hd <= 128, hd % 16 == 0
  #define VTB_ATT(g)                                                                                               \
    case g:                                                                                                      \
      e = pdl_launch(attn_partial_kernel<g>, agrid, dim3(ATT_THREADS), asmem, st, (const float*)s->qkv,             \
                     (const float*)s->kc, (const float*)s->vc, ri, l, c.n_layers, c.max_seq, H, KV, hd, s->part,     \
                     s->nsplit, kcw, vcw, (const float*)s->rope);                                                          \
      break;
      VTB_ATT(1) VTB_ATT(2) VTB_ATT(4) VTB_ATT(8)
  #undef VTB_ATT
      default:
        e = pdl_launch(attn_partial_kernel<0>, agrid, dim3(ATT_THREADS), asmem, st, (const float*)s->qkv,
                       (const float*)s->kc, (const float*)s->vc, ri, l, c.n_layers, c.max_seq, H, KV, hd, s->part,
                       s->nsplit, kcw, vcw, (const float*)s->rope);
    }
    if (e) return e;
    // 256 threads: the split weights, then blockDim / hd groups of partial sums
    if ((e = pdl_launch(attn_combine_kernel, dim3(H, R), dim3(256), (size_t)(s->nsplit + 256 + hd) * 4, st,
                        (const float*)s->part,
                        s->att, ri, H, hd, s->nsplit)))
      return e;
  }
  if ((e = residual(L.q_o, L.o, s->att, qd, 0))) return e;  // x += W_o . att (addInto fused)
  if (!gemm && L.gu && L.gu_il && L.q_gate == Q4_K) {
    // SwiGLU in the GEMV's epilogue (h directly); the FFN RMSNorm in its prologue,
    // or, with a tensor-parallel partial pending, in the all-reduce kernel before it
    const bool pend = s->pending;
    if (pend && (e = enqueue_norm(s, L.ffn_norm, 0, R))) return e;
    for (int r = 0; r < R && e == cudaSuccess; ++r)
      e = launch_gemv_q4k_mma(L.gu, (pend ? s->xb : s->x) + (size_t)r * d, nullptr, 2 * f, d, st, true, 0,
                              pend ? nullptr : L.ffn_norm, c.rms_eps, s->h + (size_t)r * f);
    if (e) return e;
    return residual(L.q_down, L.down, s->h, f, L.down_pitch);
  }
  if (fused_norm_gemv(L.ffn_norm, L.q_gate, L.gu, s->gu, 2 * f)) {
    if (e) return e;
  } else if ((e = enqueue_norm(s, L.ffn_norm, 0, R))) {
    return e;
  } else if (L.gu) {
    if ((e = proj(L.q_gate, L.gu, s->xb, s->gu, 2 * f, d, 2 * f, 0))) return e;
  } else {
    if ((e = proj(L.q_gate, L.gate, s->xb, s->gu, f, d, 2 * f, 0))) return e;
    if ((e = proj(L.q_up, L.up, s->xb, s->gu + f, f, d, 2 * f, 0))) return e;
  }
  if ((e = pdl_launch(swiglu_kernel, dim3(min(1184, (R * f + 255) / 256)), dim3(256), 0, st, (const float*)s->gu, s->h,
                      f, R, L.gu && L.gu_il ? 1 : 0)))
    return e;
  return residual(L.q_down, L.down, s->h, f, L.down_pitch);
}

// Final RMSNorm + LM head (backend_cpu.zig finalStep :88-106) and argmax.
// `last_only`: prefill computes logits for its last row only (prefill.zig:141-146).
static cudaError_t enqueue_final(VtbCudaState* s, bool last_only) {
  VtbCudaModel* m = s->m;
  const VtbCudaLlamaConfig& c = m->c;
  cudaStream_t st = s->st;
  cudaError_t e;
  const bool tp = m->tp && m->tp->world > 1;
  const int r0 = last_only ? s->rows - 1 : 0, n = last_only ? 1 : s->rows;
  if ((e = enqueue_norm(s, m->out_norm, r0, n))) return e;
  float* lg = tp ? s->logits_local : s->logits;
  if (n >= GEMM_MIN_ROWS && c.dim % 64 == 0 && !(s->q8_act && m->q_out == Q8_0)) {
    // batch decode: one GEMM reads the LM head once for all rows
    if ((e = launch_gemm_tc(m->q_out, m->out_w, s->xb, lg, m->V, c.dim, n, true, s->ws, st, s->gsplit, s->gsplit_elems))) return e;
  } else {
    for (int r = 0; r < n; ++r)
      if ((e = gemv_row(s, m->q_out, m->out_w, s->xb + (size_t)r * c.dim, lg + (size_t)r * m->V, m->V, c.dim, 0)))
        return e;
  }
  if (tp) {  // all-gather the vocabulary slices, one row at a time (rank slices are contiguous vocab ranges)
    ncclResult_t rr = ncclGroupStart();
    for (int r = 0; r < n && rr == ncclSuccess; ++r)
      rr = ncclAllGather(s->logits_local + (size_t)r * m->V, s->logits + (size_t)r * c.vocab_size, m->V, ncclFloat32,
                         m->tp->comm, st);
    if (rr == ncclSuccess) rr = ncclGroupEnd();
    if (rr != ncclSuccess) {
      nccl_status(rr);
      return cudaErrorUnknown;
    }
  }
  // the attention partials are dead after the last layer: reuse them for the argmax slices
  float* apv = s->part;
  int* api = reinterpret_cast<int*>(s->part + (size_t)n * ARGMAX_PARTS);
  argmax_partial_kernel<<<dim3(ARGMAX_PARTS, n), 256, 0, st>>>(s->logits, apv, api, c.vocab_size);
  argmax_final_kernel<<<n, 32, 0, st>>>(apv, api, s->amax);
  return cudaGetLastError();
}

static int finalize(VtbCudaState* s, int n, float* logits, int32_t* argmax) {
  const VtbCudaLlamaConfig& c = s->m->c;
  cudaError_t e = cudaSuccess;
  if (argmax) e = cudaMemcpyAsync(s->hamax, s->amax, n * 4, cudaMemcpyDeviceToHost, s->st);
  if (e == cudaSuccess && logits)
    e = cudaMemcpyAsync(logits, s->logits, (size_t)n * c.vocab_size * 4, cudaMemcpyDeviceToHost, s->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
  if (e != cudaSuccess) return mcuda(e);
  if (argmax) memcpy(argmax, s->hamax, n * 4);
  return VTB_CUDA_OK;
}

extern "C" {

// ---- the backend vtable, one call per slot (backend.zig:67-97) ----

int vtb_cuda_begin_token(VtbCudaState* s, const int32_t* tokens) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || !tokens) return merr(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  cudaSetDevice(s->m->device);
  std::vector<int32_t> seq(s->n_seqs), pos(s->n_seqs);
  for (int i = 0; i < s->n_seqs; ++i) { seq[i] = i; pos[i] = (int32_t)s->seq_pos[i]; }
  int rc = stage_rows(s, s->n_seqs, tokens, seq.data(), pos.data());
  if (rc) return rc;
  return mcuda(enqueue_embed(s));
}

int vtb_cuda_layer_step(VtbCudaState* s, int32_t layer) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || layer < 0 || layer >= s->m->c.n_layers || s->rows <= 0)
    return merr(VTB_CUDA_ERR_INVALID_ARG, "bad layer step");
  return mcuda(enqueue_layer(s, layer));
}

int vtb_cuda_final_step(VtbCudaState* s) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || s->rows <= 0) return merr(VTB_CUDA_ERR_INVALID_ARG, "no token staged");
  return mcuda(enqueue_final(s, false));
}

int vtb_cuda_finalize_token(VtbCudaState* s, float* logits, int32_t* argmax) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || s->rows <= 0) return merr(VTB_CUDA_ERR_INVALID_ARG, "no token staged");
  const int n = s->rows;
  int rc = finalize(s, n, logits, argmax);
  if (rc == VTB_CUDA_OK)  // cache.advance (forward.zig:168)
    for (int i = 0; i < s->n_seqs; ++i) s->seq_pos[i] += 1;
  s->rows = 0;
  return rc;
}

// Whole decode step (stepWithBackend, forward.zig:152-172) as one CUDA graph
// per state: the graph reads tokens and positions from pinned host staging,
// so it is captured once and replayed every token.
int vtb_cuda_step(VtbCudaState* s, const int32_t* tokens, float* logits, int32_t* argmax) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || !tokens) return merr(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  cudaSetDevice(s->m->device);
  std::vector<int32_t> seq(s->n_seqs), pos(s->n_seqs);
  for (int i = 0; i < s->n_seqs; ++i) { seq[i] = i; pos[i] = (int32_t)s->seq_pos[i]; }
  int rc = stage_rows(s, s->n_seqs, tokens, seq.data(), pos.data());
  if (rc) return rc;
  if (!s->graph || s->graph_rows != s->rows) {
    if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; }
    // Warm the kernels' one-time attribute setup outside of capture.
    cudaError_t e = enqueue_embed(s);
    for (int l = 0; l < s->m->c.n_layers && e == cudaSuccess; ++l) e = enqueue_layer(s, l);
    if (e == cudaSuccess) e = enqueue_final(s, false);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
    // The warm-up wrote this token's K/V; the replay below rewrites the same slots.
    cudaGraph_t g;
    if (e == cudaSuccess) e = cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      cudaError_t ee = enqueue_embed(s);
      for (int l = 0; l < s->m->c.n_layers && ee == cudaSuccess; ++l) ee = enqueue_layer(s, l);
      if (ee == cudaSuccess) ee = enqueue_final(s, false);
      e = cudaStreamEndCapture(s->st, &g);
      if (ee != cudaSuccess) e = ee;
    }
    if (e == cudaSuccess) {
      e = cudaGraphInstantiate(&s->graph, g, 0);
      cudaGraphDestroy(g);
    }
    if (e != cudaSuccess) return mcuda(e);
    s->graph_rows = s->rows;
  }
  cudaError_t e = cudaGraphLaunch(s->graph, s->st);
  if (e != cudaSuccess) return mcuda(e);
  return vtb_cuda_finalize_token(s, logits, argmax);
}

// Batched prompt prefill of sequence `seq` (prefillCpu, prefill.zig:111-147):
// all n tokens go through each layer together; logits of the last token.
int vtb_cuda_prefill(VtbCudaState* s, int32_t seq, const int32_t* tokens, int32_t n, float* logits, int32_t* argmax) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  if (!s || !tokens || seq < 0 || seq >= s->n_seqs) return merr(VTB_CUDA_ERR_INVALID_ARG, "bad prefill arguments");
  if (n == 0) return VTB_CUDA_OK;
  const VtbCudaLlamaConfig& c = s->m->c;
  if (s->seq_pos[seq] + n > c.max_seq) return merr(VTB_CUDA_ERR_STREAM_ABORTED, "KV cache full");
  cudaSetDevice(s->m->device);
  int done = 0;
  while (done < n) {  // chunks of max_rows tokens
    const int rows = min(n - done, s->max_rows);
    std::vector<int32_t> sq(rows, seq), pos(rows);
    for (int r = 0; r < rows; ++r) pos[r] = (int32_t)(s->seq_pos[seq] + r);
    int rc = stage_rows(s, rows, tokens + done, sq.data(), pos.data());
    if (rc) return rc;
    cudaError_t e = enqueue_embed(s);
    for (int l = 0; l < c.n_layers && e == cudaSuccess; ++l) e = enqueue_layer(s, l);
    const bool last = done + rows == n;
    if (e == cudaSuccess && last) e = enqueue_final(s, true);
    if (e != cudaSuccess) return mcuda(e);
    s->seq_pos[seq] += rows;
    done += rows;
    if (last) {
      s->rows = 1;
      rc = finalize(s, 1, logits, argmax);
      s->rows = 0;
      return rc;
    }
  }
  return VTB_CUDA_OK;
}

}  // extern "C"
