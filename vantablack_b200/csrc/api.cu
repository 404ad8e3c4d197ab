// api.cu -- the extern "C" shim (include/vtb_cuda.h): argument checks,
// status mapping, and the context/buffer layer that mirrors the reference's
// Metal bridge (src/metal/bridge.h:25-70).
#include <climits>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/vtb_cuda.h"
#include "common.cuh"

namespace vtb {
cudaError_t launch_gemv(int q, const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                        int accumulate = 0);
cudaError_t launch_gemv_q4k_mma(const void* w, const float* x, float* y, int m, int k, cudaStream_t st, bool pdl,
                                int accumulate, const float* norm_w, float eps, float* swi);
cudaError_t launch_gemv_q8_0_q8_0(const void* w, const int8_t* xq, const float* dx, float* y, int m, int k,
                                  cudaStream_t st, bool pdl, int accumulate = 0);
cudaError_t launch_dequant(int q, const void* w, float* out, long long n, cudaStream_t st);
cudaError_t launch_embed(int q, const void* table, const int32_t* ids, float* out, int dim, int n_tok,
                         cudaStream_t st);
cudaError_t launch_quantize_q8_0(const float* x, int8_t* qs, float* d, int nblocks, cudaStream_t st);
cudaError_t launch_gemv_q8_0_q8_0_x(const void* w, const float* x, int8_t* xq, float* dx, float* y, int m, int k,
                                    cudaStream_t st, bool pdl, int accumulate);

cudaError_t launch_q8_0_block_dots(const void* w, const int8_t* xq, int32_t* dots, int m, int nb, cudaStream_t st);
cudaError_t launch_gemm_tc(int q, const void* w, const float* acts, float* out, int m, int k, int nb, bool precise,
                           void* ws, cudaStream_t st, float* part, size_t part_elems, long long pitch);
}  // namespace vtb

using namespace vtb;

static thread_local char g_last_err[256] = "";
static thread_local int g_last_status = 0;

static int set_err(int status, const char* fmt, const char* detail = "") {
  snprintf(g_last_err, sizeof g_last_err, fmt, detail);
  g_last_status = status;
  return status;
}
static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return VTB_CUDA_OK;
  snprintf(g_last_err, sizeof g_last_err, "CUDA: %s", cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return VTB_CUDA_ERR_OOM;
  return VTB_CUDA_ERR_DISPATCH;
}
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_mat(int quant, const void* w, int64_t m, int64_t k) {
  if (!host_quant_ok(quant)) return set_err(VTB_CUDA_ERR_UNSUPPORTED, "unsupported quant type");
  if (!w) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null weight pointer");
  if (!aligned16(w)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "weight pointer is not 16-byte aligned");
  if (m <= 0 || k <= 0 || m > INT_MAX || k > INT_MAX)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "m and k must be in [1, 2^31)");
  if (k % host_block_elems(quant)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "k is not a whole number of blocks");
  return VTB_CUDA_OK;
}

extern "C" {

const char* vtb_cuda_version_string(void) { return "vantablack-b200 0.1.0 (sm_100a)"; }

int vtb_cuda_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  return major == 10 ? 1 : 0;
}

const char* vtb_cuda_status_string(int s) {
  switch (s) {
    case VTB_CUDA_OK: return "ok";
    case VTB_CUDA_ERR_INVALID_ARG: return "invalid argument";
    case VTB_CUDA_ERR_OOM: return "out of device memory";
    case VTB_CUDA_ERR_DEVICE: return "no usable CUDA device";
    case VTB_CUDA_ERR_DISPATCH: return "kernel dispatch failed";
    case VTB_CUDA_ERR_UNSUPPORTED: return "unsupported quant type";
    case VTB_CUDA_ERR_TIMEOUT: return "device-side bounded wait timed out";
    case VTB_CUDA_ERR_COMM: return "collective communication failed";
    case VTB_CUDA_ERR_FILE_OPEN: return "file cannot be opened";
    case VTB_CUDA_ERR_PARSE: return "malformed model file";
    default: return "unknown status";
  }
}

const char* vtb_cuda_last_error(void) { return g_last_err; }
int vtb_cuda_last_status(void) { return g_last_status; }

int64_t vtb_cuda_row_bytes(int quant, int64_t k) {
  if (k < 0 || (quant != F32 && (!host_quant_ok(quant) || k % host_block_elems(quant)))) return -1;
  return host_row_bytes(quant, k);
}

int vtb_cuda_check_device_error(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  unsigned v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, g_dev_error, sizeof v);
  if (e != cudaSuccess) return cuda_status(e);
  if (v) {
    cudaMemcpyToSymbol(g_dev_error, &zero, sizeof zero);
    snprintf(g_last_err, sizeof g_last_err, "device error word 0x%x", v);
    return VTB_CUDA_ERR_TIMEOUT;
  }
  return VTB_CUDA_OK;
}

int vtb_cuda_gemv(int quant, const void* w, const float* x, float* y, int64_t m, int64_t k, void* stream, int pdl) {
  cudaGetLastError();  // drop a stale error left by an unrelated earlier call
  int rc = check_mat(quant, w, m, k);
  if (rc) return rc;
  if (!x || !y) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null x or y");
  if (!aligned16(x)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "x is not 16-byte aligned");
  if (quant == Q4_K)
    return cuda_status(launch_gemv_q4k_mma(w, x, y, (int)m, (int)k, (cudaStream_t)stream, pdl != 0, 0, nullptr, 0.f, nullptr));
  return cuda_status(launch_gemv(quant, w, x, y, (int)m, (int)k, (cudaStream_t)stream, pdl != 0));
}

int vtb_cuda_dequant(int quant, const void* w, float* out, int64_t n, void* stream) {
  cudaGetLastError();
  if (!host_quant_ok(quant)) return set_err(VTB_CUDA_ERR_UNSUPPORTED, "unsupported quant type");
  if (!w || !out || n < 0 || n % host_block_elems(quant))
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad dequant arguments");
  if (n == 0) return VTB_CUDA_OK;
  return cuda_status(launch_dequant(quant, w, out, n, (cudaStream_t)stream));
}

int vtb_cuda_embed(int quant, const void* table, const int32_t* ids, float* out, int64_t dim, int64_t n_tokens,
                   void* stream) {
  cudaGetLastError();
  if (!host_quant_ok(quant)) return set_err(VTB_CUDA_ERR_UNSUPPORTED, "unsupported quant type");
  if (!table || !ids || !out || dim <= 0 || dim % host_block_elems(quant) || n_tokens < 0 || n_tokens > 65535)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad embed arguments");
  if (n_tokens == 0) return VTB_CUDA_OK;
  return cuda_status(launch_embed(quant, table, ids, out, (int)dim, (int)n_tokens, (cudaStream_t)stream));
}

int vtb_cuda_quantize_q8_0(const float* x, int64_t k, int8_t* qs, float* d, void* stream) {
  cudaGetLastError();
  if (!x || !qs || !d || k <= 0 || k % 32 || k > INT_MAX)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad quantize arguments");
  return cuda_status(launch_quantize_q8_0(x, qs, d, (int)(k / 32), (cudaStream_t)stream));
}

int vtb_cuda_q8_0_block_dots(const void* w, const int8_t* xq, int32_t* dots, int64_t m, int64_t k, void* stream) {
  cudaGetLastError();
  int rc = check_mat(Q8_0, w, m, k);
  if (rc) return rc;
  if (!xq || !dots || (reinterpret_cast<uintptr_t>(xq) & 3u))
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad xq/dots pointer");
  return cuda_status(launch_q8_0_block_dots(w, xq, dots, (int)m, (int)(k / 32), (cudaStream_t)stream));
}

int vtb_cuda_gemv_q8_0_q8_0(const void* w, const float* x, float* y, int64_t m, int64_t k, int8_t* xq_scratch,
                            float* dx_scratch, void* stream, int pdl) {
  cudaGetLastError();
  int rc = check_mat(Q8_0, w, m, k);
  if (rc) return rc;
  if (!x || !y || !xq_scratch || !dx_scratch) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(xq_scratch)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "xq_scratch is not 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  return cuda_status(launch_gemv_q8_0_q8_0_x(w, x, xq_scratch, dx_scratch, y, (int)m, (int)k, st, pdl != 0, 0));
}

size_t vtb_cuda_gemm_workspace_bytes(int64_t k, int64_t n_tokens, int precise) {
  if (k <= 0 || n_tokens <= 0) return 0;
  return (size_t)(k * n_tokens * 2 * (precise ? 2 : 1));
}

int vtb_cuda_gemm(int quant, const void* w, const float* acts, float* out, int64_t m, int64_t k, int64_t n_tokens,
                  int precise, void* workspace, size_t workspace_bytes, void* stream) {
  cudaGetLastError();
  int rc = check_mat(quant, w, m, k);
  if (rc) return rc;
  if (k % 64) return set_err(VTB_CUDA_ERR_INVALID_ARG, "gemm needs k to be a multiple of 64");
  if (!acts || !out || !workspace || n_tokens <= 0 || n_tokens > 65535 * 64)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad gemm arguments");
  if (workspace_bytes < vtb_cuda_gemm_workspace_bytes(k, n_tokens, precise))
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "gemm workspace too small");
  if (!aligned16(acts) || !aligned16(workspace)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "acts/workspace not 16-byte aligned");
  return cuda_status(launch_gemm_tc(quant, w, acts, out, (int)m, (int)k, (int)n_tokens, precise != 0, workspace,
                                    (cudaStream_t)stream, nullptr, 0));
}

}  // extern "C"

// ---------------- context / buffers ----------------
struct VtbSegCache;  // segment.cu: the open segment and the graphs of recent ones
namespace vtb {
void seg_cache_destroy(VtbSegCache* s);
}
struct VtbCudaCtx {
  int device;
  cudaStream_t stream;
  VtbSegCache* seg;
};
struct VtbCudaBuf {
  VtbCudaCtx* ctx;
  void* ptr;
  size_t size;
};

static bool use_ctx(VtbCudaCtx* c) { return c && cudaSetDevice(c->device) == cudaSuccess; }

extern "C" {

int vtb_cuda_capabilities(const VtbCudaCtx* ctx, VtbCudaCapabilities* out) {
  if (!out) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null output");
  out->supports_fused_qkv = 1;
  out->supports_kquant_gpu = 1;
  out->supports_mlx_q4 = 0;
  out->unified_memory = 0;
  out->name = "cuda-b200 (sm_100a)";
  if (ctx) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, ctx->device) != cudaSuccess) {
      cudaGetLastError();
      return set_err(VTB_CUDA_ERR_DEVICE, "cannot query the context's device");
    }
    if (major != 10) return set_err(VTB_CUDA_ERR_DEVICE, "the context's device is not sm_100");
  }
  return VTB_CUDA_OK;
}

VtbCudaCtx* vtb_cuda_init(int device_ordinal) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device_ordinal < 0 || device_ordinal >= n) {
    cudaGetLastError();
    set_err(VTB_CUDA_ERR_DEVICE, "no such CUDA device");
    return nullptr;
  }
  if (cudaSetDevice(device_ordinal) != cudaSuccess) return nullptr;
  VtbCudaCtx* c = new (std::nothrow) VtbCudaCtx{device_ordinal, nullptr, nullptr};
  if (!c) return nullptr;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return nullptr;
  }
  return c;
}

void vtb_cuda_destroy(VtbCudaCtx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  vtb::seg_cache_destroy(c->seg);
  cudaStreamDestroy(c->stream);
  delete c;
}

void* vtb_cuda_stream(VtbCudaCtx* c) { return c ? (void*)c->stream : nullptr; }

VtbCudaBuf* vtb_cuda_alloc(VtbCudaCtx* c, size_t bytes, void** dev_ptr_out) {
  if (!use_ctx(c) || bytes == 0) return nullptr;
  void* p = nullptr;
  // +256: bulk copies may read up to the next 16-byte boundary past the end.
  if (cudaMalloc(&p, bytes + 256) != cudaSuccess) {
    cuda_status(cudaGetLastError());
    return nullptr;
  }
  VtbCudaBuf* b = new (std::nothrow) VtbCudaBuf{c, p, bytes};
  if (!b) {
    cudaFree(p);
    return nullptr;
  }
  if (dev_ptr_out) *dev_ptr_out = p;
  return b;
}

VtbCudaBuf* vtb_cuda_upload(VtbCudaCtx* c, const void* host, size_t len) {
  if (!host) return nullptr;
  VtbCudaBuf* b = vtb_cuda_alloc(c, len, nullptr);
  if (!b) return nullptr;
  if (cudaMemcpyAsync(b->ptr, host, len, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      cudaStreamSynchronize(c->stream) != cudaSuccess) {
    vtb_cuda_release(b);
    return nullptr;
  }
  return b;
}

void vtb_cuda_release(VtbCudaBuf* b) {
  if (!b) return;
  cudaSetDevice(b->ctx->device);
  cudaStreamSynchronize(b->ctx->stream);
  cudaFree(b->ptr);
  delete b;
}

void* vtb_cuda_buf_ptr(VtbCudaBuf* b) { return b ? b->ptr : nullptr; }
size_t vtb_cuda_buf_size(VtbCudaBuf* b) { return b ? b->size : 0; }

int vtb_cuda_copy_h2d(VtbCudaCtx* c, VtbCudaBuf* dst, size_t off, const void* src, size_t bytes) {
  if (!use_ctx(c) || !dst || !src || off + bytes > dst->size) return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad h2d copy");
  return cuda_status(cudaMemcpyAsync((char*)dst->ptr + off, src, bytes, cudaMemcpyHostToDevice, c->stream));
}

int vtb_cuda_copy_d2h(VtbCudaCtx* c, void* dst, VtbCudaBuf* src, size_t off, size_t bytes) {
  if (!use_ctx(c) || !dst || !src || off + bytes > src->size) return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad d2h copy");
  cudaError_t e = cudaMemcpyAsync(dst, (const char*)src->ptr + off, bytes, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return cuda_status(e);
}

int vtb_cuda_copy_d2h_async(VtbCudaCtx* c, void* dst, VtbCudaBuf* src, size_t off, size_t bytes) {
  if (!use_ctx(c) || !dst || !src || off + bytes > src->size) return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad d2h copy");
  return cuda_status(cudaMemcpyAsync(dst, (const char*)src->ptr + off, bytes, cudaMemcpyDeviceToHost, c->stream));
}

int vtb_cuda_wait_idle(VtbCudaCtx* c) {
  if (!use_ctx(c)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null context");
  return cuda_status(cudaStreamSynchronize(c->stream));
}

static int ctx_matmul(int q, VtbCudaCtx* c, VtbCudaBuf* out, VtbCudaBuf* w, size_t w_off, VtbCudaBuf* acts, size_t m,
                      size_t k) {
  if (!use_ctx(c) || !out || !w || !acts) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null buffer");
  const int64_t rb = host_row_bytes(q, (int64_t)k);
  if (rb <= 0 || w_off + (size_t)rb * m > w->size || out->size < m * 4 || acts->size < k * 4)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "buffer too small for m x k");
  // Programmatic dependent launch: consecutive matmuls on the context stream
  // overlap launch and weight prefetch; each kernel reads acts and writes out
  // only after waiting for its predecessor, so buffer reuse stays ordered.
  return vtb_cuda_gemv(q, (const char*)w->ptr + w_off, (const float*)acts->ptr, (float*)out->ptr, (int64_t)m,
                       (int64_t)k, c->stream, 1);
}

int vtb_cuda_matmul_q8_0(VtbCudaCtx* c, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m, size_t k) {
  return ctx_matmul(Q8_0, c, o, w, off, a, m, k);
}
int vtb_cuda_matmul_q4_k(VtbCudaCtx* c, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m, size_t k) {
  return ctx_matmul(Q4_K, c, o, w, off, a, m, k);
}
int vtb_cuda_matmul_q5_k(VtbCudaCtx* c, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m, size_t k) {
  return ctx_matmul(Q5_K, c, o, w, off, a, m, k);
}
int vtb_cuda_matmul_q6_k(VtbCudaCtx* c, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m, size_t k) {
  return ctx_matmul(Q6_K, c, o, w, off, a, m, k);
}
int vtb_cuda_matmul_tq2_0(VtbCudaCtx* c, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m, size_t k) {
  return ctx_matmul(TQ2_0, c, o, w, off, a, m, k);
}

}  // extern "C"

#ifdef VTB_TIMELINE
// Development builds only (-DVTB_TIMELINE): copies the launch timeline ring
// (8 u64 per record: id | sm << 32, entry, wait returned, exit, 4 marks) into `out`,
// oldest first, and returns the record count; reset != 0 clears it.
extern "C" int vtb_cuda_timeline(unsigned long long* out, int max_records, int reset) {
  unsigned n = 0;
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(&n, vtb::g_tl_n, sizeof n) != cudaSuccess)
    return -1;
  const unsigned have = n < vtb::kTlRing ? n : vtb::kTlRing;
  std::vector<unsigned long long> ring(8 * (size_t)vtb::kTlRing);
  if (cudaMemcpyFromSymbol(ring.data(), vtb::g_tl, ring.size() * 8) != cudaSuccess) return -1;
  int k = 0;
  for (unsigned j = n - have; j < n && k < max_records; ++j, ++k)
    for (int c = 0; c < 8; ++c) out[8 * k + c] = ring[8 * (j % vtb::kTlRing) + c];
  if (reset) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(vtb::g_tl_n, &zero, sizeof zero);
  }
  return k;
}
#endif

