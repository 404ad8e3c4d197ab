// noalloc.cu -- an allocation-free variant of the Q8_0 x Q8_0 GEMV.
//
// Some hosts cannot call cudaMalloc on the decode path: an engine that runs
// under a fixed device-memory budget reserved at start-up, or a serving loop
// that forbids any allocation once it is warm (an allocation can block on
// the driver, fail under memory pressure, or fragment a pool the host
// manages itself).  vtb_cuda_gemv_q8_0_q8_0 needs scratch for the quantized
// activations, which its caller must allocate; this variant instead keeps that
// scratch in a fixed array compiled into the library, so the caller passes
// only the weights, x and y.
#include <mutex>

#include "../../include/vtb_cuda.h"
#include "common.cuh"

namespace vtb {

// Activation scratch, k <= VTB_CUDA_NOALLOC_MAX_K: k bytes of int8 quants
// followed by k/32 float scales.  Every GPU that loads the library holds this
// 72 KiB until the process exits.  Host code must not pass the symbol itself
// to a kernel: on the host it is only a stand-in; the device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_q8_scratch[VTB_CUDA_NOALLOC_MAX_K +
                                                                     (VTB_CUDA_NOALLOC_MAX_K / 32) * 4];

static std::mutex g_noalloc_mu;
static unsigned char* g_noalloc_dev_ptr[64];  // per device ordinal, filled on first use

}  // namespace vtb

extern "C" int vtb_cuda_gemv_q8_0_q8_0_noalloc(const void* w, const float* x, float* y, int64_t m, int64_t k,
                                               void* stream, int pdl) {
  using namespace vtb;
  cudaGetLastError();
  int rc = check_mat(Q8_0, w, m, k);
  if (rc) return rc;
  if (!x || !y) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null x or y");
  if (k > VTB_CUDA_NOALLOC_MAX_K)
    return set_err(VTB_CUDA_ERR_INVALID_ARG,
                   "k exceeds the fixed scratch of vtb_cuda_gemv_q8_0_q8_0_noalloc (VTB_CUDA_NOALLOC_MAX_K = 65536)");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return set_err(VTB_CUDA_ERR_DEVICE, "device ordinal above 63");
  unsigned char* base;
  {
    // First call on this device (which must be current): resolve the array's
    // device address once.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_dev_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_q8_scratch);
      if (e != cudaSuccess) return cuda_status(e);
      g_noalloc_dev_ptr[dev] = static_cast<unsigned char*>(p);
    }
    base = g_noalloc_dev_ptr[dev];
  }
  int8_t* xq = reinterpret_cast<int8_t*>(base);
  float* dx = reinterpret_cast<float*>(base + VTB_CUDA_NOALLOC_MAX_K);
  // Every call rewrites the k quants and k/32 scales before anything reads
  // them (the tensor-core path quantizes inside the GEMV and stores them; the
  // SIMT path runs the quantizer first), so nothing has to be cleared.
  cudaStream_t st = (cudaStream_t)stream;
  return cuda_status(launch_gemv_q8_0_q8_0_x(w, x, xq, dx, y, (int)m, (int)k, st, pdl != 0, 0));
}
