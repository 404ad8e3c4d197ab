/* bridge_loop.c -- a native caller of the C ABI for bench.py's end-to-end
 * measurement.  The reference's host is compiled code that calls the Metal
 * bridge directly (src/runtime/metal_backend.zig:389-455 through
 * src/metal/bridge.zig); timing the same calls from Python would mostly time
 * ctypes.  One step is what such a host does for a batch of matmuls whose
 * results it reads: copy the activations in from host memory, enqueue the
 * matmuls, read every result back, wait.  Uses only include/vtb_cuda.h. */
#define _POSIX_C_SOURCE 199309L
#include <stddef.h>
#include <time.h>

#include "../../include/vtb_cuda.h"

static double now_s(void) {
  struct timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

/* One step over n Q4_K matrices w[i] (m x k) applied to x: host hx -> xb,
 * y[i] = W_i . x, y[i] -> hy + i * m.  segment != 0: one segment per step
 * (vtb_cuda_segment_*); 0: the one-shot calls (vtb_cuda_matmul_q4_k and
 * vtb_cuda_copy_d2h_async) and vtb_cuda_wait_idle.  Returns 0 or the first
 * failing status. */
static int step(VtbCudaCtx *ctx, VtbCudaBuf **w, VtbCudaBuf **y, VtbCudaBuf *xb, const float *hx, float *hy, int n,
                size_t m, size_t k, int segment) {
  int rc;
  if (segment) {
    VtbCudaSeg *seg = vtb_cuda_segment_begin(ctx);
    if (!seg) return VTB_CUDA_ERR_INVALID_ARG;
    vtb_cuda_segment_copy_h2d(seg, xb, 0, hx, k * sizeof(float));
    for (int i = 0; i < n; ++i) vtb_cuda_segment_matmul_q4_k(seg, y[i], w[i], 0, xb, m, k);
    for (int i = 0; i < n; ++i) vtb_cuda_segment_copy_d2h(seg, hy + (size_t)i * m, y[i], 0, m * sizeof(float));
    if ((rc = vtb_cuda_segment_commit(seg)) != VTB_CUDA_OK) return rc;
  } else {
    if ((rc = vtb_cuda_copy_h2d(ctx, xb, 0, hx, k * sizeof(float))) != VTB_CUDA_OK) return rc;
    for (int i = 0; i < n; ++i)
      if ((rc = vtb_cuda_matmul_q4_k(ctx, y[i], w[i], 0, xb, m, k)) != VTB_CUDA_OK) return rc;
    for (int i = 0; i < n; ++i)
      if ((rc = vtb_cuda_copy_d2h_async(ctx, hy + (size_t)i * m, y[i], 0, m * sizeof(float))) != VTB_CUDA_OK)
        return rc;
  }
  return vtb_cuda_wait_idle(ctx);
}

/* Runs `warmup` untimed steps, then `steps` timed ones; *seconds = the timed
 * wall-clock time.  Returns 0 or the first failing status. */
int vtb_bench_bridge_q4k(VtbCudaCtx *ctx, VtbCudaBuf **w, VtbCudaBuf **y, VtbCudaBuf *xb, const float *hx, float *hy,
                         int n, size_t m, size_t k, int warmup, int steps, int segment, double *seconds) {
  int rc;
  for (int s = 0; s < warmup; ++s)
    if ((rc = step(ctx, w, y, xb, hx, hy, n, m, k, segment)) != VTB_CUDA_OK) return rc;
  const double t0 = now_s();
  for (int s = 0; s < steps; ++s)
    if ((rc = step(ctx, w, y, xb, hx, hy, n, m, k, segment)) != VTB_CUDA_OK) return rc;
  *seconds = now_s() - t0;
  return VTB_CUDA_OK;
}
