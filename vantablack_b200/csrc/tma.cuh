// tma.cuh -- 2-D tensor maps (TMA descriptors) and the tiled bulk load, shared
// by the prefill GEMM and the Q4_K decode GEMV.  The encoder comes from the
// driver entry point, so the library links only the CUDA runtime.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace vtb {

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D map of a [rows][inner] array (inner contiguous, row pitch in bytes).
// A map is a pure function of its arguments, so each host thread keeps the
// last ones it encoded (direct-mapped on the base address): a decode loop
// that launches the same matrices again skips the encode.
static bool make_tmap(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                      uint64_t pitch, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  struct Entry {
    const void* base;
    uint64_t inner, rows, pitch;
    uint32_t box_inner, box_rows;
    int dt, sw;
    CUtensorMap map;
  };
  constexpr int kSlots = 64;
  static thread_local Entry cache[kSlots];
  Entry& e = cache[(reinterpret_cast<uintptr_t>(base) >> 8) % kSlots];
  if (e.base == base && e.inner == inner && e.rows == rows && e.pitch == pitch && e.box_inner == box_inner &&
      e.box_rows == box_rows && e.dt == (int)dt && e.sw == (int)sw) {
    *map = e.map;
    return true;
  }
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  e = Entry{base, inner, rows, pitch, box_inner, box_rows, (int)dt, (int)sw, *map};
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace vtb
