// tp.cu -- tensor parallelism across GPUs of one node (NCCL over NVLink /
// NVSwitch), the multi-GPU extension of the forward loop.  The reference has
// no multi-device code; this follows the standard Llama sharding:
//   * Q, K, V: split by heads (output rows); attention and the KV cache are
//     local to a rank's heads.
//   * O: split along K (the rank's head columns); the partial outputs are
//     all-reduced (sum) and added to the residual stream.
//   * gate, up: split by output rows (ffn/world each); down: split along K,
//     then all-reduce.
//   * LM head: split by vocabulary rows; the logit slices are all-gathered.
//   * token embedding and norms are replicated.
// K splits must stay on whole quantization blocks.
#include <nccl.h>

#include <cstring>
#include <new>

#include "../../include/vtb_cuda.h"
#include "common.cuh"

struct VtbCudaTp {
  int rank = 0, world = 1, device = 0;
  ncclComm_t comm = nullptr;
};

extern "C" {

int vtb_cuda_tp_unique_id(uint8_t* out) {
  if (!out) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null id buffer");
  static_assert(sizeof(ncclUniqueId) == VTB_CUDA_TP_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  const ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_err(VTB_CUDA_ERR_COMM, "NCCL: %s", ncclGetErrorString(r));
  memcpy(out, &id, sizeof id);
  return VTB_CUDA_OK;
}

VtbCudaTp* vtb_cuda_tp_init(int device, int rank, int world, const uint8_t* id) {
  if (!id || world < 1 || rank < 0 || rank >= world) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "bad tensor-parallel rank/world");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    cuda_status(cudaGetLastError());
    return nullptr;
  }
  VtbCudaTp* tp = new (std::nothrow) VtbCudaTp();
  if (!tp) return nullptr;
  tp->rank = rank;
  tp->world = world;
  tp->device = device;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  const ncclResult_t r = ncclCommInitRank(&tp->comm, world, uid, rank);
  if (r != ncclSuccess) {
    set_err(VTB_CUDA_ERR_COMM, "NCCL: %s", ncclGetErrorString(r));
    delete tp;
    return nullptr;
  }
  return tp;
}

void vtb_cuda_tp_destroy(VtbCudaTp* tp) {
  if (!tp) return;
  if (tp->comm) ncclCommDestroy(tp->comm);
  delete tp;
}

int vtb_cuda_tp_rank(const VtbCudaTp* tp) { return tp ? tp->rank : 0; }
int vtb_cuda_tp_world(const VtbCudaTp* tp) { return tp ? tp->world : 1; }

// Pure host arithmetic: which rows / columns rank `rank` owns.
int vtb_cuda_tp_shard_plan(const VtbCudaLlamaConfig* c, int rank, int world, int32_t k_block,
                           VtbCudaTpShard* out) {
  if (!c || !out || world < 1 || rank < 0 || rank >= world || k_block <= 0)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad shard-plan arguments");
  if (c->n_heads % world || c->n_kv_heads % world || c->ffn_dim % world || c->vocab_size % world)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "heads, kv heads, ffn and vocab must divide by the world size");
  const int hd = c->head_dim;
  VtbCudaTpShard s;
  s.heads = c->n_heads / world;
  s.kv_heads = c->n_kv_heads / world;
  s.q_row0 = rank * s.heads * hd;
  s.q_rows = s.heads * hd;
  s.kv_row0 = rank * s.kv_heads * hd;
  s.kv_rows = s.kv_heads * hd;
  s.ffn_row0 = rank * (c->ffn_dim / world);
  s.ffn_rows = c->ffn_dim / world;
  s.o_col0 = s.q_row0;  // O's K range = this rank's head outputs
  s.o_cols = s.q_rows;
  s.down_col0 = s.ffn_row0;
  s.down_cols = s.ffn_rows;
  s.vocab_row0 = rank * (c->vocab_size / world);
  s.vocab_rows = c->vocab_size / world;
  if (s.o_cols % k_block || s.down_cols % k_block || s.o_col0 % k_block || s.down_col0 % k_block)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "K shards of O / down are not whole quantization blocks");
  *out = s;
  return VTB_CUDA_OK;
}

// Pure host copy of rows [row0, row0+nrows) x columns [col0, col0+ncols) of
// a [rows, k] quantized tensor (columns on block boundaries) into dst.
int vtb_cuda_tp_slice(int quant, const void* src, int64_t rows, int64_t k, int64_t row0, int64_t nrows, int64_t col0,
                      int64_t ncols, void* dst) {
  const int el = quant == F32 ? 1 : host_block_elems(quant);
  if (!src || !dst || (quant != F32 && !host_quant_ok(quant)) || k % el || col0 % el || ncols % el || row0 < 0 ||
      col0 < 0 || nrows < 0 || ncols < 0 || row0 + nrows > rows || col0 + ncols > k)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad slice");
  const int64_t rb = host_row_bytes(quant, k), off = host_row_bytes(quant, col0), w = host_row_bytes(quant, ncols);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  for (int64_t r = 0; r < nrows; ++r) memcpy(d + r * w, s + (row0 + r) * rb + off, (size_t)w);
  return VTB_CUDA_OK;
}

}  // extern "C"

namespace vtb {
static int nccl_status(ncclResult_t r) {
  if (r == ncclSuccess) return VTB_CUDA_OK;
  return set_err(VTB_CUDA_ERR_COMM, "NCCL: %s", ncclGetErrorString(r));
}
}  // namespace vtb
