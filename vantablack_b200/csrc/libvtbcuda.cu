// libvtbcuda.cu -- single translation unit of the backend library: the
// kernels share device globals (the error word), so they are compiled
// together without relocatable device code.
#include "gemv_q6k_mma.cu"
#include "gemv.cu"
#include "gemv_mma.cu"
#include "gemv_q8_mma.cu"
#include "quant_aux.cu"
#include "gemm_tc.cu"
#include "api.cu"
#include "segment.cu"
#include "tp.cu"
#include "model.cu"
#include "gguf.cu"
#include "noalloc.cu"
#include "sampler.cu"
#include "mlx.cu"
