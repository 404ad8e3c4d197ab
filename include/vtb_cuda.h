/*
 * vtb_cuda.h -- C ABI of the vantablack B200 (sm_100a) CUDA backend.
 *
 * This is the flat shim a `backend_cuda.zig` binds with `extern "c"`
 * declarations, the way the reference binds its Metal bridge
 * (src/metal/bridge.h:25-228 declared in src/metal/bridge.zig:16-60).
 * Every signature uses plain pointers, sizes and opaque handles only.
 *
 * Conventions
 *  - Every function returning int returns VTB_CUDA_OK (0) on success and a
 *    negative status on failure (the reference's bridge returns nonzero on
 *    failure, bridge.h:47; the codes reuse include/vantablack.h:25-33 values
 *    so the Zig side can map them straight through mapStreamErr,
 *    src/c_api.zig:332-340).
 *  - Quant types are ggml type ids (src/core/parser.zig GgmlType):
 *    VTB_CUDA_Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14.
 *  - "Device pointer" arguments are CUDA global-memory addresses on the
 *    current device.  `stream` is a cudaStream_t passed as void* (NULL = the
 *    legacy default stream).  Launches are asynchronous on that stream.
 *  - Weight tensors are row-major packed blocks (m rows of k/elems blocks).
 *    Their base must be 16-byte aligned and the allocation readable up to
 *    the next 16-byte boundary past its end (cudaMalloc and the context
 *    allocator below guarantee both).
 */
#ifndef VTB_CUDA_H
#define VTB_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VTB_CUDA_OK 0
#define VTB_CUDA_ERR_INVALID_ARG (-1)
#define VTB_CUDA_ERR_FILE_OPEN (-2) /* VTB_ERR_FILE_OPEN: a GGUF file cannot be opened or mapped */
#define VTB_CUDA_ERR_PARSE (-3)     /* VTB_ERR_PARSE: malformed GGUF or missing model metadata */
#define VTB_CUDA_ERR_OOM (-4)
#define VTB_CUDA_ERR_DEVICE (-5)
#define VTB_CUDA_ERR_DISPATCH (-6)
#define VTB_CUDA_ERR_STREAM_ABORTED (-7)
#define VTB_CUDA_ERR_UNSUPPORTED (-8)
#define VTB_CUDA_ERR_TIMEOUT (-9)
#define VTB_CUDA_ERR_COMM (-10)

#define VTB_CUDA_F32 0
#define VTB_CUDA_Q8_0 8
#define VTB_CUDA_Q4_K 12
#define VTB_CUDA_Q5_K 13
#define VTB_CUDA_Q6_K 14
/* TQ2_0 (66 B / 256 weights) with the reference's GgmlType id (parser.zig:62) and
 * its block layout (simd.zig:436-472), which differs from ggml's. */
#define VTB_CUDA_TQ2_0 32

/* ------------------------------------------------------------------ */
/* Introspection                                                        */
/* ------------------------------------------------------------------ */

/* Static version string (cf. vtb_version_string, include/vantablack.h:128). */
const char *vtb_cuda_version_string(void);
/* 1 when a CUDA device of compute capability 10.x is visible (cf. vtb_has_metal,
 * include/vantablack.h:131). */
int vtb_cuda_available(void);
/* The vtable's `capabilities` slot (src/runtime/backend.zig:43-55, :93):
 * what this backend reports to the forward loop.  supports_fused_qkv = 1
 * (Q|K|V and gate|up rows are concatenated at upload), supports_kquant_gpu =
 * 1, supports_mlx_q4 = 0, unified_memory = 0 (weights and state live in HBM;
 * finalize_token copies the logits to the host).  `name` is a static string.
 * `ctx` may be NULL; with a context the device is checked to be sm_100. */
typedef struct VtbCudaCapabilities {
  int32_t supports_fused_qkv;
  int32_t supports_kquant_gpu;
  int32_t supports_mlx_q4;
  int32_t unified_memory;
  const char *name;
} VtbCudaCapabilities;
struct VtbCudaCtx;
int vtb_cuda_capabilities(const struct VtbCudaCtx *ctx, VtbCudaCapabilities *out);
/* Human-readable text for a status code. */
const char *vtb_cuda_status_string(int status);
/* Text of the last CUDA error this thread saw inside the library. */
const char *vtb_cuda_last_error(void);
/* Status of the last failure recorded with that text (for calls that return
 * a NULL handle, e.g. vtb_cuda_gguf_open: -2 open / map, -3 malformed). */
int vtb_cuda_last_status(void);
/* Bytes per row of k weights in `quant` format (forward.zig rowBytes :629-641);
 * -1 if unsupported or k is not a whole number of blocks. */
int64_t vtb_cuda_row_bytes(int quant, int64_t k);
/* Reads and clears the device error word that bounded waits in the kernels
 * set when they give up (then VTB_CUDA_ERR_TIMEOUT); synchronizes the device. */
int vtb_cuda_check_device_error(void);

/* ------------------------------------------------------------------ */
/* Stream-level kernels (device pointers)                               */
/* ------------------------------------------------------------------ */

/* y[m] = W[m,k] . x[k], f32 activations, fp32 accumulation.  Replaces the
 * per-quant CPU kernels matmul_q8_0 / q4_k / q5_k / q6_k
 * (src/kernels/simd.zig:159, 245, 321, 406) behind comptime_gen.zig:44-58
 * dispatch, and the Metal one-shots vtb_metal_matmul_* (bridge.h:48-70).
 * `pdl` != 0 launches with programmatic dependent launch, so the weight
 * stream starts before the previous kernel on `stream` has finished. */
int vtb_cuda_gemv(int quant, const void *w, const float *x, float *y, int64_t m, int64_t k,
                  void *stream, int pdl);

/* Dequantize n elements (whole blocks) to f32, bit-exact with
 * dequantBlockQ*_* (simd.zig:153, 221, 290, 366) / dequantToF32
 * (src/runtime/forward.zig:654-736). */
int vtb_cuda_dequant(int quant, const void *w, float *out, int64_t n, void *stream);

/* out[t, :] = dequantized row ids[t] of a [rows, dim] table
 * (gatherEmbedding, forward.zig:738-845). */
int vtb_cuda_embed(int quant, const void *table, const int32_t *ids, float *out, int64_t dim,
                   int64_t n_tokens, void *stream);

/* Q8_0 activation quantizer for the Q8_0 x Q8_0 path: per 32-block
 * d = max|x| / 127, q = round-half-away(x * (1/d)).  The reference has no
 * quantizer (only dot_i8, simd.zig:31-62); this rule is the backend's own. */
int vtb_cuda_quantize_q8_0(const float *x, int64_t k, int8_t *qs, float *d, void *stream);

/* dots[i, b] = dot_i8(W_qs[i, b, :], xq[b, :]) as int32 (simd.zig:40-62). */
int vtb_cuda_q8_0_block_dots(const void *w, const int8_t *xq, int32_t *dots, int64_t m, int64_t k,
                             void *stream);

/* Q8_0 x Q8_0 GEMV: quantizes x into caller scratch (xq_scratch: k bytes,
 * dx_scratch: k/32 floats), then y[i] = sum_b (d_w * d_x) * float(int32 dot). */
int vtb_cuda_gemv_q8_0_q8_0(const void *w, const float *x, float *y, int64_t m, int64_t k,
                            int8_t *xq_scratch, float *dx_scratch, void *stream, int pdl);

/* Prefill GEMM: out[b, i] = sum_j W[i, j] * acts[b, j] for n_tokens rows of
 * f32 activations (acts [n_tokens][k], out [n_tokens][m]) -- matmulBatched
 * (src/runtime/prefill.zig:325-378).  Runs on the tcgen05 tensor cores with
 * W dequantized (bit-exactly) to bf16 tiles in shared memory.  precise = 0:
 * bf16 operands (tolerance 2e-2); precise = 1: hi/lo-split operands, three
 * MMAs per tile (~16-bit products, fp32-class results).  k % 64 == 0.
 * `workspace` (device, 16-byte aligned) holds the converted activations:
 * vtb_cuda_gemm_workspace_bytes(k, n_tokens, precise) bytes. */
size_t vtb_cuda_gemm_workspace_bytes(int64_t k, int64_t n_tokens, int precise);
int vtb_cuda_gemm(int quant, const void *w, const float *acts, float *out, int64_t m, int64_t k,
                  int64_t n_tokens, int precise, void *workspace, size_t workspace_bytes, void *stream);

/* Allocation-free Q8_0 x Q8_0 GEMV.  No counterpart in the reference: it is
 * for hosts that cannot call cudaMalloc on their decode path (a fixed device
 * memory budget reserved up front, or a warm serving loop that forbids
 * allocation).  Same result as vtb_cuda_gemv_q8_0_q8_0, but the activation
 * scratch lives in a fixed array inside the library (72 KiB per GPU that
 * loads it, held until exit), so k must be <= VTB_CUDA_NOALLOC_MAX_K; larger
 * k is rejected with VTB_CUDA_ERR_INVALID_ARG.  The first call on a device
 * resolves the array's address on the current device; make that first call
 * before any stream capture.  The address is kept for the life of the
 * process: after cudaDeviceReset (or in another primary context) it is stale,
 * so do not call this entry point again in that process.  Every call rewrites
 * the quantized activations before anything reads them, so nothing carries
 * over from the previous call.  All calls share the one array: calls that can
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialized by the caller.  Allocates nothing. */
#define VTB_CUDA_NOALLOC_MAX_K 65536
int vtb_cuda_gemv_q8_0_q8_0_noalloc(const void *w, const float *x, float *y, int64_t m, int64_t k,
                                    void *stream, int pdl);

/* ------------------------------------------------------------------ */
/* Context / buffers (mirrors the Metal bridge, bridge.h:25-46)         */
/* ------------------------------------------------------------------ */

typedef struct VtbCudaCtx VtbCudaCtx;
typedef struct VtbCudaBuf VtbCudaBuf;

/* Bind device `device_ordinal`, create the context's stream (vtb_metal_init). */
VtbCudaCtx *vtb_cuda_init(int device_ordinal);
void vtb_cuda_destroy(VtbCudaCtx *ctx);
/* The context's cudaStream_t, as void*. */
void *vtb_cuda_stream(VtbCudaCtx *ctx);
/* Device allocation (vtb_metal_alloc); *dev_ptr_out receives the address. */
VtbCudaBuf *vtb_cuda_alloc(VtbCudaCtx *ctx, size_t bytes, void **dev_ptr_out);
/* Copy `len` host bytes (e.g. the GGUF mmap) into a new device buffer.
 * Replaces the no-copy vtb_metal_wrap (bridge.h:36-39): a discrete GPU
 * cannot alias host pages, so weights are uploaded once. */
VtbCudaBuf *vtb_cuda_upload(VtbCudaCtx *ctx, const void *host, size_t len);
void vtb_cuda_release(VtbCudaBuf *buf);
void *vtb_cuda_buf_ptr(VtbCudaBuf *buf);
size_t vtb_cuda_buf_size(VtbCudaBuf *buf);
int vtb_cuda_copy_h2d(VtbCudaCtx *ctx, VtbCudaBuf *dst, size_t dst_off, const void *src, size_t bytes);
/* Waits for the context stream, then copies. */
int vtb_cuda_copy_d2h(VtbCudaCtx *ctx, void *dst, VtbCudaBuf *src, size_t src_off, size_t bytes);
/* Enqueues the copy on the context stream and returns at once; dst holds the
 * data once vtb_cuda_wait_idle returns (the Metal bridge's read-after-
 * waitIdle pattern, bridge.h, without a wait per buffer).  dst must stay valid
 * until then; pinned host memory makes the copy asynchronous. */
int vtb_cuda_copy_d2h_async(VtbCudaCtx *ctx, void *dst, VtbCudaBuf *src, size_t src_off, size_t bytes);
/* Block until all work on the context stream is done (vtb_metal_wait_idle). */
int vtb_cuda_wait_idle(VtbCudaCtx *ctx);

/* One-shot matmuls with the Metal bridge's signature (bridge.h:48-70):
 * out_buf[m] = W(w_buf + w_offset)[m,k] . acts_buf[k].  Enqueued on the
 * context stream; results are visible to vtb_cuda_copy_d2h. */
int vtb_cuda_matmul_q8_0(VtbCudaCtx *ctx, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                         VtbCudaBuf *acts_buf, size_t m, size_t k);
int vtb_cuda_matmul_q4_k(VtbCudaCtx *ctx, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                         VtbCudaBuf *acts_buf, size_t m, size_t k);
int vtb_cuda_matmul_q5_k(VtbCudaCtx *ctx, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                         VtbCudaBuf *acts_buf, size_t m, size_t k);
int vtb_cuda_matmul_q6_k(VtbCudaCtx *ctx, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                         VtbCudaBuf *acts_buf, size_t m, size_t k);
/* TQ2_0: the reference's matmul_ternary158 (simd.zig:474-498), which it runs
 * on the CPU only; same signature as the bridge matmuls above. */
int vtb_cuda_matmul_tq2_0(VtbCudaCtx *ctx, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                          VtbCudaBuf *acts_buf, size_t m, size_t k);

/* Batched dispatch (vtb_metal_segment_*, bridge.h:72-183).  Operations
 * enqueued into a segment are recorded on the host; commit launches them as
 * one CUDA graph on the context stream without waiting (vtb_cuda_wait_idle
 * drains, as vtb_metal_wait_idle does).  The context keeps the graphs of the
 * last 8 distinct operation lists, so re-committing the same list (same
 * buffers, offsets and shapes, as a decode loop does every token) is one
 * graph launch.  One segment per context is open at a time; begin returns it
 * (NULL on a bad context).  Enqueue functions return nothing: the first bad
 * argument is reported by commit (and the segment is dropped).  Matmul
 * weights and activations must be 16-byte aligned.  Host buffers of the copy
 * functions should be pinned; with pageable memory commit runs the list
 * eagerly instead of as a graph.  The buffers a committed segment uses must
 * stay alive until it has finished. */
typedef struct VtbCudaSeg VtbCudaSeg;
VtbCudaSeg *vtb_cuda_segment_begin(VtbCudaCtx *ctx);
int vtb_cuda_segment_commit(VtbCudaSeg *seg);
void vtb_cuda_segment_matmul_q8_0(VtbCudaSeg *seg, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                                  VtbCudaBuf *acts_buf, size_t m, size_t k);
void vtb_cuda_segment_matmul_q4_k(VtbCudaSeg *seg, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                                  VtbCudaBuf *acts_buf, size_t m, size_t k);
void vtb_cuda_segment_matmul_q5_k(VtbCudaSeg *seg, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                                  VtbCudaBuf *acts_buf, size_t m, size_t k);
void vtb_cuda_segment_matmul_q6_k(VtbCudaSeg *seg, VtbCudaBuf *out_buf, VtbCudaBuf *w_buf, size_t w_offset,
                                  VtbCudaBuf *acts_buf, size_t m, size_t k);
/* f32 copy dst[dst_off..] = src[src_off..], n_floats values, byte offsets 4-aligned
 * (vtb_metal_segment_copy). */
void vtb_cuda_segment_copy(VtbCudaSeg *seg, VtbCudaBuf *dst_buf, size_t dst_offset_bytes, VtbCudaBuf *src_buf,
                           size_t src_offset_bytes, size_t n_floats);
/* Host <-> device copies inside a segment (Metal buffers are host-visible;
 * CUDA device buffers are not, so inputs go in and results come back here). */
void vtb_cuda_segment_copy_h2d(VtbCudaSeg *seg, VtbCudaBuf *dst_buf, size_t dst_offset, const void *host_src,
                               size_t bytes);
void vtb_cuda_segment_copy_d2h(VtbCudaSeg *seg, void *host_dst, VtbCudaBuf *src_buf, size_t src_offset, size_t bytes);

/* ------------------------------------------------------------------ */
/* Llama forward loop (the backend vtable, src/runtime/backend.zig:67-97) */
/* ------------------------------------------------------------------ */

/* LlamaConfig (src/runtime/model.zig:40-149), GGUF llama fields only. */
typedef struct {
  int32_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab_size, max_seq;
  float rope_base, rms_eps;
} VtbCudaLlamaConfig;

/* LayerWeights (model.zig:172-189): HOST pointers to each tensor's packed
 * bytes (e.g. into the GGUF mmap) and ggml type ids; norms are f32. */
typedef struct {
  const void *attn_q, *attn_k, *attn_v, *attn_o, *ffn_gate, *ffn_up, *ffn_down;
  const float *attn_norm, *ffn_norm;
  int32_t q_attn_q, q_attn_k, q_attn_v, q_attn_o, q_ffn_gate, q_ffn_up, q_ffn_down;
} VtbCudaLayerWeights;

typedef struct VtbCudaModel VtbCudaModel;
typedef struct VtbCudaState VtbCudaState;

/* Upload every weight once to the context's device (Model.init + the Metal
 * backend's initShards, model.zig:201-243, metal_backend.zig:134).  Q|K|V and
 * gate|up are row-concatenated when their quant types match (the reference's
 * -Dweight_fusion fuseRowConcat, model.zig:358-378).  Every projection must be
 * Q8_0/Q4_K/Q5_K/Q6_K: anything else is refused with NULL (no CPU fallback;
 * BackendUnsupportedQuant, backend.zig:61). */
VtbCudaModel *vtb_cuda_model_create(VtbCudaCtx *ctx, const VtbCudaLlamaConfig *cfg,
                                    const VtbCudaLayerWeights *layers, const void *token_embd,
                                    int32_t q_token_embd, const float *output_norm, const void *output_w,
                                    int32_t q_output);
void vtb_cuda_model_destroy(VtbCudaModel *m);
size_t vtb_cuda_model_weight_bytes(VtbCudaModel *m);
/* Dynamic activation quantization for Q8_0 weights: with on = 1, every Q8_0
 * projection of states created afterwards quantizes its activation row per
 * 32-block to Q8_0 (d = max|x|/127, round half away from zero) and runs the
 * Q8_0 x Q8_0 path -- exact int32 block dots (dot_i8, simd.zig:31-62) scaled
 * by d_w * d_x -- instead of the f32-activation matmul_q8_0 of matmulRuntime
 * (forward.zig:552-627).  Prefill rows of such projections run one row at a
 * time.  Other quant types are unaffected.  Default off. */
int vtb_cuda_model_set_q8_activations(VtbCudaModel *m, int on);

/* Per-session device state (forward.zig State :33-113 + KvCache kv_cache.zig:20-73):
 * n_seqs independent sequences decoded together (batch decode), and up to
 * max_rows rows per step (prefill chunk size). */
VtbCudaState *vtb_cuda_state_create(VtbCudaModel *m, int32_t n_seqs, int32_t max_rows);
void vtb_cuda_state_destroy(VtbCudaState *s);
/* KvCache.reset (kv_cache.zig:80). */
int vtb_cuda_state_reset(VtbCudaState *s);
/* KvCache.pos of sequence `seq` (host-authoritative). */
int64_t vtb_cuda_state_pos(VtbCudaState *s, int32_t seq);

/* 1 when this tensor-parallel state all-reduces over NVLink peer memory
 * (partials summed by the following RMSNorm kernel), 0 when it uses NCCL or
 * runs on one GPU.  No reference counterpart (the reference has no
 * multi-device code). */
int vtb_cuda_state_tp_p2p(const VtbCudaState *s);

/* The vtable, slot by slot.  begin_token is stepWithBackend's preamble
 * (token checks + gatherEmbedding, forward.zig:158-163) for one token per
 * sequence; layer_step / final_step / finalize_token are the VTable slots.
 * finalize_token copies logits ([n_seqs][vocab], may be NULL) and the
 * greedy argmax ([n_seqs], may be NULL) to the host and advances the cache. */
int vtb_cuda_begin_token(VtbCudaState *s, const int32_t *tokens);
int vtb_cuda_layer_step(VtbCudaState *s, int32_t layer);
int vtb_cuda_final_step(VtbCudaState *s);
int vtb_cuda_finalize_token(VtbCudaState *s, float *logits, int32_t *argmax);

/* One whole decode step for all sequences (stepWithBackend), replayed as a
 * CUDA graph captured on first use. */
int vtb_cuda_step(VtbCudaState *s, const int32_t *tokens, float *logits, int32_t *argmax);

/* Batched prompt prefill of one sequence (prefillCpu, src/runtime/prefill.zig:111-147):
 * advances the sequence by n; logits/argmax of the last token. */
int vtb_cuda_prefill(VtbCudaState *s, int32_t seq, const int32_t *tokens, int32_t n, float *logits,
                     int32_t *argmax);

/* ---- MLX affine quantization (src/kernels/mlx.zig) ----
 * w: [m][k / (32 / bits)] little-endian u32 words, 32 / bits values per word,
 * low bits first; scales, biases: [m][k / group_size] f16 (scale_is_bf16 = 0)
 * or bf16; weight = q * scale + bias.  bits in {2, 3, 4, 5, 6, 8}; group_size
 * divides k and is a multiple of 32 / bits.  w, scales and biases may sit at
 * any byte offset (safetensors shards); x must be 16-byte aligned.
 * vtb_cuda_gemv_mlx: y[m] = W . x (matmul, mlx.zig:213-235, fp32 accumulation). */
int vtb_cuda_gemv_mlx(const void *w, const void *scales, const void *biases, const float *x, float *y, int64_t m,
                      int64_t k, int bits, int group_size, int scale_is_bf16, void *stream);
/* out[rows][k] = dequantized rows, bit-exact with dequantRowDispatch (mlx.zig:261-279). */
int vtb_cuda_dequant_mlx(const void *w, const void *scales, const void *biases, float *out, int64_t rows, int64_t k,
                         int bits, int group_size, int scale_is_bf16, void *stream);
/* Bridge one-shot, same arguments as vtb_metal_matmul_mlx_q4 (src/metal/bridge.h:217-229):
 * weight, scales, biases and acts each as buffer + byte offset. */
int vtb_cuda_matmul_mlx_q4(struct VtbCudaCtx *ctx, struct VtbCudaBuf *out_buf, struct VtbCudaBuf *weight_buf,
                           size_t weight_offset, struct VtbCudaBuf *scales_buf, size_t scales_offset,
                           struct VtbCudaBuf *biases_buf, size_t biases_offset, struct VtbCudaBuf *acts_buf,
                           size_t acts_offset, size_t m, size_t k, uint32_t group_size, uint32_t scale_dtype_is_bf16);

/* ---- token sampling on the device (Sampler.sample, src/runtime/sampler.zig:44-104) ----
 * Same fields, meaning and layout as the reference's VtbSamplerConfig
 * (include/vantablack.h:46-51).  temperature 0 = greedy argmax; top_k 0 =
 * off; top_p 0 or >= 1 = off.  The PRNG stays with the caller: `u` holds one
 * uniform draw in [0, 1) per row (what prng.random().float(f32) returns at
 * sampler.zig:92), so `seed` is not read here.  Logits are rewritten in place
 * with the pipeline's probabilities, as the reference mutates them.  Tokens
 * equal the reference's for the same logits and draw unless the draw falls
 * within a few ulp of a cumulative-probability boundary (the sums are formed
 * in another order); argmax, the top-k cut and the nucleus set are exact.
 * Logits must be finite or -inf.  rows <= 256, n <= 2^24. */
typedef struct VtbCudaSamplerConfig {
  float temperature;
  size_t top_k;
  float top_p;
  uint64_t seed;
} VtbCudaSamplerConfig;

/* logits: device [rows][ld] f32 (first n of each row used), u: host [rows]
 * (may be NULL when temperature == 0), tokens: device [rows] int32. */
int vtb_cuda_sample(float *logits, int64_t rows, int64_t n, int64_t ld, const VtbCudaSamplerConfig *cfg,
                    const float *u, int32_t *tokens, void *stream);

/* Sample rows [0, rows) of the state's logits after vtb_cuda_step /
 * vtb_cuda_final_step (one row per sequence) or vtb_cuda_prefill (row 0),
 * and copy the rows' tokens to the host: 4 bytes per sequence cross PCIe
 * instead of the f32[vocab] row that finalize_token would copy for the
 * reference's host-side Sampler.sample (stream.zig:82, 96). */
int vtb_cuda_state_sample(VtbCudaState *s, int32_t rows, const VtbCudaSamplerConfig *cfg, const float *u,
                          int32_t *tokens);

/* ------------------------------------------------------------------ */
/* Tensor parallelism (NCCL over NVLink/NVSwitch; no counterpart in the   */
/* reference, which is single-device)                                   */
/* ------------------------------------------------------------------ */

#define VTB_CUDA_TP_ID_BYTES 128
typedef struct VtbCudaTp VtbCudaTp;

/* Rows and columns one rank owns: Q/K/V and gate/up by output rows, O and
 * down along K (head / ffn columns, whole quantization blocks), LM head by
 * vocabulary rows. */
typedef struct {
  int32_t heads, kv_heads;
  int32_t q_row0, q_rows, kv_row0, kv_rows, ffn_row0, ffn_rows;
  int32_t o_col0, o_cols, down_col0, down_cols, vocab_row0, vocab_rows;
} VtbCudaTpShard;

/* Rank 0 creates the communicator id and shares it with the other ranks
 * (any host channel); every rank then calls vtb_cuda_tp_init. */
int vtb_cuda_tp_unique_id(uint8_t *id_out /* VTB_CUDA_TP_ID_BYTES */);
VtbCudaTp *vtb_cuda_tp_init(int device, int rank, int world, const uint8_t *id);
void vtb_cuda_tp_destroy(VtbCudaTp *tp);
int vtb_cuda_tp_rank(const VtbCudaTp *tp);
int vtb_cuda_tp_world(const VtbCudaTp *tp);
/* Host-only helpers (no GPU needed): the shard plan, and a copy of a row x
 * column block of a quantized tensor (columns on block boundaries). */
int vtb_cuda_tp_shard_plan(const VtbCudaLlamaConfig *cfg, int rank, int world, int32_t k_block,
                           VtbCudaTpShard *out);
int vtb_cuda_tp_slice(int quant, const void *src, int64_t rows, int64_t k, int64_t row0, int64_t nrows,
                      int64_t col0, int64_t ncols, void *dst);
/* vtb_cuda_model_create for one rank of a tensor-parallel group: takes the
 * full host tensors and uploads this rank's shard; layer steps then
 * all-reduce after O and down and all-gather the logits.  tp = NULL is the
 * single-GPU model. */
VtbCudaModel *vtb_cuda_model_create_tp(VtbCudaCtx *ctx, VtbCudaTp *tp, const VtbCudaLlamaConfig *cfg,
                                       const VtbCudaLayerWeights *layers, const void *token_embd,
                                       int32_t q_token_embd, const float *output_norm, const void *output_w,
                                       int32_t q_output);

/* ---- GGUF files (src/core/parser.zig, src/core/mapper.zig; src/runtime/
 * model.zig LlamaConfig.fromCatalog and Model.init) ----
 * vtb_cuda_gguf_open maps the file read-only and parses the v2/v3 header,
 * the typed metadata and the tensor descriptors; tensor bytes stay in the
 * map (zero-copy) until a model upload reads them.  Errors: -2 open / map,
 * -3 malformed file (not GGUF, unsupported version, truncation, unknown
 * metadata type, arrays nested deeper than 4, element counts that overflow
 * or do not fill whole blocks, tensors outside the file). */
typedef struct VtbCudaGguf VtbCudaGguf;
#define VTB_CUDA_GGUF_MAX_DIMS 8
VtbCudaGguf *vtb_cuda_gguf_open(const char *path);
void vtb_cuda_gguf_close(VtbCudaGguf *g);
int vtb_cuda_gguf_info(const VtbCudaGguf *g, uint32_t *version, uint32_t *alignment, uint64_t *data_offset,
                       int64_t *n_tensors, int64_t *n_meta);
/* Descriptor i (file order): name (NUL-terminated, owned by g), ggml type id,
 * dims (ne0 = innermost; up to VTB_CUDA_GGUF_MAX_DIMS written), offset from
 * the data segment and byte size (0 for types without a known block size). */
int vtb_cuda_gguf_tensor_info(const VtbCudaGguf *g, int64_t i, const char **name, uint32_t *ggml_type,
                              uint32_t *n_dims, uint64_t *dims, uint64_t *rel_offset, uint64_t *size_bytes);
/* Bounds-checked pointer to a tensor's bytes inside the map (tensorSlice). */
const void *vtb_cuda_gguf_tensor(const VtbCudaGguf *g, const char *name, uint32_t *ggml_type,
                                 uint64_t *size_bytes);
int vtb_cuda_gguf_meta_int(const VtbCudaGguf *g, const char *key, int64_t *out);
int vtb_cuda_gguf_meta_float(const VtbCudaGguf *g, const char *key, double *out);
int vtb_cuda_gguf_meta_string(const VtbCudaGguf *g, const char *key, const char **ptr, uint64_t *len);
int vtb_cuda_gguf_meta_array(const VtbCudaGguf *g, const char *key, uint32_t *elem_type, uint64_t *count);
/* The Llama configuration from `llama.*` metadata (head_count_kv defaults to
 * head_count, rope.freq_base to 10000, layer_norm_rms_epsilon to 1e-5, the
 * vocabulary to the token list's length); other architectures: -8. */
int vtb_cuda_gguf_llama_config(const VtbCudaGguf *g, VtbCudaLlamaConfig *cfg);
/* Model.init + upload: blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,
 * ffn_norm,ffn_gate,ffn_up,ffn_down}.weight, token_embd.weight,
 * output_norm.weight, output.weight (absent: tied to token_embd).  Shapes and
 * types are checked (norms f32; projections Q8_0/Q4_K/Q5_K/Q6_K).  max_seq > 0
 * replaces the file's context_length (it sizes every state's KV cache).  The
 * file may be closed once the model exists. */
VtbCudaModel *vtb_cuda_model_create_gguf(VtbCudaCtx *ctx, const VtbCudaGguf *g, int32_t max_seq);
VtbCudaModel *vtb_cuda_model_create_gguf_tp(VtbCudaCtx *ctx, VtbCudaTp *tp, const VtbCudaGguf *g, int32_t max_seq);

#ifdef __cplusplus
}
#endif
#endif /* VTB_CUDA_H */
