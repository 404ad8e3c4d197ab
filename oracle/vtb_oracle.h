/*
 * vtb_oracle.h -- CPU restatement of vantablack's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * backend is compared against (and the timed CPU baseline in bench.py).  It
 * is never linked into, loaded by, or called from the product library
 * (vantablack_b200/libvtbcuda.so).
 *
 * Every function restates one function of the reference (Zig 0.16 sources,
 * paths relative to the reference project root) with the same arithmetic
 * order, so that results are bit-identical to the reference's CPU kernels
 * when both are compiled without FP contraction (the reference's default
 * "strict" float mode; this file is built with -ffp-contract=off).
 *
 * Parity pin: the reference cannot be compiled in this environment (no Zig
 * toolchain), so the restatement is pinned by (1) the reference's own
 * known-answer tests in src/kernels/simd.zig:500-806 and
 * src/kernels/math.zig:205-254, ported to tests/test_oracle_kat.py, and
 * (2) bit-exact agreement of every dequantizer with gguf-py's independent
 * numpy implementation of the same ggml block formats (fixtures under
 * tests/golden/).
 */
#ifndef VTB_ORACLE_H
#define VTB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, as used by GGUF (src/core/parser.zig GgmlType). */
enum {
    VTBO_F32 = 0,
    VTBO_Q8_0 = 8,
    VTBO_Q4_K = 12,
    VTBO_Q5_K = 13,
    VTBO_Q6_K = 14,
    VTBO_TQ2_0 = 32, /* the reference's GgmlType id (parser.zig:62) */
};

float vtbo_f16_to_f32(uint16_t bits);
float vtbo_dot_f32(const float *a, const float *b, size_t n);
int32_t vtbo_dot_i8(const int8_t *a, const int8_t *b, size_t n);

void vtbo_dequant_q8_0_block(const uint8_t *blk, float *out32);
void vtbo_dequant_q4_k_block(const uint8_t *blk, float *out256);
void vtbo_dequant_q5_k_block(const uint8_t *blk, float *out256);
void vtbo_dequant_q6_k_block(const uint8_t *blk, float *out256);
void vtbo_dequant_tq2_0_block(const uint8_t *blk, float *out256);
/* Dequantize n elements (a whole number of blocks) of type `quant`. */
int vtbo_dequant(int quant, const uint8_t *w, float *out, size_t n);

size_t vtbo_row_bytes(int quant, size_t k);

/* Single-threaded GEMV kernels: out[m] = W[m,k] . acts[k]. */
void vtbo_matmul_q8_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);
void vtbo_matmul_q4_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);
void vtbo_matmul_q5_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);
void vtbo_matmul_q6_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);
void vtbo_matmul_tq2_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);

/* Thread pool with the reference's row striping (chunk = ceil(m/n)). */
int vtbo_pool_init(int n_threads);
int vtbo_pool_threads(void);
void vtbo_pool_shutdown(void);

/* Row-striped GEMV through the pool (forward.zig matmulRuntime). */
int vtbo_matmul(int quant, float *out, const uint8_t *w, const float *acts, size_t m, size_t k);
/* Prefill batched matmul: out[B,m] = acts[B,k] . W^T (prefill.zig matmulBatched). */
int vtbo_matmul_batched(int quant, float *out, const uint8_t *w, const float *acts,
                        size_t m, size_t k, size_t B);

/* Q8_0 x Q8_0 path (activation quantizer defined here; the reference has none). */
void vtbo_quantize_q8_0(const float *x, size_t k, int8_t *qs, float *d);
void vtbo_q8_0_block_dots(int32_t *dots, const uint8_t *w, const int8_t *xq, size_t m, size_t k);
int vtbo_matmul_q8_0_q8_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k);

/* math.zig */
void vtbo_rms_norm(float *x, const float *w, size_t n, float eps);
void vtbo_rope(float *x, size_t head_dim, size_t pos, float base);
void vtbo_softmax(float *x, size_t n);
void vtbo_swiglu(float *gate, const float *up, size_t n);
void vtbo_geglu(float *gate, const float *up, size_t n);
void vtbo_add_into(float *a, const float *b, size_t n);
size_t vtbo_argmax(const float *x, size_t n);
/* Sampler.sample (sampler.zig:44-104) with the uniform draw u in [0, 1) supplied. */
uint32_t vtbo_sample(float *logits, size_t n, float temperature, size_t top_k, float top_p, float u);
/* MLX affine quantization (mlx.zig): dequantRow for `rows` rows, and matmul. bits in {2,3,4,5,6,8};
 * bf16 != 0: scales/biases are bf16, else f16.  Return -1 on unsupported arguments. */
int vtbo_mlx_dequant(float *out, const uint8_t *w, const uint8_t *scales, const uint8_t *biases, size_t rows,
                     size_t k, unsigned bits, size_t group, int bf16);
int vtbo_mlx_matmul(float *out, const uint8_t *w, const uint8_t *scales, const uint8_t *biases, const float *x,
                    size_t m, size_t k, unsigned bits, size_t group, int bf16);

/* Llama forward (forward.zig / prefill.zig / kv_cache.zig). */
typedef struct {
    int64_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab_size, max_seq;
    float rope_base, rms_eps;
} vtbo_config;

typedef struct {
    const uint8_t *attn_q, *attn_k, *attn_v, *attn_o, *ffn_gate, *ffn_up, *ffn_down;
    const float *attn_norm, *ffn_norm;
    int q_attn_q, q_attn_k, q_attn_v, q_attn_o, q_ffn_gate, q_ffn_up, q_ffn_down;
} vtbo_layer;

typedef struct vtbo_model vtbo_model;

vtbo_model *vtbo_model_create(const vtbo_config *c, const vtbo_layer *layers,
                              const uint8_t *token_embd, int q_token_embd,
                              const float *output_norm,
                              const uint8_t *output_w, int q_output);
void vtbo_model_destroy(vtbo_model *m);
/* Q8_0 projections take Q8_0-quantized activations (the Q8_0 x Q8_0 path). */
void vtbo_model_set_q8_activations(vtbo_model *m, int on);
void vtbo_model_reset(vtbo_model *m);
int64_t vtbo_model_pos(const vtbo_model *m);
/* One token through stepWithBackend + CpuBackend; logits written to `logits`. */
int vtbo_step(vtbo_model *m, uint32_t token, float *logits);
/* prefillCpu over B tokens; the last token's logits written to `logits`. */
int vtbo_prefill(vtbo_model *m, const uint32_t *tokens, size_t B, float *logits);
/* Read back the KV cache of one layer ([max_seq][n_kv_heads*head_dim] f32). */
const float *vtbo_kv_keys(const vtbo_model *m, size_t layer);
const float *vtbo_kv_values(const vtbo_model *m, size_t layer);

#ifdef __cplusplus
}
#endif
#endif
