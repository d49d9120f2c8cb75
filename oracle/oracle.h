/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of synapse's CPU decode path (branes-ai/synapse
 * v0.15.12, header-only C++20), used as the parity checker for the CUDA
 * implementation in synapse_b200/. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it. The product never links it.
 *
 * The reference itself cannot be compiled here: every kernel header includes
 * MTL5 v5.20.0 (an external library absent from the image), so this file
 * restates the algorithms in the reference's portable scalar configuration
 * (one SIMD lane), citing the reference line each function follows.
 *
 * Pinned against the reference's own golden fixtures (tests/golden/, made by
 * tests/golden/make_golden.py from the reference's tests/data GGUF files):
 *   - kernel_golden.gguf: Q4_0/Q8_0 activations bit-identical, gemv y within
 *     1e-5 of ggml's vec_dot;
 *   - kernel_golden.gguf: Q4_K/Q6_K on Q8_K activations, the same checks;
 *   - quant_golden.gguf: Q4_0/Q8_0/F16/Q4_K/Q6_K dequantizers bit-identical;
 *   - llama_tiny_f32(_golden).gguf: 16 decode steps of logits within 1e-4
 *     relative max of llama.cpp (RoPE with frequency factors, GQA, F16 KV
 *     cache, softmax, RMSNorm, residuals, tied F32 head);
 *   - the reference's known answers (Q8_0 quantizer, fp16 rounding, GQA
 *     attention against a double reference, pos 0 == V).
 */
#ifndef SYNAPSE_ORACLE_H
#define SYNAPSE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type tags (ggml_type values), as in the reference's
 * gguf/tensor_type.hpp:25-46. */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14 };

#define ORC_QK 32
#define ORC_QK_K 256

typedef struct { uint16_t d; uint8_t qs[16]; } orc_block_q4_0;   /* 18 B */
typedef struct { uint16_t d; int8_t qs[32]; } orc_block_q8_0;    /* 34 B */
/* quant/blocks.hpp:56-70 and quant/q8.hpp:33-38 */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } orc_block_q4_k;           /* 144 B */
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } orc_block_q6_k;  /* 210 B */
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } orc_block_q8_k;                     /* 292 B */

/* numeric/half.hpp */
float orc_fp16_to_float(uint16_t h);
uint16_t orc_float_to_fp16(float f);

/* quant/q8.hpp, quant/blocks.hpp */
void orc_quantize_row_q8_0(const float* x, size_t n, orc_block_q8_0* y);
void orc_quantize_row_q4_0(const float* x, size_t n, orc_block_q4_0* y);
void orc_quantize_row_q8_k(const float* x, size_t n, orc_block_q8_k* y);
void orc_dequantize_row(int type, const void* row, size_t n, float* y);
size_t orc_row_bytes(int type, size_t cols);

/* kernels/gemv.hpp + kernels/dot.hpp: y = W x with x quantized to Q8_0 once
 * (quantized formats) or kept float (F32/F16). */
void orc_gemv(int type, const void* w, size_t rows, size_t cols, const float* x, float* y);
/* The same product on already-quantized activations (cols/32 blocks). */
void orc_gemv_q8act(int type, const void* w, size_t rows, size_t cols, const orc_block_q8_0* act, float* y);
/* Q4_K / Q6_K rows on Q8_K activations (cols/256 blocks). */
void orc_gemv_q8k(int type, const void* w, size_t rows, size_t cols, const orc_block_q8_k* act, float* y);
/* kernels/gemm.hpp: Y[n x rows] = X[n x cols] W^T, each row as orc_gemv (G1). */
void orc_gemm(int type, const void* w, size_t rows, size_t cols, const float* x, size_t n, float* y);

/* kernels/attention.hpp */
float orc_rope_theta_scale(float base, size_t head_dim);
typedef struct {
    float freq_scale, ext_factor, attn_factor, corr_low, corr_high;
} orc_rope_scaling;
void orc_rope(const float* x, float* out, size_t n, size_t head_dim, uint32_t pos, float theta_scale,
              const float* freq_factors /* NULL or head_dim/2 */, int neox, const orc_rope_scaling* scaling);
void orc_kv_append(const float* k, const float* v, uint16_t* kc, uint16_t* vc, size_t max_ctx, size_t n_kv,
                   size_t head_dim, uint32_t pos);
void orc_attend_group(const float* q, const uint16_t* kc, const uint16_t* vc, size_t max_ctx, size_t n_kv,
                      size_t head_dim, uint32_t pos, size_t n_heads, float scale, float* out, float* scratch,
                      size_t g);
size_t orc_attention_group_floats(size_t n_heads, size_t n_kv, size_t head_dim, size_t max_ctx);
/* kv_append then every group; scratch holds n_kv * orc_attention_group_floats floats. */
void orc_attention(const float* q, const float* k, const float* v, uint16_t* kc, uint16_t* vc, size_t max_ctx,
                   size_t n_kv, size_t head_dim, uint32_t pos, size_t n_heads, float scale, float* out,
                   float* scratch);

/* kernels/elementwise.hpp */
void orc_expf(const float* x, float* y, size_t n);
void orc_softmax(const float* x, float* out, size_t n);
void orc_rms_norm(const float* x, const float* gamma, float eps, float* out, size_t n);
void orc_silu(const float* x, float* out, size_t n);
void orc_mul(const float* a, const float* b, float* out, size_t n);
void orc_add(const float* a, const float* b, float* out, size_t n);

/* models/llama.hpp + graph/session.hpp: the Llama decode graph, run one token
 * at a time. Weights are borrowed host pointers (GGUF row-major bytes). */
typedef struct {
    size_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, max_ctx;
    float rms_eps, rope_base;
} orc_llama_config;

typedef struct {
    int type;
    const void* data;
} orc_tensor;

typedef struct {
    orc_tensor attn_norm, wq, wk, wv, wo, ffn_norm, gate, up, down;
} orc_layer;

typedef struct orc_llama orc_llama;
/* layers: n_layer entries; output.data == NULL means tied to token_embd;
 * freq_factors NULL or head_dim/2 floats. Norm weights must be F32. */
orc_llama* orc_llama_create(const orc_llama_config* c, orc_tensor token_embd, orc_tensor output_norm,
                            orc_tensor output, const orc_layer* layers, const float* freq_factors);
void orc_llama_destroy(orc_llama* m);
void orc_llama_reset(orc_llama* m);
/* Decode one token at pos (positions 0..pos-1 already run); logits: n_vocab. */
int orc_llama_step(orc_llama* m, uint32_t token, uint32_t pos, float* logits);
/* Part of a step, for bounded CPU timing samples: optionally the embedding of
 * `token`, then layers [l0, l1) on the running hidden state, then (logits
 * non-NULL) the final norm and head. */
int orc_llama_run(orc_llama* m, uint32_t token, uint32_t pos, size_t l0, size_t l1, int embed, float* logits);
/* Direct access to the KV cache of a layer (for tests): K then V, each max_ctx*n_kv*hd halves. */
uint16_t* orc_llama_kcache(orc_llama* m, size_t layer);
uint16_t* orc_llama_vcache(orc_llama* m, size_t layer);

/* Seeded N(0, sigma) weights (splitmix64 counters, Box-Muller) in `type`
 * (GGUF bytes; F32 as floats), rows x cols, on the oracle's threads. For
 * synthetic CPU-baseline models only. */
void orc_fill_random(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tensor, float sigma, void* out);

/* Threads the oracle may use (pthreads); results do not depend on it. */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
