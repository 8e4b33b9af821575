/*
 * oracle.h -- CPU restatement of the open-cuda reference's hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * library (libopencuda_cuda.so) and the timed CPU baseline; it is never
 * linked into, loaded by, or called from the product path.
 *
 * Every function restates a loop of the reference (Rust) crate with the same
 * per-element arithmetic order, so results are bit-identical to what the
 * reference's CPU (rayon) backend computes:
 *   crates/opencuda-blas/src/lib.rs   ("blas")
 *   crates/open-cuda-llm/src/lib.rs   ("llm")
 *   crates/opencuda-cpu/src/lib.rs    ("cpu")
 * Compile with -ffp-contract=off: Rust never contracts a*b+c into an FMA.
 *
 * Return convention: 0 = ok, nonzero = the reference's `bail!` cases
 * (dimension mismatch, zero group size, empty input, ...).
 */
#ifndef OC_ORACLE_H
#define OC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Worker threads used by the parallel loops (0 = all online cores). */
void ocr_set_threads(int n);
int ocr_get_threads(void);

/* ---- GEMM (blas:148-237, blas:260-295) -------------------------------- */
/* C = alpha*A*B + beta*C, row-major.  transpose_b: B is n x k (blas:206-210).
 * faithful=1 restates the reference's execution literally: one output
 * element per task, blocks of 256 elements spread over the workers
 * (cpu:191-213, blas:218), strided B reads, plus the per-call scoped
 * allocation and host<->"device" copies of A, B and C (blas:174-181,233).
 * faithful=0 computes the same per-element expression (ascending-k f32
 * sum, then alpha*acc + beta*c) with a cache-friendly loop order; the
 * results are bit-identical. */
int ocr_sgemm(size_t m, size_t k, size_t n, float alpha, const float *a,
              const float *b, int transpose_b, float beta, float *c,
              int faithful);

/* ---- quantization (blas:777-1012) -------------------------------------- */
void ocr_group_scales(const float *in, size_t len, size_t group, float qmax,
                      float *scales);
void ocr_quantize_symmetric(const float *in, size_t len, const float *scales,
                            size_t group, float qmin, float qmax, int8_t *out);
int ocr_quantize_int8(const float *in, size_t len, size_t group, int8_t *data,
                      float *scales);
int ocr_quantize_int4(const float *in, size_t len, size_t group, uint8_t *data,
                      float *scales);
void ocr_dequantize_int8(const int8_t *data, const float *scales, size_t len,
                         size_t group, float *out);
void ocr_dequantize_int4(const uint8_t *data, const float *scales, size_t len,
                         size_t group, float *out);
int ocr_quantize_int4_awq(const float *weight, size_t rows, size_t cols,
                          const float *act_scale, size_t group, float alpha,
                          uint8_t *data, float *scales, float *awq_scale);
void ocr_dequantize_int4_awq(const uint8_t *data, const float *scales,
                             size_t rows, size_t cols, size_t group,
                             const float *awq_scale, float *out);

/* ---- attention (blas:411-678) ------------------------------------------ */
void ocr_row_softmax(const float *scores, size_t rows, size_t cols,
                     float *probs);
int ocr_sdpa(const float *q, const float *k, const float *v, size_t seq,
             size_t d, float *out);
int ocr_flash_attention(const float *q, const float *k, const float *v,
                        size_t seq, size_t d, size_t block, float *out);
/* One query row against n cached rows: row 0 of the reference's decode
 * attention, which replicates q n times and keeps row 0 (llm:358-387).
 * Each query row is computed independently there, so row 0 alone is
 * bit-identical.  flash=1: blas:589-678 with `block`; flash=0: the
 * unfused SDPA path (blas:475-540). */
void ocr_attend_one(const float *q, const float *k, const float *v, size_t n,
                    size_t d, int flash, size_t block, float *out);

/* ---- MLA (blas:1045-1078) ------------------------------------------------ */
int ocr_mla_compress_kv(size_t seq, size_t d_h, size_t d_c, const float *kv,
                        const float *down, float *latent);
int ocr_mla_decompress_kv(size_t seq, size_t d_c, size_t d_h,
                          const float *latent, const float *up, float *out);
double ocr_mla_memory_reduction_percent(size_t d_h, size_t d_c);

/* ---- quantized matmul oracles (new API; composed from the reference) ----
 * Weight layout: W^T flattened [n][k] and quantized by the reference's own
 * routine (per-output-channel: group = k; INT4: group = 32).
 *
 * W8A8 exact: A is quantized per row by quantize_int8(A, group=k); the
 * accumulator acc[m][n] = sum_k qa*qw is exact int32 and
 *   y = ((float)acc * sa[m]) * sw[n] + bias[n]      (no FMA)
 * W4A8 exact (group g over k): P[m][n][j] = sum_{k in group j} qa*qw exact,
 *   s = 0; for j ascending: s = fmaf((float)P, sw[n][j], s);
 *   y = s * sa[m] + bias[n]                          (mul, then add)
 * acc_out (optional, may be NULL): W8A8 -> [m][n] int32,
 *   W4A8 -> [m][n][k/g] int32 partials. */
int ocr_quantize_rows_int8(const float *a, size_t m, size_t k, int8_t *qa,
                           float *sa);
int ocr_qgemm_w8a8(size_t m, size_t k, size_t n, const float *a,
                   const int8_t *wq, const float *wscale, const float *bias,
                   float *y, int32_t *acc_out);
int ocr_qgemm_w4a8(size_t m, size_t k, size_t n, size_t group, const float *a,
                   const uint8_t *wq, const float *wscale, const float *bias,
                   float *y, int32_t *acc_out);
/* Weight-only: y = sgemm(A, dequantize(W)^T) + bias (llm:227-238 with a
 * dequantized weight), f32 activations. bits = 8 or 4. */
int ocr_qgemm_weight_only(int bits, size_t m, size_t k, size_t n,
                          size_t group, const float *a, const void *wq,
                          const float *wscale, const float *bias, float *y,
                          int faithful);

/* ---- mixture of experts (oracle_moe.c; no reference counterpart) -------- */
int ocr_moe_route(const float *logits, size_t T, size_t E, size_t k, int32_t *idx, float *w);
/* x [T][D], logits [T][E]; expert e: w1 [E][F][D] (scales s1 [E][F]),
 * w2 [E][D][F] (s2 [E][D]); shared expert sw1 [F][D], sw2 [D][F]. */
int ocr_moe_forward(size_t T, size_t D, size_t F, size_t E, size_t k, const float *x, const float *logits,
                    const int8_t *w1, const float *s1, const int8_t *w2, const float *s2, const int8_t *sw1,
                    const float *ss1, const int8_t *sw2, const float *ss2, float *y);

/* ---- GPT decoder (llm:45-942) -------------------------------------------- */
typedef struct ocr_gpt ocr_gpt;
typedef struct {
  size_t vocab_size, hidden_size, num_layers, num_heads, intermediate_size,
      max_seq_len;
  float layer_norm_eps;
} ocr_gpt_config;

/* SplitMix64 (llm:178-206) */
uint64_t ocr_splitmix64_next(uint64_t *state);
float ocr_splitmix64_next_f32(uint64_t *state, float scale);
void ocr_splitmix64_fill(uint64_t seed, float scale, size_t len, float *out);

/* load_random (llm:635-646): draw order wte, wpe, per layer qkv, attn_out,
 * fc, proj, then the untied lm_head. */
ocr_gpt *ocr_gpt_load_random(const ocr_gpt_config *cfg, uint64_t seed);
void ocr_gpt_free(ocr_gpt *m);
/* Attention mode: flash=1 uses flash_attention(block) (the fused slot),
 * flash=0 the unfused SDPA path.  faithful=1 replicates q n times and
 * computes all n rows, and runs every Linear through faithful sgemm, as the
 * reference does (for timing); faithful=0 computes row 0 only (same bits). */
void ocr_gpt_set_attention(ocr_gpt *m, int flash, size_t block, int faithful);
/* enable_mla_kv_compression (llm:822-838) */
int ocr_gpt_enable_mla(ocr_gpt *m, size_t d_c, uint64_t seed);
/* Weight views (row-major as stored by the reference, weight_t = in x out).
 * which: 0 wte, 1 wpe, 2 qkv_w, 3 qkv_b, 4 attn_out_w, 5 attn_out_b,
 * 6 fc_w, 7 fc_b, 8 proj_w, 9 proj_b, 10 ln1_w, 11 ln1_b, 12 ln2_w,
 * 13 ln2_b, 14 lnf_w, 15 lnf_b, 16 lm_head_w, 17 lm_head_b,
 * 18 mla_down (layer, head via *len in/out), 19 mla_up */
const float *ocr_gpt_weight(const ocr_gpt *m, int which, size_t layer,
                            size_t head, size_t *len);
/* KV cache session */
typedef struct ocr_gpt_state ocr_gpt_state;
ocr_gpt_state *ocr_gpt_state_new(const ocr_gpt *m);
void ocr_gpt_state_free(ocr_gpt_state *s);
/* GptModel::forward_step (llm:846-864): logits[vocab] */
int ocr_gpt_forward_step(const ocr_gpt *m, ocr_gpt_state *s, uint32_t token,
                         size_t pos, float *logits);
/* forward_prefill_all_layers (llm:869-899) */
int ocr_gpt_forward_prefill(const ocr_gpt *m, ocr_gpt_state *s,
                            const uint32_t *ids, size_t len, float *logits);
/* generate (llm:910-929); returns the number of tokens written (<= max_new)
 * or -1 on error.  logits_out (optional): [max_new][vocab], the logits each
 * generated token was taken from. */
long ocr_gpt_generate(const ocr_gpt *m, const uint32_t *prompt, size_t len,
                      size_t max_new, uint32_t *out, float *logits_out);
/* argmax, first maximum wins (llm:932-942) */
uint32_t ocr_argmax(const float *x, size_t n);
/* LayerNorm (llm:252-262) and gelu_new (llm:268-275), exposed for tests. */
void ocr_layer_norm(float *x, size_t rows, size_t dim, const float *w,
                    const float *b, float eps);
void ocr_gelu(float *x, size_t n);

#ifdef __cplusplus
}
#endif
#endif
