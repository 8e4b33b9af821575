/*
 * oracle_moe.c -- CPU oracle of the mixture-of-experts block (test
 * infrastructure only; the checker for the CUDA library).
 *
 * The reference has no MoE; this restates the semantics the CUDA library
 * defines (include/opencuda_cuda.h), built from the reference's own
 * routines: every expert and the shared expert is an MLP fc -> gelu_new ->
 * proj (the reference's GPT MLP, crates/open-cuda-llm/src/lib.rs:400-403)
 * whose Linears are W8A8 quantized matmuls (ocr_qgemm_w8a8: activations
 * quantized per row with quantize_int8, exact int32 products), no biases.
 *   route:   top-k of the router logits, ties to the lower expert index,
 *            NaN never selected; w = softmax of the k selected logits:
 *            e_i = (float)exp((double)(l_i - l_max)) (f64 exp rounded to
 *            f32, so any correctly-rounding-to-1-ulp exp agrees), summed in
 *            selection order, then divided; if every selected logit is
 *            -inf (or NaN) the weights are 1/k
 *   combine: y = shared(x); for i < k: y = y + w_i * expert_{e_i}(x)
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

int ocr_moe_route(const float *logits, size_t T, size_t E, size_t k, int32_t *idx, float *w) {
  if (k == 0 || k > E) return 1;
  unsigned char *taken = (unsigned char *)malloc(E);
  float *sv = (float *)malloc(k * sizeof(float));
  if (!taken || !sv) {
    free(taken);
    free(sv);
    return 2;
  }
  for (size_t t = 0; t < T; t++) {
    const float *l = logits + t * E;
    memset(taken, 0, E);
    for (size_t s = 0; s < k; s++) {
      float bv = -INFINITY;
      size_t bi = (size_t)-1;
      for (size_t e = 0; e < E; e++) {
        if (taken[e]) continue;
        float v = isnan(l[e]) ? -INFINITY : l[e];
        if (bi == (size_t)-1 || v > bv) {
          bv = v;
          bi = e;
        }
      }
      taken[bi] = 1;
      idx[t * k + s] = (int32_t)bi;
      sv[s] = bv;
    }
    float sum = 0.0f;
    float *e = w + t * k;
    if (sv[0] == -INFINITY) {
      for (size_t s = 0; s < k; s++) e[s] = 1.0f / (float)k;
      continue;
    }
    for (size_t s = 0; s < k; s++) {
      e[s] = (float)exp((double)(sv[s] - sv[0]));
      sum += e[s];
    }
    for (size_t s = 0; s < k; s++) e[s] = e[s] / sum;
  }
  free(taken);
  free(sv);
  return 0;
}

/* One expert MLP on one row: out[D] = proj(gelu(fc(x))). */
static int expert_row(size_t D, size_t F, const float *x, const int8_t *w1, const float *s1, const int8_t *w2,
                      const float *s2, float *h, float *out) {
  int rc = ocr_qgemm_w8a8(1, D, F, x, w1, s1, NULL, h, NULL);
  if (rc) return rc;
  ocr_gelu(h, F);
  return ocr_qgemm_w8a8(1, F, D, h, w2, s2, NULL, out, NULL);
}

int ocr_moe_forward(size_t T, size_t D, size_t F, size_t E, size_t k, const float *x, const float *logits,
                    const int8_t *w1, const float *s1, const int8_t *w2, const float *s2, const int8_t *sw1,
                    const float *ss1, const int8_t *sw2, const float *ss2, float *y) {
  int32_t *idx = (int32_t *)malloc(T * k * sizeof(int32_t));
  float *w = (float *)malloc(T * k * sizeof(float));
  float *h = (float *)malloc(F * sizeof(float));
  float *o = (float *)malloc(D * sizeof(float));
  int rc = 0;
  if (!idx || !w || !h || !o) {
    rc = 2;
    goto out;
  }
  if ((rc = ocr_moe_route(logits, T, E, k, idx, w))) goto out;
  for (size_t t = 0; t < T; t++) {
    const float *xr = x + t * D;
    float *yr = y + t * D;
    if ((rc = expert_row(D, F, xr, sw1, ss1, sw2, ss2, h, yr))) goto out;
    for (size_t s = 0; s < k; s++) {
      size_t e = (size_t)idx[t * k + s];
      if ((rc = expert_row(D, F, xr, w1 + e * F * D, s1 + e * F, w2 + e * D * F, s2 + e * D, h, o))) goto out;
      const float ws = w[t * k + s];
      for (size_t c = 0; c < D; c++) yr[c] = yr[c] + ws * o[c];
    }
  }
out:
  free(idx);
  free(w);
  free(h);
  free(o);
  return rc;
}
