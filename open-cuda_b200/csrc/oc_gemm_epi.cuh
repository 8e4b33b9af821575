// oc_gemm_epi.cuh -- epilogues of the f32 (3xTF32) GEMM for the GPT linears,
// applied where the GEMM's sums are finished (the GEMM's own epilogue, or
// the split-K reduction).  With v = alpha * acc and b = bias[col]:
//   kGemmEpiPlain     C = v (+ beta * C) + b          (sgemm, blas:200-214)
//   kGemmEpiGelu      C = gelu_new(v + b)             (fc, llm:400-402)
//   kGemmEpiResidual  C = C + (v + b)                 (residual adds, llm:396, 404)
//   kGemmEpiQkv       C = v + b, and the k / v thirds of the row also go to
//                     the KV cache at the row's position (llm:568-590)
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace oc {

enum GemmEpiMode { kGemmEpiPlain = 0, kGemmEpiGelu = 1, kGemmEpiResidual = 2, kGemmEpiQkv = 3 };

struct GemmEpi {
  int mode = kGemmEpiPlain;
  float* kc = nullptr;  // kGemmEpiQkv: caches [batch][max_seq][H]
  float* vc = nullptr;
  const int* pos = nullptr;  // position of row i of each sequence = *pos + i
  int L = 1, H = 0, max_seq = 0;
};

// gelu_new in f64, cast to f32 (llm:268-275).
__device__ __forceinline__ float gelu_new_f64(float v) {
  const double xf = (double)v;
  const double inner = 0.7978845608028654 * (xf + 0.044715 * (xf * xf * xf));
  return (float)(0.5 * xf * (1.0 + tanh(inner)));
}

// The finished value of element (row, col) whose current output is *cp.
__device__ __forceinline__ float gemm_epi_value(const GemmEpi& e, float v, float beta, float b, const float* cp) {
  switch (e.mode) {
    case kGemmEpiGelu:
      return gelu_new_f64(__fadd_rn(v, b));
    case kGemmEpiResidual:
      return __fadd_rn(*cp, __fadd_rn(v, b));
    case kGemmEpiQkv:
      return __fadd_rn(v, b);
    default:
      if (beta != 0.0f) v = __fadd_rn(v, __fmul_rn(beta, *cp));
      return __fadd_rn(v, b);
  }
}

// kGemmEpiQkv: the k / v columns of a finished qkv row into the caches.
__device__ __forceinline__ void gemm_epi_kv(const GemmEpi& e, int row, int col, float y) {
  if (e.mode != kGemmEpiQkv || col < e.H) return;
  const int b = row / e.L, i = row % e.L;
  const size_t slot = ((size_t)b * e.max_seq + *e.pos + i) * e.H;
  if (col < 2 * e.H) e.kc[slot + col - e.H] = y;
  else e.vc[slot + col - 2 * e.H] = y;
}

// C = epilogue(A . B) through the 3xTF32 GEMM, B prepared by
// oc_sgemm_prepare_b (oc_sgemm.cu).
int sgemm_prepared_epi(int m, int n, int k, const float* A, int lda, const float* prepared, float* C, int ldc,
                       const float* bias, const GemmEpi& epi, cudaStream_t s);

}  // namespace oc
