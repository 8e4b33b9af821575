/*
 * opencuda_cuda.h -- C ABI of libopencuda_cuda.so, the B200 (sm_100a)
 * backend for the open-cuda workspace's matmul / attention hot path.
 *
 * Each entry point names the reference interface it replaces (paths are
 * relative to the open-cuda workspace):
 *   core  = crates/opencuda-core/src/device.rs  (the GpuDevice trait)
 *   blas  = crates/opencuda-blas/src/lib.rs
 *   llm   = crates/open-cuda-llm/src/lib.rs
 *
 * Conventions
 *  - Every function returns an int status: 0 on success, otherwise one of
 *    the OC_ERR_* codes.  The codes of GpuError::to_cuda_code
 *    (crates/opencuda-core/src/error.rs:39-48) are kept: 1 invalid
 *    value/pointer, 2 out of memory, 8 launch failure/unsupported kernel,
 *    100 no device.  oc_get_last_error() returns this thread's message.
 *  - No function calls exit/abort or traps on the device.
 *  - Device-pointer entry points (oc_sgemm, oc_qgemm_*, ...) take raw CUDA
 *    device addresses and a cudaStream_t passed as void*; they are
 *    asynchronous on that stream.  Host-slice entry points (oc_blas_*)
 *    mirror the reference's blas signatures on host memory: they copy the
 *    inputs to the device, launch, copy the result back and synchronize.
 *  - Matrices are row-major and densely packed unless a leading dimension
 *    is given.
 */
#ifndef OPENCUDA_CUDA_H
#define OPENCUDA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OC_OK 0
#define OC_ERR_INVALID_VALUE 1   /* GpuError::InvalidPtr / bad shapes */
#define OC_ERR_OUT_OF_MEMORY 2   /* GpuError::OutOfMemory */
#define OC_ERR_LAUNCH_FAILED 8   /* GpuError::LaunchFailed / UnsupportedKernel */
#define OC_ERR_NO_DEVICE 100     /* GpuError::NoDevice */
#define OC_ERR_NOT_SUPPORTED 801 /* shape or device not handled by this build */
#define OC_ERR_TIMEOUT 702       /* a bounded wait inside a kernel expired */

/* ---- device object: implements GpuDevice (core:88-132) ----------------- */

typedef struct oc_device oc_device;

typedef struct {
  int ordinal;              /* DeviceInfo::id (core:35-42) */
  int cc_major, cc_minor;   /* GpuVendor::Nvidia{compute_capability} */
  uint64_t total_memory;    /* DeviceInfo::total_memory */
  uint32_t compute_units;   /* DeviceInfo::compute_units (SM count) */
  char name[256];           /* DeviceInfo::name */
} oc_device_info;

/* A launch configuration as the reference describes it (LaunchConfig,
 * core:45-85).  The CUDA backend picks its own launch shape for each named
 * kernel, so grid/block are accepted for contract compatibility only. */
typedef struct {
  uint32_t grid[3], block[3], shared_mem;
} oc_launch_config;

/* KernelArg (crates/opencuda-core/src/kernel.rs:88-100). */
enum { OC_ARG_PTR = 0, OC_ARG_U32 = 1, OC_ARG_I32 = 2, OC_ARG_F32 = 3, OC_ARG_USIZE = 4 };
typedef struct {
  int kind;
  union {
    uint64_t ptr; /* a DevicePtr.addr returned by oc_device_alloc */
    uint32_t u32;
    int32_t i32;
    float f32;
    uint64_t usize;
  } v;
} oc_kernel_arg;

/* Number of CUDA devices (registry enumerate, crates/opencuda-core/src/registry.rs). */
int oc_get_device_count(int *count);
/* Opens device `ordinal` (a GpuDevice instance). */
int oc_device_open(int ordinal, oc_device **dev);
/* Frees every allocation still held and the device object. */
int oc_device_close(oc_device *dev);
/* GpuDevice::info (core:89) */
int oc_device_get_info(const oc_device *dev, oc_device_info *info);
/* GpuDevice::alloc (core:92): bytes == 0 is an error, as on the CPU backend
 * (crates/opencuda-cpu/src/lib.rs:85-87).  *addr receives the raw CUDA
 * address, which is DevicePtr.addr. */
int oc_device_alloc(oc_device *dev, size_t bytes, uint64_t *addr);
/* GpuDevice::free (core:93): unknown address -> OC_ERR_INVALID_VALUE. */
int oc_device_free(oc_device *dev, uint64_t addr);
/* GpuDevice::memcpy_h2d/d2h/d2d (core:94-96): copies larger than the
 * allocation are rejected (crates/opencuda-cpu/src/lib.rs:120-151). */
int oc_device_memcpy_h2d(oc_device *dev, uint64_t dst, const void *src, size_t bytes);
int oc_device_memcpy_d2h(oc_device *dev, void *dst, uint64_t src, size_t bytes);
int oc_device_memcpy_d2d(oc_device *dev, uint64_t dst, uint64_t src, size_t bytes);
/* GpuDevice::synchronize (core:106); also reports kernel status words. */
int oc_device_synchronize(oc_device *dev);

/* ---- multi-device (crates/opencuda-multidev/src/lib.rs) ----------------- */

/* DevicePartition (multidev:17-22): layers [layer_start, layer_end) on the
 * device at index device_id of the list. */
typedef struct {
  size_t device_id, layer_start, layer_end;
} oc_device_partition;
/* partition_layers (multidev:28-74): device i < n-1 gets
 * floor(total_layers * mem_i / sum(mem)) layers, the last device the rest;
 * when every device reports 0 bytes, total_layers / n each and the rest to
 * the last.  An empty list is OC_ERR_INVALID_VALUE ("no devices to partition
 * across").  out receives num_devices entries.  No GPU work. */
int oc_partition_layers_by_memory(const uint64_t *total_memory, size_t num_devices, size_t total_layers,
                                  oc_device_partition *out);
/* The same over device objects (their oc_device_info total_memory). */
int oc_partition_layers(oc_device *const *devices, size_t num_devices, size_t total_layers,
                        oc_device_partition *out);
/* transfer_between_devices (multidev:78-83, a stub in the reference): copies
 * bytes from src_addr (an allocation of src) to dst_addr (an allocation of
 * dst), over NVLink as a peer copy when the two GPUs can access each other,
 * else staged through pinned host memory; returns when the copy is done.
 * Unknown addresses or sizes past either allocation are OC_ERR_INVALID_VALUE. */
int oc_transfer_between_devices(oc_device *src, uint64_t src_addr, oc_device *dst, uint64_t dst_addr, size_t bytes);
/* GpuDevice::launch_kernel (core:99-104), routed by kernel name the way the
 * Vulkan backend routes SPIR-V entry points
 * (crates/opencuda-vulkan/src/real.rs:868-887).  Names and argument
 * contracts (the reference's KernelArg lists):
 *   "sgemm_naive"        [A,B,C ptr; m,k,n usize; alpha,beta f32; u32
 *                        transpose_b] (blas:183-232).  The reference captures
 *                        transpose_b in the kernel closure (blas:206-210) and
 *                        launches only the first 8; that 8-argument form is
 *                        refused (OC_ERR_LAUNCH_FAILED) because its SDPA
 *                        caller needs B transposed (blas:517): route
 *                        scaled_dot_product_attention* to oc_blas_sdpa
 *   "matmul"             [A,B,C ptr; m,k,n usize], C = A.B (blas:335-348)
 *   "quantize_symmetric" [in,scales,out ptr; len,group usize; qmin,qmax f32]
 *                        (blas:834-868), one int8 per element
 *   "softmax"            [data ptr; rows,cols usize], in place (blas:383-385)
 *   "flash_attention"    [q,k,v,o ptr; seq,head_dim,block usize; scale f32]
 *                        (blas:745-760)
 *   "qgemm_w8"           [A,Wq,scales,bias,Y ptr; m,n,k usize]: oc_qgemm_w8
 *   "qgemm_w4"           [A,Wq,scales,bias,Y ptr; m,n,k,group usize]:
 *                        oc_qgemm_w4 (new blas functions launch these; no
 *                        counterpart kernel in the reference)
 * Pointer arguments must be allocations of this device large enough for
 * the shapes.  Other names: OC_ERR_LAUNCH_FAILED ("kernel source not
 * supported by this backend").  Asynchronous until oc_device_synchronize. */
int oc_device_launch(oc_device *dev, const char *kernel_name, const oc_launch_config *cfg,
                     const oc_kernel_arg *args, size_t nargs);
/* The stream this device object launches on (a cudaStream_t). */
void *oc_device_stream(oc_device *dev);

/* Message of the last failing call on this thread ("" if none). */
const char *oc_get_last_error(void);
/* Reads and clears the current device's kernel status word: 0 if every
 * kernel since the last call finished normally, else the code of the
 * first bounded wait that expired.  Synchronizes the device. */
int oc_get_device_status(int *status);

/* ---- GEMM (blas:148-295) ------------------------------------------------ */

/* C = alpha * A.op(B) + beta * C (+ bias[n] per column if bias != NULL).
 * A [m][lda], op(B) = B [k][ldb] (trans_b = 0, the reference's b[kk*n+col])
 * or B^T with B [n][ldb] (trans_b = 1, the transpose_b form of
 * launch_naive_gemm, blas:206-210); C [m][ldc].  f32 in and out, f32-level
 * accuracy (<= 1e-5 relative Frobenius): for beta == 0, m > 16, k % 64 == 0
 * (A 16-byte aligned, lda % 4 == 0; for trans_b the same for B) on tcgen05
 * f16 tensor cores with both operands split into two f16 terms after a
 * power-of-two scale per row of A and per column of op(B) (three MMAs per
 * product step); other large shapes on tf32 tensor cores with the 3xTF32
 * split; small m on a CUDA-core split-K GEMV.  beta == 0 does not read C.
 * Replaces the GemmPath::CuBlas arm of sgemm (blas:293). */
int oc_sgemm(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb, int trans_b,
             float beta, float *C, int ldc, const float *bias, void *stream);
/* For a B that is reused across calls (weights): oc_sgemm prepares B's
 * tensor-core operands on every call; these entry points split B into tf32
 * hi/lo halves laid out [n][k] once.  prepared holds
 * oc_sgemm_prepared_b_size() bytes; then oc_sgemm_prepared computes the same
 * product on the tf32 tensor cores with the 3xTF32 split (A must be 16-byte
 * aligned with lda % 4 == 0). */
int oc_sgemm_prepared_b_size(int k, int n, size_t *bytes);
int oc_sgemm_prepare_b(int k, int n, const float *B, int ldb, int trans_b, float *prepared, void *stream);
int oc_sgemm_prepared(int m, int n, int k, float alpha, const float *A, int lda, const float *prepared, float beta,
                      float *C, int ldc, const float *bias, void *stream);

/* ---- attention (blas:373-766) ------------------------------------------ */

/* In-place row softmax of data [rows][cols]: e = exp(x - max), divided by
 * the sum only if the sum is > 0 (cpu_row_softmax, blas:545-562;
 * softmax_vulkan_generic's contract, blas:373-391). */
int oc_softmax_rows(float *data, int rows, int cols, void *stream);
/* The fused slot flash_attention_with_spirv (blas:707-766): q, k, v, o are
 * [seq_len][head_dim]; every query row attends to all seq_len keys with
 * scale 1/sqrt(head_dim) and an online softmax (flash_attention,
 * blas:589-678).  block_size must be > 0; head_dim and block_size <= 256
 * (the limits the reference's shader enforces,
 * crates/opencuda-vulkan/src/real.rs:524-533).  The kernels tile keys by
 * 128 (head_dim 64 and 128: tcgen05 tensor cores) or 64 (other head dims)
 * regardless of block_size; results match the reference up to rounding. */
int oc_flash_attention(const float *q, const float *k, const float *v, float *o, int seq_len, int head_dim,
                       int block_size, void *stream);
/* General form: q/o [batch_heads][q_len][head_dim], k/v
 * [batch_heads][kv_len][head_dim], any scale; causal = 1 lets query i see
 * keys j <= i + (kv_len - q_len).  Covers multi-head SDPA (BERT,
 * crates/open-cuda-bert/src/lib.rs:141-167) and q_len != kv_len cross
 * attention (crates/open-cuda-whisper/src/lib.rs:288-300).  head_dim 64 and
 * 128 with 16-byte-aligned pointers run on the tcgen05 tensor cores: Q, K
 * (per row), V (per 128-key tile) and P are carried as two f16 terms each
 * (~22 significant bits), f32 accumulation; other shapes run a CUDA-core
 * f32 kernel. */
int oc_flash_attention_fwd(const float *q, const float *k, const float *v, float *o, int batch_heads, int q_len,
                           int kv_len, int head_dim, float scale, int causal, void *stream);
/* Unfused scaled_dot_product_attention (blas:411-540): scores = Q.K^T /
 * sqrt(d) (oc_sgemm, transpose_b), row softmax, O = P.V.  workspace holds
 * the seq_len x seq_len scores. */
int oc_sdpa_workspace_size(int seq_len, size_t *bytes);
int oc_sdpa(const float *q, const float *k, const float *v, float *o, int seq_len, int head_dim, void *workspace,
            size_t workspace_bytes, void *stream);

/* ---- MLA low-rank KV projections (blas:1045-1078) ----------------------- */

/* mla_compress_kv: latent [seq][d_c] = kv [seq][d_h] . down [d_h][d_c]. */
int oc_mla_compress_kv(int seq_len, int d_h, int d_c, const float *kv, const float *down_proj, float *latent,
                       void *stream);
/* mla_decompress_kv: out [seq][d_h] = latent [seq][d_c] . up [d_c][d_h]. */
int oc_mla_decompress_kv(int seq_len, int d_c, int d_h, const float *latent, const float *up_proj, float *out,
                         void *stream);

/* ---- GPT decoder (crates/open-cuda-llm/src/lib.rs:45-942) --------------- */

/* GptConfig (llm:45-69). */
typedef struct {
  size_t vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seq_len;
  float layer_norm_eps;
} oc_gpt_config;

typedef struct oc_gpt oc_gpt;
/* A device-resident GptModel on CUDA device `device` for up to max_batch
 * sequences with prompts of up to max_prompt_len tokens.  head_dim
 * (hidden_size / num_heads) must be <= 128 and hidden / intermediate sizes
 * multiples of 4.  Weights, KV cache and activations live in HBM; nothing is
 * copied per token. */
int oc_gpt_create(int device, const oc_gpt_config *cfg, int max_batch, int max_prompt_len, oc_gpt **model);
int oc_gpt_destroy(oc_gpt *model);
/* GptModel::load_random (llm:635-646): weights generated on the device from
 * SplitMix64(seed) in the reference's draw order, bit-identical to the
 * reference's values. */
int oc_gpt_load_random(oc_gpt *model, uint64_t seed);
/* Uploads one weight tensor from host memory (for real checkpoints,
 * llm:661-731).  which: 0 wte [V][H], 1 wpe [ctx][H], per layer 2 qkv_w
 * [H][3H], 3 qkv_b, 4 attn_out_w [H][H], 5 attn_out_b, 6 fc_w [H][I], 7 fc_b,
 * 8 proj_w [I][H], 9 proj_b, 10 ln1_w, 11 ln1_b, 12 ln2_w, 13 ln2_b; 14
 * lnf_w, 15 lnf_b, 16 lm_head_w [H][V], 17 lm_head_b.  Linear weights are
 * weight_t = [in][out] as the reference stores them. */
int oc_gpt_set_weight(oc_gpt *model, int which, int layer, const float *host, size_t len);
/* enable_mla_kv_compression (llm:822-838): K and V rows are kept as d_c-dim
 * latents per head (KvCacheHead::push, llm:564-583) and attention reads
 * their reconstruction (current_kv, llm:586-595), with per-layer, per-head
 * projections drawn from SplitMix64(seed) in the reference's order (down
 * [head_dim][d_c], then up [d_c][head_dim], next_f32(0.02)), bit-identical
 * to its values.  0 < d_c < head_dim, else OC_ERR_INVALID_VALUE.  Weight ids
 * 18 / 19 of oc_gpt_get_weight / oc_gpt_set_weight are then a layer's
 * down / up projections, [heads][head_dim][d_c] / [heads][d_c][head_dim]. */
int oc_gpt_enable_mla(oc_gpt *model, size_t d_c, uint64_t seed);
/* Copies one weight tensor back to host memory (same ids and shapes). */
int oc_gpt_get_weight(oc_gpt *model, int which, int layer, float *host, size_t len);
/* GptModel::generate (llm:910-929), greedy, for `batch` independent
 * sequences with prompts [batch][prompt_len] (host).  out [batch][max_new]
 * (host); logits_out (optional, host) [batch][max_new][vocab], the logits
 * each token was taken from; *produced = tokens per sequence (fewer than
 * max_new only when max_seq_len is reached, as in the reference). */
int oc_gpt_generate(oc_gpt *model, int batch, const uint32_t *prompts, int prompt_len, int max_new,
                    uint32_t *out, float *logits_out, int *produced);
/* The stream the model runs on (a cudaStream_t). */
int oc_gpt_stream(oc_gpt *model, void **stream);
/* Kernels launched by oc_gpt_generate on this model since it was created
 * (graph replays count every kernel node).  No counterpart in the
 * reference; for benchmarks and launch accounting. */
int oc_gpt_kernel_launches(oc_gpt *model, uint64_t *total);

/* ---- quantization (blas:777-945) ---------------------------------------
 * Groups are contiguous runs of `group` elements of the flat input
 * (group_scales, blas:797-809); scale = max|x| / qmax (0 for an all-zero
 * group); q = clamp(round_half_away(x / scale), -qmax, qmax). */

/* quantize_int8 (blas:935-940): data[len] int8, scales[ceil(len/group)]. */
int oc_quantize_int8(const float *x, size_t len, size_t group, int8_t *data, float *scales, void *stream);
/* quantize_int4 (blas:901-919): data[(len+1)/2] bytes, nibble = q + 8,
 * even index in the low nibble, odd in the high nibble. */
int oc_quantize_int4(const float *x, size_t len, size_t group, uint8_t *data, float *scales, void *stream);
/* dequantize_int8 / dequantize_int4 (blas:922-945). */
int oc_dequantize_int8(const int8_t *data, const float *scales, size_t len, size_t group, float *out,
                       void *stream);
int oc_dequantize_int4(const uint8_t *data, const float *scales, size_t len, size_t group, float *out,
                       void *stream);

/* quantize_int4_awq / dequantize_int4_awq (blas:958-1012) for a row-major
 * weight [rows][cols]: oc_awq_scales computes the per-column scales on the
 * host exactly as the reference does (s <= 0 ? 1 : powf(s, alpha)); the
 * device routines quantize weight * awq_scale[col] with quantize_int4 and
 * undo the column scale on dequantization.  awq_scale is device memory. */
int oc_awq_scales(const float *act_scale, size_t cols, float alpha, float *awq_scale);
int oc_quantize_int4_awq(const float *weight, size_t rows, size_t cols, const float *awq_scale, size_t group,
                         uint8_t *data, float *scales, void *stream);
int oc_dequantize_int4_awq(const uint8_t *data, const float *scales, size_t rows, size_t cols, size_t group,
                           const float *awq_scale, float *out, void *stream);

/* ---- quantized matmul (new API: the reference only quantizes) ----------
 * Y[m][n] = A[m][k] . W^T + bias with W^T stored as the reference quantizes
 * it: a [n][k] matrix flattened and passed to quantize_int8 (group = k, one
 * scale per output channel) or quantize_int4 (group = `group`, packed two
 * per byte).  The activation rows are quantized on the device with
 * quantize_int8(A, group = k).  The defined results are
 *   W8A8:  y = ((float)acc * sa[m]) * sw[n] + bias[n]
 *   W4A8:  s = 0; for each group j: s = fma((float)P_j, sw[n][j], s);
 *          y = s * sa[m] + bias[n]
 * with acc / P_j the exact int32 (group) partial sums.  W8A8 is computed
 * exactly so (tcgen05 kind::i8, exact int32).  W4A8 is computed exactly so
 * when acc_out is requested, for m <= 16, or when k % 128 != 0; otherwise
 * by the dequantizing tensor-core GEMM (each weight dequantized in f32 as
 * dequantize_int4 does, carried as two f16 terms, f32 accumulation), whose
 * y agrees with the definition to about 1e-6 relative.  `workspace` is device
 * scratch of at least oc_qgemm_workspace_size() bytes (quantized
 * activations and their scales); bias may be NULL.  acc_out (optional,
 * NULL to skip): the int32 accumulators, [m][n] for W8A8 and
 * [m][n][k/group] for W4A8. */
int oc_qgemm_workspace_size(int m, int k, size_t *bytes);
int oc_qgemm_w8a8(int m, int n, int k, const float *A, const int8_t *Wq, const float *w_scales,
                  const float *bias, float *Y, void *workspace, size_t workspace_bytes, int32_t *acc_out,
                  void *stream);
int oc_qgemm_w4a8(int m, int n, int k, int group, const float *A, const uint8_t *Wq, const float *w_scales,
                  const float *bias, float *Y, void *workspace, size_t workspace_bytes, int32_t *acc_out,
                  void *stream);

/* Weight-only quantized matmul: f32 activations, quantized weights, the
 * product the reference forms as Linear::forward over dequantized weights
 * (sgemm(A, dequantize(Wq)^T) + bias; llm:227-238 with blas:922-945):
 *   Y[m][n] = sum_k A[m][k] * x[n][k] + bias[n],
 *   x = q * w_scales[n]                    (oc_qgemm_w8: quantize_int8 of
 *                                           W^T with group = k)
 *   x = (nib - 8) * w_scales[(n*k + k') / group]   (oc_qgemm_w4: quantize_int4
 *                                           of W^T, packed two per byte)
 * f32 work, within 1e-5 relative Frobenius of the f32 reference.  INT4
 * with group 32, 1 <= m <= 64, k % 128 == 0 and n >= 18944 (enough
 * 128-column tiles for every SM) runs a tcgen05 kind::i8 GEMM on the packed
 * weights widened to int8 on chip and each activation row as three int8
 * digits of a per-row power-of-two scaling (rounding at 2^-23 of the row's
 * largest |a|; a row holding a NaN or an infinity yields NaN outputs).
 * Otherwise m <= 16 streams the weights once on the CUDA cores; larger m
 * runs a tcgen05 GEMM on f16 terms of both operands (~22 significant bits
 * each, f32 accumulation), in column chunks whose expanded weights fit in L2.
 * Scratch for the digits, the expanded terms and K-split partial sums is kept per
 * (device, stream) inside the library and grows on first use of a larger
 * shape (that first call synchronizes the device: make it before any stream
 * capture).  bias may be NULL.  Any group > 0 is accepted for INT4 (groups
 * may straddle rows as in the reference's flat quantization). */
int oc_qgemm_w8(int m, int n, int k, const float *A, const int8_t *Wq, const float *w_scales, const float *bias,
                float *Y, void *stream);
int oc_qgemm_w4(int m, int n, int k, int group, const float *A, const uint8_t *Wq, const float *w_scales,
                const float *bias, float *Y, void *stream);

/* The same products on activations that are already quantized, as
 * quantize_int8(A, group = k) returns them: qa [m][k] int8 and sa [m] f32
 * (for example tokens that arrive quantized).  No workspace needed. */
int oc_igemm_w8a8(int m, int n, int k, const int8_t *qa, const float *sa, const int8_t *Wq, const float *w_scales,
                  const float *bias, float *Y, int32_t *acc_out, void *stream);
int oc_igemm_w4a8(int m, int n, int k, int group, const int8_t *qa, const float *sa, const uint8_t *Wq,
                  const float *w_scales, const float *bias, float *Y, int32_t *acc_out, void *stream);
/* quantize_int8(A, group = k) for a row-major A [m][k]: qa [m][k], sa [m]. */
int oc_quantize_rows_int8(const float *A, int m, int k, int8_t *qa, float *sa, void *stream);

/* oc_qgemm_w8a8 for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Same arguments and result as
 * oc_qgemm_w8a8, minus the workspace: the quantized activations live in a
 * 16 MiB device array inside the library, so the call allocates nothing.
 * For hosts that may not call cudaMalloc (stream callbacks, embedders whose
 * device memory belongs to another allocator, bindings that only receive
 * input and output buffers).  Requires align256(m*k) + align256(4*m) <=
 * 16 MiB, else OC_ERR_INVALID_VALUE.  Every GPU that loads the library
 * keeps the array until exit; concurrent calls on one device that overlap
 * on the GPU race on it, so order them on one stream.  The first call on a
 * device looks up the array's address; make it before any stream capture.
 * The address is kept for the life of the process (as the library keeps its
 * other per-device state): do not call cudaDeviceReset on a device while the
 * library is in use on it. */
int oc_qgemm_w8a8_noalloc(int m, int n, int k, const float *A, const int8_t *Wq, const float *w_scales,
                          const float *bias, float *Y, void *stream);
/* The size of that array in bytes (16 MiB). */
int oc_qgemm_w8a8_noalloc_max_bytes(size_t *bytes);

/* ---- mixture of experts (no counterpart in the reference, which has no
 * MoE; the semantics are defined here) -----------------------------------
 * Experts are MLPs fc [F][D] -> gelu_new -> proj [D][F] with INT8
 * per-output-channel weights (W8A8 products as oc_qgemm_w8a8, no biases).
 * oc_moe_route: top-k of each token's logits [T][E] (ties -> lower expert
 *   index, NaN never chosen); topk_w = softmax of the k chosen logits:
 *   (float)exp((double)(l - l_max)) summed in f32 in selection order, then
 *   divided; 1/k each when every chosen logit is -inf or NaN.
 * oc_moe_dispatch: counts [E], offs [E+1] (row offsets of each expert's
 *   rows), pos [T*k] (row of each (token, choice)), src [T*k] (token of each
 *   row) and the gathered int8 rows xg [T*k][D] with scales sg; cursor is
 *   [E] ints of scratch.  Rows of one expert are contiguous; their order
 *   inside the expert is unspecified (results do not depend on it).  Ids
 *   outside [0, E) are dropped: their pos is -1 and the combine skips them.
 * oc_grouped_igemm_w8a8: Y[r] = xg[r] . W_g^T for the group g owning row r
 *   (offs in device memory, G <= 1024, non-decreasing from >= 0 to <= R),
 *   W stacked [G*N][K] with scales [G*N] and optional biases [G*N]; tiles
 *   are scheduled on the device.  Rows outside the groups are not written.
 * oc_gelu_quantize_rows: q, s = quantize_int8(gelu_new(H[r]), group = F).
 * oc_moe_combine: y[t] = shared[t] (or 0) + sum_{i<k} w[t][i] *
 *   expert_out[pos[t][i]], i ascending, multiply then add. */
int oc_moe_route(const float *logits, int T, int E, int k, int *topk_idx, float *topk_w, void *stream);
int oc_moe_dispatch(const int *topk_idx, int T, int k, int E, const int8_t *qx, const float *sx, int D, int *counts,
                    int *offs, int *pos, int *src, int8_t *xg, float *sg, int *cursor, void *stream);
int oc_grouped_igemm_w8a8(int R, int N, int K, const int8_t *xg, const float *sg, const int8_t *W, const float *sw,
                          const float *bias, const int *offs, int G, float *Y, void *stream);
int oc_gelu_quantize_rows(const float *H, int R, int F, int8_t *q, float *s, void *stream);
int oc_moe_combine(const float *shared_out, const float *expert_out, const int *pos, const float *topk_w, int T,
                   int k, int D, float *y, void *stream);

/* ---- multi-GPU column sharding (no counterpart in the reference, whose
 * only multi-device code is a layer partition stub,
 * crates/opencuda-multidev/src/lib.rs:28-83) ------------------------------
 * Each of g ranks computes Y_r = A . W_r^T for its block of N/g output
 * columns (rows of the quantized W^T); after an all-gather the shards sit
 * as [g][m][shard_cols].  oc_gather_columns writes them as out [m][g *
 * shard_cols], shard r at columns r*shard_cols .. */
int oc_gather_columns(const float *shards, float *out, int num_shards, int m, int shard_cols, void *stream);

/* ---- host-slice entry points (blas signatures on host memory) ---------- */

/* sgemm (blas:260-271): a [m][k], b [k][n], c [m][n] in/out. */
int oc_blas_sgemm(oc_device *dev, size_t m, size_t k, size_t n, float alpha, const float *a, const float *b,
                  float beta, float *c);
/* softmax_vulkan_generic (blas:373-391): out = row softmax of data. */
int oc_blas_softmax_rows(oc_device *dev, size_t rows, size_t cols, const float *data, float *out);
/* flash_attention_with_spirv (blas:707-766) without the SPIR-V bytes. */
int oc_blas_flash_attention(oc_device *dev, const float *q, const float *k, const float *v, size_t seq_len,
                            size_t head_dim, size_t block_size, float *out);
/* scaled_dot_product_attention (blas:411-423). */
int oc_blas_sdpa(oc_device *dev, const float *q, const float *k, const float *v, size_t seq_len, size_t head_dim,
                 float *out);
/* mla_compress_kv / mla_decompress_kv (blas:1045-1067). */
int oc_blas_mla_compress_kv(oc_device *dev, size_t seq_len, size_t d_h, size_t d_c, const float *kv,
                            const float *down_proj, float *latent);
int oc_blas_mla_decompress_kv(oc_device *dev, size_t seq_len, size_t d_c, size_t d_h, const float *latent,
                              const float *up_proj, float *out);
/* quantize_int8 / quantize_int4 (blas:901, 935); empty input or group 0
 * is OC_ERR_INVALID_VALUE (blas:867-872). */
int oc_blas_quantize_int8(oc_device *dev, const float *input, size_t len, size_t group, int8_t *data,
                          float *scales);
int oc_blas_quantize_int4(oc_device *dev, const float *input, size_t len, size_t group, uint8_t *data,
                          float *scales);
/* The quantized matmuls on host memory: A [m][k] f32, W^T quantized as
 * above, bias [n] (may be NULL), Y [m][n]. */
int oc_blas_qgemm_w8a8(oc_device *dev, size_t m, size_t n, size_t k, const float *a, const int8_t *wq,
                       const float *w_scales, const float *bias, float *y);
int oc_blas_qgemm_w4a8(oc_device *dev, size_t m, size_t n, size_t k, size_t group, const float *a,
                       const uint8_t *wq, const float *w_scales, const float *bias, float *y);
/* The weight-only matmuls (oc_qgemm_w8 / oc_qgemm_w4) on host memory, the
 * host-slice form of Linear::forward over dequantized weights (llm:227-238):
 * A [m][k] f32, W^T quantized as the reference quantizes it, bias [n] (may
 * be NULL), Y [m][n]; copies in, multiplies, copies out, synchronizes. */
int oc_blas_qgemm_w8(oc_device *dev, size_t m, size_t n, size_t k, const float *a, const int8_t *wq,
                     const float *w_scales, const float *bias, float *y);
int oc_blas_qgemm_w4(oc_device *dev, size_t m, size_t n, size_t k, size_t group, const float *a,
                     const uint8_t *wq, const float *w_scales, const float *bias, float *y);

#ifdef __cplusplus
}
#endif
#endif /* OPENCUDA_CUDA_H */
