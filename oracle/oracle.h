/*
 * oracle.h -- CPU restatement of Nimformer's quantised-weight matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * library, never part of it: only tests/, __graft_entry__.smoke() and the
 * cpu-baseline leg of bench.py load it.  The product library
 * (libnimf_cuda.so) has no CPU fallback and never calls into this code.
 *
 * Each function restates one reference procedure; the citation on each
 * declaration is "file:line" inside the reference project.  The reference
 * is written in Nim (no Nim toolchain here) and Python (the .nimq exporter);
 * the Python pieces are pinned bit-exactly by the golden fixtures under
 * tests/golden/ which were produced by importing the reference module
 * itself.  Built with -O2 -ffp-contract=off so every float32 operation is
 * rounded exactly where the reference rounds it (no fused multiply-add,
 * matching the x86-64 baseline code Nim emits).
 */
#ifndef NIMF_ORACLE_H
#define NIMF_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- quant.nim */

/* quant.nim:51-61  quantizeInt8: per-tensor scale = absmax/127 (1 if absmax==0),
 * q = clamp(int(round(v/scale)), -127, 127), Nim round = half away from zero. */
void orc_quantize_int8(const float* arr, int64_t n, int8_t* q, float* scale);

/* quant.nim:63-67  dequantizeInt8: w = float32(int8) * scale. */
void orc_dequantize_int8(const int8_t* q, int64_t n, float scale, float* out);

/* quant.nim:69-85  quantizeInt4 (symmetric, per-tensor, flat packing,
 * element i -> byte i/2, even i low nibble). */
void orc_quantize_int4_sym(const float* arr, int64_t n, uint8_t* packed, float* scale);

/* quant.nim:87-98  dequantizeInt4: nibble>=8 -> nibble-16, times scale. */
void orc_dequantize_int4_sym(const uint8_t* packed, int64_t n, float scale, float* out);

/* quant.nim:104-129 quantizeInt4Asymmetric (per-tensor). */
void orc_quantize_int4_asym_tensor(const float* arr, int64_t n, uint8_t* packed,
                                   float* scale, float* zero);

/* quant.nim:131-192 dequantizeInt4Asymmetric.
 *   group_size > 0 : per-group (rows x ceil(cols/group_size) scales), LUT per group
 *   n_scales > 1   : per-row
 *   otherwise      : per-tensor with flat packing (i/2)
 * Per-group / per-row packing is row-padded: bytesPerRow = ceil(cols/2). */
void orc_dequantize_int4_asym(const uint8_t* data, const float* scale, const float* zero,
                              int64_t n_scales, int64_t rows, int64_t cols,
                              int64_t group_size, float* out);

/* quant.nim:256-345 dequantizeTensorTransposed for the int kinds
 * (kind byte: 1 int8, 2 int4 sym, 3 int4 asym).  Output layout [cols, rows]. */
int orc_dequantize_transposed(int kind, const uint8_t* data, const float* scale,
                              const float* zero, int64_t n_scales, int64_t rows,
                              int64_t cols, int64_t group_size, float* out);

/* ------------------------------------------------------------ customfloat.nim */

/* customfloat.nim:15-31 newCustomFloat field derivation. */
typedef struct {
  int exponent_bits, mantissa_bits, total_bits, item_size;
  int bias, max_exp;
  int uses_uint64;
} orc_custom_float;
orc_custom_float orc_cf_new(int exponent_bits, int mantissa_bits);

/* customfloat.nim:49-78 fp32ToPackedU64 (truncating encode). */
uint64_t orc_cf_fp32_to_packed(float x, int exponent_bits, int mantissa_bits);

/* customfloat.nim:80-102 packedU64ToFp32. */
float orc_cf_packed_to_fp32(uint64_t packed, int exponent_bits, int mantissa_bits);

/* customfloat.nim:108-113,125-129 cpuEncodeArray / encodeArray
 * (itemSize little-endian bytes per element). Returns 0, or -1 if
 * total_bits > 64 (encodeArray's assert). */
int orc_cf_encode_array(const float* arr, int64_t n, int exponent_bits,
                        int mantissa_bits, uint8_t* out);

/* customfloat.nim:115-123,131-136 cpuDecodeArray / decodeArray.  Returns 0,
 * or -1 if nbytes is not a multiple of itemSize or total_bits > 64. */
int orc_cf_decode_array(const uint8_t* buf, int64_t nbytes, int exponent_bits,
                        int mantissa_bits, float* out);

/* customfloat.nim:149-165 computeRequiredExponentBits. */
int orc_cf_required_exponent_bits(const float* arr, int64_t n, int exp_margin);

/* customfloat.nim:167-198 computeRequiredMantissaBits (grad may be NULL/0). */
int orc_cf_required_mantissa_bits(const float* arr, int64_t n, double rel_error_tol,
                                  const float* grad, int64_t n_grad);

/* ----------------------------------------------------- vendor/bybylang/gpubackend.nim */

/* gpubackend.nim:560-582 cpuMatmul: C[m,n] = A[m,k] . B[k,n], blocked 64,
 * per output a sequential float32 sum over k ascending, skipping a == 0. */
void orc_cpu_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n,
                    float* c);

/* gpubackend.nim:628-653 cpuDequantMatmulQ4Fallback: LUT dequant of the
 * packed int4 [n rows of ceil(k/2) bytes] into wT[k,n], then cpuMatmul.
 * wt_scratch must hold k*n floats. */
void orc_dequant_matmul_q4(const float* a, const uint8_t* wq, const float* scales,
                           const float* zeros, int64_t m, int64_t k, int64_t n,
                           int64_t group_size, int64_t n_groups_per_row,
                           float* wt_scratch, float* out);

/* ------------------------------------------------------------ export_to_nimq.py */

/* export_to_nimq.py:363-395 quantize_int4_asymmetric_per_group.  numpy
 * semantics: min/max/range/scale/zp in float64, the element arithmetic
 * chunk/scale + zp in float32 (NEP 50 weak python scalars), np.round =
 * half-to-even, clip to [0,15]; scales/zeros stored as float32. */
void orc_quantize_int4_asym_per_group(const float* arr, int64_t rows, int64_t cols,
                                      int64_t group_size, uint8_t* packed,
                                      float* scales, float* zeros);

/* export_to_nimq.py:353-360 quantize_int8_vectorized (per-tensor, half-even). */
void orc_quantize_int8_vectorized(const float* arr, int64_t n, int8_t* q, float* scale);

/* export_to_nimq.py:219-254 dequantize_gptq_linear (GPTQ-native layout):
 * qweight int32 [K/8, N], qzeros int32 [G, N/8], scales fp16 bits [G, N],
 * g_idx [K]; zero = ((z & 0xF) + 1) & 0xF; w = (float(q) - float(zero)) * scale;
 * output float32 [N, K]. */
void orc_dequantize_gptq_linear(const int32_t* qweight, const int32_t* qzeros,
                                const uint16_t* scales_f16, const int32_t* g_idx,
                                int64_t in_features, int64_t out_features,
                                int64_t n_groups, float* out);

/* ------------------------------------------------ extensions with no reference */

/* FP4 E2M1 (OCP MX value set {0,.5,1,1.5,2,3,4,6}) with a per-16-element
 * E4M3 (OCP) block scale and a float32 tensor scale.  No reference
 * implementation exists: parity unpinned.  Packing: element k of a row at
 * byte k/2, even k in the low nibble (same order as quant.nim int4).
 * Quantisation: block amax/6 -> e4m3 (RNE, saturating), element RNE to the
 * nearest E2M1 value of x / (block_scale * tensor_scale). */
float orc_e4m3_ocp_to_float(uint8_t v);
uint8_t orc_float_to_e4m3_ocp(float x);
float orc_e2m1_to_float(uint8_t nib);
void orc_quantize_fp4_block16(const float* arr, int64_t rows, int64_t cols,
                              float tensor_scale, uint8_t* packed, uint8_t* block_scales);
void orc_dequantize_fp4_block16(const uint8_t* packed, const uint8_t* block_scales,
                                float tensor_scale, int64_t rows, int64_t cols, float* out);

/* Plain float64-accumulated reference GEMV y[m,n] = sum_k x[m,k] * w[n,k]
 * (w row-major [n,k]); a checker for tolerance tests, not a reference
 * restatement. */
void orc_gemv_f64(const float* x, const float* w, int64_t m, int64_t k, int64_t n,
                  float* y);

/* ------------------------------------------------ nim_inference.nim decode glue */

/* nim_inference.nim:143-200 (+ rmsNormPrep :114-140): y = (x * invStd) * w,
 * invStd = 1 / sqrt(sum(x*x) / cols + eps), sum in orc_cpu_matmul order. */
void orc_rmsnorm(const float* x, const float* w, int64_t rows, int64_t cols, float eps,
                 float* y);
/* nimformer.nim:188-197 LayerNorm.forward, CPU path vendor/bybylang/gpubackend.nim:252-266:
 * two sequential passes (mean, then variance about the mean);
 * y = ((x - mean) * invStd) * gamma + beta. */
void orc_layernorm(const float* x, const float* gamma, const float* beta, int64_t rows,
                   int64_t cols, float eps, float* y);
/* vendor/bybylang/gpubackend.nim:268-278 cpuEmbeddingLookup (zeros for ids out of range). */
void orc_embedding_lookup(const float* table, int64_t vocab, int64_t dim, const int32_t* ids,
                          int64_t n, float* out);
/* nim_inference.nim:1019-1036 sampleTopP, temperature <= 0 (greedy with the
 * repetition penalty), one id per row of logits. */
void orc_greedy_sample(const float* logits, int64_t rows, int64_t vocab, const int32_t* recent,
                       int64_t n_recent, float penalty, int32_t* out_ids);
/* nim_inference.nim:336-356 + vendor/bybylang/gpubackend.nim:111-114:
 * out = (g * (1 / (1 + exp(-g)))) * u. */
void orc_swiglu(const float* g, const float* u, int64_t n, float* out);
/* nim_inference.nim:261-330 applyRoPEInplace (rotate-half) with the caller's
 * cos / sin tables [max_seq][D/2] (newRoPEL :246-259). */
void orc_rope(float* data, int64_t B, int64_t T, int64_t H, int64_t D, int64_t pos_offset,
              const float* cos_t, const float* sin_t);
/* nim_inference.nim:404-426 appendKV + forwardDecode :624-748 attention core
 * (softmax as vendor/bybylang/gpubackend.nim:236-250). */
void orc_attention_decode(const float* q, const float* k_new, const float* v_new,
                          float* k_cache, float* v_cache, int64_t H, int64_t HKV, int64_t D,
                          int64_t max_seq, int64_t pos, float scale, float* out);

/* forwardPrefill's attention (nim_inference.nim:574-620) for T prompt tokens at
 * positions pos0 ..: appendKV, then causal cpuAttentionFused
 * (vendor/bybylang/gpubackend.nim:171-201) per query head; q, out [T][H][D],
 * k_new / v_new [T][HKV][D], caches [HKV][max_seq][D]. */
void orc_attention_prefill(const float* q, const float* k_new, const float* v_new,
                           float* k_cache, float* v_cache, int64_t T, int64_t H, int64_t HKV,
                           int64_t D, int64_t max_seq, int64_t pos0, float scale, float* out);

#ifdef __cplusplus
}
#endif
#endif
