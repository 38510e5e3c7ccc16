/*
 * nimf_cuda.h -- C ABI of libnimf_cuda.so, the B200 (sm_100a) implementation
 * of Nimformer's quantised-weight matmul path.
 *
 * Drop-in boundary.  Every entry point below replaces one call of the
 * reference's backend path; the citation beside it names the reference
 * procedure ("file:line" inside the Nimformer project).  The reference host
 * code binds these with {.importc: "nimf_...", dynlib: "libnimf_cuda.so".}.
 *
 * Conventions
 *   - Plain C types only; all sizes are int64_t element counts.
 *   - Every function returns NIMF_OK (0) or a negative NIMF_ERR_* code and
 *     never falls back to the CPU.  nimf_last_error() returns a thread-local
 *     message for the last failure on the calling thread (the Nim wrapper
 *     raises CatchableError(msg), like cuda_runtime.nim:64-66).
 *   - One process drives one GPU (nimf_init(device)).  Calls are made from
 *     one host thread; the library is not re-entrant.
 *   - Functions taking HOST pointers are blocking: inputs are copied to the
 *     device, the kernel runs, results are copied back before return (the
 *     same contract as backend.nim's be* procs).  Functions with the _dev
 *     suffix take DEVICE pointers and a cudaStream_t (passed as void*, NULL =
 *     the library stream) and are asynchronous.
 *   - Weight layout on entry is the reference's QuantTensor layout
 *     (quant.nim:22-35): row = output channel, W[N][K].
 */
#ifndef NIMF_CUDA_H
#define NIMF_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NIMF_OK 0
#define NIMF_ERR_ARG (-1)         /* bad pointer / argument                    */
#define NIMF_ERR_SHAPE (-2)       /* inconsistent sizes                        */
#define NIMF_ERR_CUDA (-3)        /* CUDA runtime / launch failure             */
#define NIMF_ERR_NCCL (-4)        /* collective failure                        */
#define NIMF_ERR_TIMEOUT (-5)     /* bounded device / host wait expired        */
#define NIMF_ERR_UNSUPPORTED (-6) /* format or shape not implemented           */
#define NIMF_ERR_STATE (-7)       /* nimf_init not called / bad handle         */

typedef uint64_t nimf_weight_t; /* opaque handle of a device-resident weight */

/* Weight kinds (values equal the reference's on-disk QuantKind ordinal,
 * quant.nim:12-20, where one exists). */
#define NIMF_KIND_F32 0
#define NIMF_KIND_INT8 1
#define NIMF_KIND_INT4_SYM 2
#define NIMF_KIND_INT4_ASYM 3
#define NIMF_KIND_CUSTOM_FLOAT 6
#define NIMF_KIND_FP4_E2M1 100 /* no reference counterpart (extension) */

/* ------------------------------------------------------------ lifetime */

/* Replaces cuda_driver.nim:173-194 ensureInit (context, stream, PTX module
 * load) for this path: binds the calling process to `device`, creates the
 * library stream.  Idempotent for the same device. */
int nimf_init(int device);

/* Frees every registered weight and the library stream.  cuda_driver.nim has
 * no counterpart (its singletons live until exit). */
int nimf_shutdown(void);

/* Thread-local message of the last failure (cuda_driver.nim:88-92 gpuCheck
 * raises with such a message). */
const char* nimf_last_error(void);

/* Number of visible CUDA devices (cuda_runtime.nim:116-120 cudaRuntimeAvailable). */
int nimf_device_count(int* count);

/* Blocks until all work on the library stream is done. */
int nimf_sync(void);

/* Number of device allocations (cudaMalloc) the library has made since it
 * was loaded, for hosts that check which calls allocate.  No counterpart in
 * the reference. */
int nimf_alloc_count(int64_t* count);

/* ------------------------------------------------------------ weights */

/* int4 asymmetric per-group weights exactly as QuantTensor holds them
 * (quant.nim:131-167, export_to_nimq.py:363-395):
 *   wq      : N rows of ceil(K/2) bytes, element k of a row in byte k/2,
 *             even k in the low nibble
 *   scales, zeros : float32 [N * n_groups_per_row], group g = k / group_size
 *   w[n,k] = (float(nibble) - zero) * scale
 * group_size <= 0 means one group per row (gpubackend.nim:645, gc = 0).
 * Rows [row_begin, row_end) are uploaded (an N-shard); pass 0, N for all.
 * Uploads once; the returned handle replaces the per-call copies of
 * beMatmulQ4 (backend.nim:93-101).  Weights are repacked on the device into
 * a tensor-core fragment order (the dequantised values are unchanged). */
int nimf_weight_register_q4g(const uint8_t* wq, const float* scales, const float* zeros,
                             int64_t n, int64_t k, int64_t group_size,
                             int64_t n_groups_per_row, int64_t row_begin, int64_t row_end,
                             nimf_weight_t* out);

/* int8 symmetric weights, quant.nim:51-67: q int8 [N][K], n_scales == 1
 * (per-tensor, the reference) or n_scales == N (per output channel, an
 * extension the reference does not have).  w = float(q) * scale. */
int nimf_weight_register_i8(const int8_t* q, const float* scales, int64_t n_scales,
                            int64_t n, int64_t k, int64_t row_begin, int64_t row_end,
                            nimf_weight_t* out);

/* CustomFloat-encoded weights (customfloat.nim:49-136, quant.nim:198-206,254):
 * data holds N*K items of ceil((1+e+m)/8) little-endian bytes, decoded with
 * packedU64ToFp32 semantics.  row_scales (nullable) multiplies output channel
 * n after decoding (the per-channel fp8 scale extension; the reference stores
 * no scale, quant.nim:203). */
int nimf_weight_register_cf(const uint8_t* data, int exponent_bits, int mantissa_bits,
                            const float* row_scales, int64_t n, int64_t k,
                            int64_t row_begin, int64_t row_end, nimf_weight_t* out);

/* FP4 E2M1 with one OCP-E4M3 scale per 16 elements of a row and a float32
 * tensor scale (no reference counterpart: the reference's CustomFloat(2,1)
 * is a different format).  packed: N rows of ceil(K/2) bytes, even k low
 * nibble; block_scales: N * ceil(K/16) bytes.
 * w = e2m1(nibble) * (e4m3(block_scale) * tensor_scale). */
int nimf_weight_register_fp4(const uint8_t* packed, const uint8_t* block_scales,
                             float tensor_scale, int64_t n, int64_t k, int64_t row_begin,
                             int64_t row_end, nimf_weight_t* out);

/* GPTQ-native int4 checkpoint tensors as export_to_nimq.py:219-254
 * (dequantize_gptq_linear) reads them: qweight int32 [in_features/8][out],
 * nibble k % 8 of qweight[k/8][n]; qzeros int32 [n_groups][out/8], nibble
 * n % 8; scales fp16 bits [n_groups][out]; g_idx int32 [in_features].
 * w[n][k] = (nib - ((z + 1) & 15)) * float(scale), bit-identical to the
 * reference, without its fp32 round-trip.  Groups must hold equal numbers of
 * input features (the last may hold fewer); act-order g_idx is supported by
 * storing k grouped and gathering x through the permutation at each call.
 * Output channels [row_begin, row_end) are uploaded.  Resulting weights
 * behave as int4 group weights (nimf_weight_info reports kind 3). */
int nimf_weight_register_gptq(const int32_t* qweight, const int32_t* qzeros,
                              const uint16_t* scales_f16, const int32_t* g_idx,
                              int64_t in_features, int64_t out_features, int64_t n_groups,
                              int64_t row_begin, int64_t row_end, nimf_weight_t* out);

/* Raw float32 weights given as beMatmul's b operand [K][N] row-major
 * (backend.nim:87, gpubackend.nim:584). */
int nimf_weight_register_f32(const float* b_kn, int64_t k, int64_t n, nimf_weight_t* out);

/* Releases the device copy (cuda_driver.nim:262-265 freeResident). */
int nimf_weight_free(nimf_weight_t w);

/* Logical shape, kind and device bytes of a registered weight. */
int nimf_weight_info(nimf_weight_t w, int64_t* n_rows, int64_t* k, int* kind,
                     int64_t* device_bytes);

/* ------------------------------------------------------------ matmul */

/* y[M][N_shard] = x[M][K] . W^T for any registered weight, HOST buffers,
 * blocking.  Format-generic form of Linear.forward's dispatch
 * (nimformer.nim:101-133): int4 -> beMatmulQ4, other kinds -> the
 * dequantizeTensorTransposed + beMatmul branch, without the host dequant. */
int nimf_matmul_w(nimf_weight_t w, const float* x, int64_t m, float* y);

/* Same on DEVICE buffers (x [M][K], y [M][N_shard] row-major, fp32),
 * asynchronous on `stream` (NULL = library stream).  This is the resident
 * form the reference's CUDA session API has for fp32 only
 * (cuda_runtime.nim:158-180 cudaMatmulF32R). */
int nimf_matmul_w_dev(nimf_weight_t w, const float* x_dev, int64_t m, float* y_dev,
                      void* stream);

/* Several weights with the same K applied to the same x, DEVICE buffers:
 * y_devs[i][M][N_i] = x[M][K] . W_i^T.  int4 weights of one group size run as a
 * single persistent launch that streams all their rows back to back (the
 * fused q/k/v and gate/up projections of nim_inference.nim:506-508,818-819,
 * which the reference issues as separate linearFastBias calls).  Other kinds
 * are applied one after another. */
int nimf_matmul_w_group_dev(const nimf_weight_t* handles, int count, const float* x_dev,
                            int64_t m, float* const* y_devs, void* stream);

/* HOST-buffer, blocking form of nimf_matmul_w_group_dev.  x is copied in
 * once for the group; outputs whose host buffers follow one another
 * (ys[i+1] == ys[i] + M * N_i) come back in one copy. */
int nimf_matmul_w_group(const nimf_weight_t* handles, int count, const float* x, int64_t m,
                        float* const* ys);

/* Drop-in for beMatmulQ4 (backend.nim:93-110 -> gpubackend.nim:655-676):
 * same arguments, HOST arrays, out = float32 [M*N].  The reference reads the
 * arrays afresh on every call; here their device copy is cached, keyed by the
 * wq, scales and zeros pointers and the shape, and a hit also needs the same
 * fingerprint of the three arrays' contents (by default over every byte:
 * about 3 ms for a 4096 x 12288 weight on one host core).  So a weight freed
 * and replaced by another of the same shape at the same address, or scales /
 * zeros changed in place, give fresh results.  nimf_weight_cache_clear()
 * drops the cache. */
int nimf_matmul_q4(const float* a, const uint8_t* wq, const float* scales,
                   const float* zeros, int64_t m, int64_t k, int64_t n, int64_t group_size,
                   int64_t n_groups_per_row, float* out);
int nimf_weight_cache_clear(void);

/* How nimf_matmul_q4 checks a cache hit (no reference counterpart):
 * FULL (default) fingerprints every byte of wq, scales and zeros on each call;
 * SAMPLED only the first and last 4 KB of each and 64 bytes of every 4 KB in
 * between (a change elsewhere can go unseen); NONE trusts the pointers and
 * shape, for hosts whose weights are immutable after setQuantWeight
 * (nimformer.nim:94-100) and that call nimf_weight_cache_clear() whenever
 * they free or replace one. */
#define NIMF_Q4_CACHE_CHECK_FULL 0
#define NIMF_Q4_CACHE_CHECK_SAMPLED 1
#define NIMF_Q4_CACHE_CHECK_NONE 2
int nimf_q4_cache_set_check(int mode);
/* Number of weights the nimf_matmul_q4 cache holds. */
int nimf_q4_cache_size(int64_t* entries);

/* Drop-in for beMatmul (backend.nim:87-91 -> cuda_runtime.nim:122-152):
 * C[M][N] = A[M][K] . B[K][N], fp32, HOST arrays.  k2 must equal k. */
int nimf_matmul_f32(const float* a, int64_t m, int64_t k, const float* b, int64_t k2,
                    int64_t n, float* out);

/* Drop-in for beMatmul2 (backend.nim:112-119 -> gpubackend.nim:606-626):
 * two independent fp32 GEMMs issued together. */
int nimf_matmul2_f32(const float* a1, int64_t m1, int64_t k1, const float* b1, int64_t k1b,
                     int64_t n1, const float* a2, int64_t m2, int64_t k2, const float* b2,
                     int64_t k2b, int64_t n2, float* out1, float* out2);

/* Test hook: writes the dequantised weight of a registered int / fp format as
 * float32 [N_shard][K] in the reference's row-major layout, computed by the
 * device with the reference's rounding ((float(q) - zero) * scale,
 * quant.nim:162), so a bit-exact comparison with dequantizeTensor is possible. */
int nimf_dequant_w(nimf_weight_t w, float* out_host);

/* Which tensor-core GEMM serves int4 group weights at more than 16 rows of x
 * (prefill).  No reference counterpart (the reference dequantises on the host,
 * gpubackend.nim:628-653).  AUTO (default): the fp16-tile GEMM, where each
 * weight is dequantised into fp16 tiles ((nibble - zp) * scale times a
 * per-weight power of two) and one fp32 accumulator runs over K, for weights
 * whose values fit fp16 tiles, else the exact-nibble GEMM; EXACT: always the
 * exact-nibble GEMM (nibbles exact in fp16, an fp32 epilogue per group).
 * Both keep max|y - y_ref| / max|y_ref| within 1e-3; the exact form is about
 * 2e-4, the fp16 tiles about 3e-4 at K = 4096. */
#define NIMF_Q4_PREFILL_AUTO 0
#define NIMF_Q4_PREFILL_EXACT 1
int nimf_q4_prefill_mode(int mode);

/* ------------------------------------------------------------ decode glue */
/* The steps between the linears of a Llama-style decode step
 * (nim_inference.nim), on DEVICE buffers and asynchronous on `stream`, so the
 * activations stay in HBM across the quantised matmuls.  Products and sums the
 * reference rounds separately are rounded separately; reductions run in a
 * tree order. */

/* RMSNormL.forward (nim_inference.nim:143-200, rmsNormPrep :114-140):
 * y[r][c] = (x[r][c] * inv_r) * w[c], inv_r = 1 / sqrt(sum_c x^2 / cols + eps). */
int nimf_rmsnorm_dev(const float* x, const float* w, int64_t rows, int64_t cols, float eps,
                     float* y, void* stream);

/* LayerNorm.forward (nimformer.nim:188-197) = beLayernorm (backend.nim:149-150),
 * following the CPU path cpuLayernorm (vendor/bybylang/gpubackend.nim:252-266):
 * mean = sum_c x / cols, var = sum_c (x - mean)^2 / cols,
 * y[r][c] = ((x[r][c] - mean) * (1 / sqrt(var + eps))) * gamma[c] + beta[c].
 * x and y may alias. */
int nimf_layernorm_dev(const float* x, const float* gamma, const float* beta, int64_t rows,
                       int64_t cols, float eps, float* y, void* stream);

/* beAdd (backend.nim) as the residual connections of TransformerBlockLlama
 * use it (nim_inference.nim:847-875): out = a + b. */
int nimf_add_dev(const float* a, const float* b, int64_t n, float* out, void* stream);

/* The residual add and the next RMSNorm in one launch: h = a + b (the
 * residual stream, TransformerBlockLlama.forward nim_inference.nim:847-875),
 * then y = RMSNorm(h) as nimf_rmsnorm_dev.  h may alias a. */
int nimf_add_rmsnorm_dev(const float* a, const float* b, const float* w, int64_t rows,
                         int64_t cols, float eps, float* h, float* y, void* stream);

/* SwiGLUL.forward gating (nim_inference.nim:336-356): out = (g * sigmoid(g)) * up,
 * sigmoid = 1 / (1 + exp(-g)) (vendor/bybylang/gpubackend.nim:111-114). */
int nimf_swiglu_dev(const float* gate, const float* up, int64_t n, float* out, void* stream);

/* applyRoPEInplace (nim_inference.nim:261-330) on data [B][T][H][D] in place:
 * rotate-half with the caller's tables cos_t / sin_t [max_seq][D/2] built as
 * newRoPEL does (:246-259); position of token t is pos_offset + t. */
int nimf_rope_dev(float* data, int64_t B, int64_t T, int64_t H, int64_t D, int64_t pos_offset,
                  const float* cos_t, const float* sin_t, int64_t max_seq, void* stream);

/* One decode token of GQAAttention.forwardDecode (nim_inference.nim:624-748):
 * appends k_new / v_new [HKV][D] at row `pos` of the caches [HKV][max_seq][D]
 * (appendKV :404-426), then for each query head h of H (KV head h / (H/HKV)):
 * scores over the pos + 1 cached rows of (q * scale) . K^T, softmax
 * (vendor/bybylang/gpubackend.nim:236-250), out[h] = P . V.  D a multiple of 32,
 * at most 256.  Internal partial buffers grow on first use (make the first
 * call with a given size before any stream capture). */
int nimf_attention_decode_dev(const float* q, const float* k_new, const float* v_new,
                              float* k_cache, float* v_cache, int64_t H, int64_t HKV, int64_t D,
                              int64_t max_seq, int64_t pos, float scale, float* out, void* stream);

/* The attention of forwardPrefill (nim_inference.nim:574-620) for T prompt
 * tokens at positions pos0 .. pos0 + T - 1 (pos0 = 0: the whole prompt; > 0:
 * a later chunk): appendKV (:404-426) of k_new / v_new [T][HKV][D] into rows
 * pos0 .. of the caches [HKV][max_seq][D], then for each token t and query
 * head h the causal softmax attention of cpuAttentionFused
 * (vendor/bybylang/gpubackend.nim:171-201) over cache rows 0 .. pos0 + t of
 * KV head h / (H / HKV): score = (q . k) * scale.  q and out are [T][H][D]
 * (the projections' rows).  D a multiple of 32, at most 256;
 * pos0 + T <= max_seq. */
int nimf_attention_prefill_dev(const float* q, const float* k_new, const float* v_new,
                               float* k_cache, float* v_cache, int64_t T, int64_t H, int64_t HKV,
                               int64_t D, int64_t max_seq, int64_t pos0, float scale, float* out,
                               void* stream);

/* One decode token for each of B sequences at positions read on the device,
 * so a captured batch step can be replayed token after token (the batch form
 * of nimf_rope_dev + nimf_attention_decode_dev; forwardDecode,
 * nim_inference.nim:624-748, per sequence).  q [B][H][D], k_new / v_new
 * [B][HKV][D], caches [B][HKV][max_seq][D], pos_dev [B] int32 (each
 * sequence's position; outside [0, max_seq) the sequence appends nothing, its
 * output is undefined and nimf_sync reports NIMF_ERR_TIMEOUT-class error 4).
 * With cos_t / sin_t (nullable together) q and k_new are first rotated in
 * place at pos[b] (applyRoPEInplace, :261-330).  advance_pos != 0 adds 1 to
 * every pos[b] after the call's last use of it.  out [B][H][D]. */
int nimf_attention_decode_batch_dev(float* q, float* k_new, const float* v_new, float* k_cache,
                                    float* v_cache, int64_t B, int64_t H, int64_t HKV, int64_t D,
                                    int64_t max_seq, int32_t* pos_dev, const float* cos_t,
                                    const float* sin_t, float scale, int advance_pos, float* out,
                                    void* stream);

/* Token embedding rows, as cpuEmbeddingLookup (vendor/bybylang/gpubackend.nim:268-278,
 * beEmbeddingLookup backend.nim:152-153; Embedding.lookupBatch nimformer.nim:401-411):
 * out[i][0..dim) = table[ids[i]][0..dim) for 0 <= ids[i] < vocab, zeros otherwise.
 * table [vocab][dim] fp32, ids [n] int32, out [n][dim], all on the device. */
int nimf_embedding_lookup_dev(const float* table, int64_t vocab, int64_t dim,
                              const int32_t* ids, int64_t n, float* out, void* stream);

/* The greedy branch of sampleTopP (nim_inference.nim:1019-1036, temperature <= 0),
 * per row of logits [rows][vocab]: for each entry of the row's recent ids
 * recent[row][0..n_recent) inside [0, vocab), in order, the logit is divided by
 * repeat_penalty if it is positive, else multiplied by it (an id listed twice is
 * adjusted twice); out_ids[row] = the first index of the largest adjusted logit
 * (a strict-greater scan from index 0: NaNs never win, a NaN at index 0 gives 0).
 * repeat_penalty 1 skips the adjustment.  vocab <= 262144, n_recent <= 2048;
 * the logits are not modified.  All buffers on the device. */
int nimf_greedy_sample_dev(const float* logits, int64_t rows, int64_t vocab, const int32_t* recent,
                           int64_t n_recent, float repeat_penalty, int32_t* out_ids, void* stream);

/* ------------------------------------------------------------ whole decode step */
/* One decode token of a Llama-style stack with int4 group-128 weights as ONE
 * persistent, cooperative launch: LlamaModelL.forwardStep(ids = [token],
 * isPrefill = false) (nim_inference.nim:887-921) -- embedding lookup, per
 * layer RMSNorm, q/k/v, RoPE, KV append and attention (forwardDecode
 * :624-748), o, residual add + RMSNorm, gate/up, SwiGLU, down, residual add --
 * then the final RMSNorm and the lm_head, followed by the greedy branch of
 * sampleTopP (:1019-1036) when a next-token buffer is given.  The results
 * equal the one-launch-per-op path of the glue entry points above up to the
 * order of the reductions (x is quantised into two 8-bit digits per element
 * with one scale per stage, as in the GEMV).
 *
 * Every pointer in the descriptors is a device pointer borrowed by the plan
 * (it must stay valid until nimf_decode_destroy); every weight is a handle of
 * an int4 asymmetric weight with group size 128 registered without an
 * act-order permutation: wq [d_model x d_model], wk / wv [n_kv_heads*head_dim
 * x d_model], wo [d_model x d_model], wgate / wup [ffn x d_model], wdown
 * [d_model x ffn], lm_head [vocab x d_model] (rows = output features, as
 * quant.nim).  Caches are [n_kv_heads][max_seq][head_dim] fp32 and rope
 * tables [max_seq][head_dim/2] (newRoPEL).  Limits: d_model and ffn multiples
 * of 128 up to 14336, head_dim 64 or 128, n_heads * head_dim = d_model,
 * n_heads <= 64 and a multiple of n_kv_heads, at most 256 recent ids. */
typedef struct nimf_decode_layer_desc {
  nimf_weight_t wq, wk, wv, wo, wgate, wup, wdown;
  const float* attn_norm; /* [d_model] RMSNorm weight before attention */
  const float* ffn_norm;  /* [d_model] RMSNorm weight before the FFN   */
  float* k_cache;         /* [n_kv_heads][max_seq][head_dim]            */
  float* v_cache;
} nimf_decode_layer_desc;

typedef struct nimf_decode_desc {
  int64_t n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq;
  int64_t n_recent_max;   /* recent ids a step may pass (<= 256) */
  float norm_eps;
  const float* embedding; /* [vocab][d_model] */
  const float* final_norm;
  nimf_weight_t lm_head;
  const float* rope_cos;  /* [max_seq][head_dim/2] */
  const float* rope_sin;
  const nimf_decode_layer_desc* layers; /* host array of n_layers (copied) */
} nimf_decode_desc;

/* Builds the step's stage table and its device scratch (a few hundred KB).
 * The environment variable NIMF_DECODE_L2_AHEAD (0 .. 16, default 0), read
 * here, sets how many of its items each weight-streaming lane prefetches into
 * L2 ahead of its shared-memory ring (0: none). */
int nimf_decode_create(const nimf_decode_desc* desc, int64_t* plan);
/* The same step N-sharded over the communicator's GPUs (nimf_comm_init; no
 * counterpart in the reference, which has no multi-GPU path).  Collective:
 * every rank calls it with its own descriptor.  Every weight handle holds
 * this rank's nimf_shard_range rows of the full weight; the caches hold this
 * rank's KV heads, [n_kv_heads / world][max_seq][head_dim] (KV heads
 * [rank * n_kv_heads / world, ...) and the query heads that read them);
 * n_heads and n_kv_heads must be multiples of world.  Each step computes
 * this rank's rows of every projection and its heads' attention and stores
 * them into every rank's plan scratch over NVLink (plain peer stores through
 * CUDA IPC, no multicast); a stage starts once every rank's last CTA has
 * raised its arrival on every rank (bounded waits, as the one-GPU step).
 * logits_dev receives this rank's lm_head rows at their positions of the
 * full [vocab] vector; next_token_dev receives the same greedy choice on
 * every rank.  Every rank must make the same sequence of step calls;
 * nimf_decode_destroy of a sharded plan is collective too. */
int nimf_decode_create_sharded(const nimf_decode_desc* desc, int64_t* plan);
/* Enqueues one step on `stream` (NULL: the library stream); asynchronous.
 * token_dev [1] int32: the input token (out-of-range ids embed as zeros);
 * pos_dev [1] int32: its position (the KV row appended; 0 <= pos < max_seq,
 * else the step reports NIMF_ERR_TIMEOUT-class device error 4 through
 * nimf_sync and appends nothing), incremented by the step when advance_pos is
 * non-zero; logits_dev [vocab] fp32 receives the logits; next_token_dev
 * (nullable, may equal token_dev) receives the greedy choice over the logits
 * with repeat_penalty applied once per occurrence of an id in
 * recent_dev[0..n_recent).  Both token and position are read on the device,
 * so a CUDA graph of this call can be replayed token after token.  A grid
 * barrier that waits longer than the bound (nimf_decode_set_timeout_ms, 2 s by
 * default) gives up, and nimf_sync reports NIMF_ERR_TIMEOUT. */
int nimf_decode_step_dev(int64_t plan, int32_t* token_dev, int32_t* next_token_dev,
                         int32_t* pos_dev, int advance_pos, const int32_t* recent_dev,
                         int64_t n_recent, float repeat_penalty, float* logits_dev, void* stream);
/* Profiling aid (no reference counterpart): while timeline_dev (device,
 * n >= 12 * stages uint64 entries) is set, each step records for CTA `cta`
 * the %globaltimer nanoseconds at which, per stage: [0] its consumers passed
 * the stage's grid barrier, [1] finished the stage's x prologue, [2] its merge
 * warp (attention stages: its consumers) arrived, and inside the prologue
 * [3] x's inputs were in, [4] the norm's sum, [5] max|x| was reduced, and in
 * the GEMV body [6] consumer warp 0 had its first item, [7] finished its last
 * chunk, [8] the merge warp had stored y, and for warp 0's first chunk [9] its
 * products were summed, [10] its partial slot was free, [11] the partial was
 * handed to the merge warp (0 where a stage has no such step).  NULL stops
 * recording. */
int nimf_decode_timeline(int64_t plan, uint64_t* timeline_dev, int64_t n, int cta);
/* Grid size (CTAs), number of stages and attention position splits of a plan. */
int nimf_decode_info(int64_t plan, int64_t* grid, int64_t* stages, int64_t* attn_splits);
/* Bound of the step's grid-barrier waits, milliseconds (1 .. 600000). */
int nimf_decode_set_timeout_ms(int64_t ms);
int nimf_decode_destroy(int64_t plan);

/* ------------------------------------------------- sharded outputs over peer memory */
/* The reference has no multi-GPU path.  These calls gather N-shard outputs
 * (rank r computed output columns [r*cols, (r+1)*cols)) into the full x of the
 * next projection, one process per GPU, with plain peer stores over NVLink
 * through CUDA IPC and one bounded flag wait per peer, no collective library.
 *
 * nimf_p2p_create (each rank, after nimf_init): allocates this rank's shared
 *   buffer for slices of up to slot_floats floats and writes its 64-byte IPC
 *   handle to ipc_handle_out; *group receives the group id.  2 <= world <= 8.
 * nimf_p2p_connect: opens the peers' buffers from the world handles
 *   (world * 64 bytes, rank order), exchanged by the host (e.g. over the
 *   process group's object all-gather).  Call on every rank before the first
 *   all-gather.
 * nimf_p2p_allgather_dev: dst[i][q*cols + j] = rank q's src[i][j] for every
 *   rank q, i < rows, j < cols (row strides ld_src, ld_dst in floats;
 *   rows * cols <= slot_floats).  Every rank must make the same sequence of
 *   calls on the group (the calls are counted); asynchronous on `stream` and
 *   capturable in a CUDA graph.  A peer that does not arrive within the wait
 *   bound (2 s unless nimf_p2p_set_timeout_ms changed it) makes the kernel
 *   return with dst incomplete and the next nimf_sync report
 *   NIMF_ERR_TIMEOUT; until then later calls give up at once.
 * nimf_p2p_set_timeout_ms: the bound of every peer wait of this process, in
 *   milliseconds (1 .. 600000), for calls launched afterwards.
 * nimf_p2p_destroy: synchronises the device and releases the mappings and
 *   the buffer (call on every rank after the last all-gather of every rank,
 *   e.g. after a host barrier). */
int nimf_p2p_create(int world, int rank, int64_t slot_floats, void* ipc_handle_out,
                    int64_t* group);
int nimf_p2p_connect(int64_t group, const void* ipc_handles);
int nimf_p2p_allgather_dev(int64_t group, const float* src, int64_t rows, int64_t cols,
                           int64_t ld_src, float* dst, int64_t ld_dst, void* stream);
int nimf_p2p_set_timeout_ms(int64_t ms);
int nimf_p2p_destroy(int64_t group);
/* nimf_p2p_connect_comm: nimf_p2p_connect with the handles exchanged over the
 * library's communicator (nimf_comm_init) instead of by the host.  Collective:
 * every rank of the group calls it once, after nimf_p2p_create. */
int nimf_p2p_connect_comm(int64_t group);

/* ------------------------------------------------- communicator (NCCL) */
/* N-sharded weights (row = output channel) with an NCCL all-gather of the output
 * slices, inside the library so that a host binding only this header gets
 * the sharded path.  The reference has no multi-GPU path (its CUDA device is
 * fixed at 0, vendor/bybylang/backends/cuda/cuda_driver.nim:183); these calls
 * replace nothing of it.  One process per GPU.  NCCL is opened at run time
 * (libnccl.so.2); without it these calls return NIMF_ERR_UNSUPPORTED.
 *
 * nimf_comm_unique_id: rank 0 writes 128 bytes that every rank must receive
 *   out of band (a file, a pipe, the launcher's environment).
 * nimf_comm_init: after nimf_init, on every rank, with the same id; world
 *   1 .. 8.  Collective (blocks until every rank has joined).
 * nimf_comm_info: world and rank (1 and 0 without a communicator).
 * nimf_comm_allgather_dev: dst[q * bytes .. (q + 1) * bytes) = rank q's src,
 *   asynchronous on `stream` (NULL: the library stream).
 * nimf_comm_barrier: blocks until every rank has called it.
 * nimf_comm_destroy: synchronises and releases the communicator.
 * nimf_shard_range: rows [*row_begin, *row_end) of an n-row weight that rank
 *   `rank` of `world` holds -- whole 16-row tiles, sizes within one tile.
 *   Register each rank's shard with exactly this range (row = output channel,
 *   nimformer.nim:90).
 * nimf_matmul_w_allgather_dev: y[m][N] = x[m][K] . W^T on every rank, where
 *   this rank's handle holds its nimf_shard_range rows of the N-row weight:
 *   the shard's matmul, an NCCL all-gather of the slices and (unless m == 1
 *   and the shards are equal) a layout pass.  Collective; asynchronous on
 *   `stream`.  A call that must grow its gather buffers refuses a capturing
 *   stream (NIMF_ERR_STATE): run it once before capture. */
int nimf_comm_unique_id(void* id_out);
int nimf_comm_init(int world, int rank, const void* id);
int nimf_comm_info(int* world, int* rank);
int nimf_comm_allgather_dev(const void* src, int64_t bytes, void* dst, void* stream);
int nimf_comm_barrier(void);
int nimf_comm_destroy(void);
int nimf_shard_range(int64_t n, int world, int rank, int64_t* row_begin, int64_t* row_end);
int nimf_matmul_w_allgather_dev(nimf_weight_t w, const float* x_dev, int64_t m, float* y_dev,
                                void* stream);
/* The all-gather fused into the int4 GEMV (no separate collective):
 * nimf_gather_create (collective) allocates a buffer of `bytes` on every rank,
 * shared by CUDA IPC, and returns its local address; outputs of
 * nimf_matmul_w_group_gather_dev must lie inside it.  That call runs the
 * grouped GEMV of up to 16 int4 group weights (shards per nimf_shard_range,
 * the same K, 1 .. 8 rows of x) whose merge warps store every finished output
 * value into the same place of every rank's buffer with plain peer stores
 * over NVLink (no multicast); y_devs[i] is where weight i's full output
 * [m][N_i] starts.  The launch's last CTA raises an arrival on every rank and
 * waits (bounded: nimf_gather_set_timeout_ms, 2 s by default; expiry is
 * reported by nimf_sync as NIMF_ERR_TIMEOUT) for every rank's arrival, so
 * when the call completes in stream order the gathered outputs are in place.
 * Every rank must make the same sequence of calls on a group, and an output
 * must not be overwritten by a call while another rank may still read the
 * previous call's values there (a chain of dependent projections, as in
 * decode, satisfies this; alternate buffers otherwise).  nimf_gather_destroy
 * is collective. */
int nimf_gather_create(int64_t bytes, int64_t* group, void** buffer_dev);
int nimf_matmul_w_group_gather_dev(int64_t group, const nimf_weight_t* handles, int count,
                                   const float* x_dev, int64_t m, float* const* y_devs,
                                   void* stream);
int nimf_gather_set_timeout_ms(int64_t ms);
int nimf_gather_destroy(int64_t group);

/* ------------------------------------------------------------ .nimq state dicts */

/* One tensor record of a NIMQ2 stream (quant.nim:386-409 readQuantTensor).
 * The pointers point into the caller's buffer; scales and zeros are
 * n_scales little-endian float32 values that may be unaligned. */
typedef struct {
  const char* name;
  int64_t name_len;
  int kind;                /* QuantKind ordinal, quant.nim:12-20 */
  int ndims;
  int64_t dims[8];
  int64_t n_scales;
  const uint8_t* scales;
  const uint8_t* zeros;
  int64_t group_size;
  int exponent_bits, mantissa_bits;
  const uint8_t* data;
  int64_t data_len;
} nimf_nimq_tensor;

/* loadQuantStateDict (quant.nim:429-448) on a stream held in memory: checks
 * the "NIMQ2" magic (NIMF_ERR_ARG otherwise) and that every record lies
 * inside [buf, buf + len) (NIMF_ERR_SHAPE otherwise); returns the 5
 * architecture integers (arch may be NULL) and the tensor count.  Host only:
 * needs neither nimf_init nor a device. */
int nimf_nimq_parse(const uint8_t* buf, int64_t len, int32_t* arch, int64_t* count);

/* Record `index` of the stream (host only). */
int nimf_nimq_get(const uint8_t* buf, int64_t len, int64_t index, nimf_nimq_tensor* out);

/* Uploads rows [row_begin, row_end) of record `index`, a 2-D weight W[N][K]
 * (row = output channel, nimformer.nim:90), as a device-resident weight:
 * kind 1 int8 (scale[0], as dequantizeInt8), kind 2 / 3 int4 with rows of
 * ceil(K/2) bytes as dequantizeTensorTransposed reads them (quant.nim:270-330;
 * per group, per row or per tensor), kinds 4-7 CustomFloat codes, kind 0 raw
 * fp32 (whole tensor only, registered as beMatmul's b = W^T).  Replaces
 * setQuantWeight's host copy and per-forward dequantisation
 * (nimformer.nim:94-133): the packed codes go from the file to HBM once. */
int nimf_nimq_register(const uint8_t* buf, int64_t len, int64_t index, int64_t row_begin,
                       int64_t row_end, nimf_weight_t* out);

/* ------------------------------------------------------------ CustomFloat / APF */

/* beCustomfloatEncode (backend.nim:177-178 -> customfloat.nim:125-129):
 * out receives n * itemSize bytes.  total bits must be <= 64. */
int nimf_cf_encode(const float* x, int64_t n, int exponent_bits, int mantissa_bits,
                   uint8_t* out);

/* beCustomfloatDecode (backend.nim:180-181 -> customfloat.nim:131-136):
 * nbytes must be a multiple of itemSize; out receives nbytes/itemSize floats. */
int nimf_cf_decode(const uint8_t* buf, int64_t nbytes, int exponent_bits, int mantissa_bits,
                   float* out);

/* Device-buffer forms of the two above (asynchronous on `stream`). */
int nimf_cf_encode_dev(const float* x_dev, int64_t n, int exponent_bits, int mantissa_bits,
                       uint8_t* out_dev, void* stream);
int nimf_cf_decode_dev(const uint8_t* buf_dev, int64_t nbytes, int exponent_bits,
                       int mantissa_bits, float* out_dev, void* stream);

/* buildCustomDtypeForTensor (customfloat.nim:149-206): chooses exponent and
 * mantissa bits for x (grad nullable, n_grad may be 0). */
int nimf_cf_autoselect(const float* x, int64_t n, const float* grad, int64_t n_grad,
                       double rel_error_tol, int exp_margin, int* exponent_bits,
                       int* mantissa_bits);

/* beApfCastForTraining (backend.nim:183-186 -> customfloat.nim:208-213):
 * autoselect + encode.  out must hold n * 8 bytes (the largest itemSize);
 * the chosen format is returned in exponent_bits / mantissa_bits and the
 * encoded length is n * ceil((1+e+m)/8). */
int nimf_apf_cast(const float* x, int64_t n, const float* grad, int64_t n_grad,
                  double rel_error_tol, int exp_margin, int* exponent_bits,
                  int* mantissa_bits, uint8_t* out);

/* Allocation-free form of nimf_cf_autoselect on device buffers.  No
 * counterpart in the reference: it is for callers that cannot allocate device
 * memory at the point of the call -- a host whose allocator owns the whole
 * GPU memory and forbids other cudaMalloc calls, or code that must not add
 * allocations while it runs.  x_dev / grad_dev are device pointers (grad_dev
 * nullable, n_grad may be 0); the reductions run on `stream` (NULL: the
 * library stream) and the call returns when the chosen format is known.
 * Scratch lives in a fixed 8,200-byte device array inside the library, so it
 * allocates nothing.  The first call on each device looks up that array's
 * address.  The call reads its reductions back to the host and synchronises
 * `stream`; on a stream that is being captured it returns NIMF_ERR_STATE.
 * Limits: n and n_grad at most 2^31 - 1 (larger gives NIMF_ERR_SHAPE); calls
 * that overlap on the GPU share the array and race, so issue them one at a
 * time. */
int nimf_cf_autoselect_dev_noalloc(const float* x_dev, int64_t n, const float* grad_dev,
                                   int64_t n_grad, double rel_error_tol, int exp_margin,
                                   int* exponent_bits, int* mantissa_bits, void* stream);

#ifdef __cplusplus
}
#endif
#endif
