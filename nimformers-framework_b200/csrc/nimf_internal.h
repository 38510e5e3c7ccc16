// nimf_internal.h -- host-side internals shared by the translation units of
// libnimf_cuda.so (error reporting, the per-process device context, the
// weight registry and the kernel launchers).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <memory>
#include <vector>

#include "../../include/nimf_cuda.h"

namespace nimf {

// ----------------------------------------------------------------- errors
// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);

#define NIMF_CUDA_TRY(expr)                                                                   \
  do {                                                                                        \
    cudaError_t e__ = (expr);                                                                 \
    if (e__ != cudaSuccess)                                                                   \
      return ::nimf::set_error(NIMF_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                \
                               cudaGetErrorString(e__), __FILE__, __LINE__);                  \
  } while (0)

#define NIMF_TRY(expr)           \
  do {                           \
    int s__ = (expr);            \
    if (s__ != NIMF_OK) return s__; \
  } while (0)

// ----------------------------------------------------------------- weights
// Device copy of an int4 asymmetric per-group weight (N-shard of rows).
//   fast layout (group_size % 64 == 0):
//     frag : [n_rt][kq_total][32 lanes] uint4, word j of a lane = the
//            mma.m16n8k16 A-fragment nibbles of k-tile 4*kq+j (see q4g.cu)
//     sz   : [n_rt][groups][8] float4 {scale(r), zero(r), scale(r+8), zero(r+8)}
//   generic layout (any other group size):
//     raw  : the reference bytes [rows][ceil(K/2)], scales/zeros [rows][ngr]
struct Q4GWeight {
  int64_t rows = 0, k = 0, gs = 0, ngr = 0;
  bool fast = false;
  bool tc_zp_ok = false;  // every zero point finite with |zp| < 60000 (tensor-core GEMM)
  bool tc16_ok = false;   // (n - zp) * sc * 2^tc16_exp fits fp16 tiles (fp16-tile GEMM)
  int tc16_exp = 0;
  int64_t n_rt = 0, kq_total = 0, groups = 0;
  void* frag = nullptr;   // uint4*
  void* sz = nullptr;     // float4*
  void* raw = nullptr;    // uint8_t*
  void* scales = nullptr; // float*
  void* zeros = nullptr;  // float*
};

// Tensor-core GEMV layout of a byte-coded float weight (fw.cu): int8, one-byte
// CustomFloat E4M3 / E5M2 whose codes decode exactly like OCP FP8, FP4 E2M1.
enum { FW_I8 = 0, FW_E4M3 = 1, FW_E5M2 = 2, FW_FP4 = 3 };
struct FWLayout {
  int fmt = -1;                    // FW_*; -1: no fast layout (generic kernels)
  int64_t rows = 0, k = 0, n_rt = 0, ntk = 0;
  void* frag = nullptr;            // uint4 [n_rt][ntk][32]
  void* sfrag = nullptr;           // FP4: uint2 [n_rt][ntk][8] block scales
  const float* rscale = nullptr;   // per-row output scale (not owned), or
  float uscale = 1.0f;             // one scale for every row
};

// Device copy of an int8 weight: q [rows][K] int8, scales [1 or rows].
struct I8Weight {
  int64_t rows = 0, k = 0, n_scales = 0;
  void* q = nullptr;
  void* scales = nullptr;
};

// Device copy of a CustomFloat weight: item bytes [rows][K*item], optional
// per-row scale.
struct CFWeight {
  int64_t rows = 0, k = 0;
  int e = 0, m = 0, item = 0;
  void* data = nullptr;
  void* row_scales = nullptr;
};

// Device copy of an FP4 E2M1 block-16 weight.
struct FP4Weight {
  int64_t rows = 0, k = 0;
  float tensor_scale = 1.0f;
  void* packed = nullptr;  // [rows][ceil(K/2)]
  void* bscale = nullptr;  // [rows][ceil(K/16)]
};

// Device copy of an fp32 weight stored [N][K] (transposed from beMatmul's b).
struct F32Weight {
  int64_t rows = 0, k = 0;
  void* w = nullptr;
};

struct Weight {
  int kind = -1;
  int64_t device_bytes = 0;
  Q4GWeight q4;
  I8Weight i8;
  CFWeight cf;
  FP4Weight fp4;
  F32Weight f32;
  FWLayout fw;  // int8 / CustomFloat / FP4: tensor-core GEMV copy of the codes
  // act-order GPTQ weights: stored column j holds input feature kperm[j]
  // (device int32 [K]; x is gathered through it before each matmul)
  void* kperm = nullptr;
  std::vector<int32_t> kperm_host;
  // N-shard registration: rows [row_begin, row_begin + rows()) of n_full
  int64_t row_begin = 0, n_full = 0;
  int64_t rows() const;
  int64_t k() const;
};

// ----------------------------------------------------------------- context
struct Context {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  // growable device staging buffers for the host-pointer entry points
  void* stage_in = nullptr;
  size_t stage_in_bytes = 0;
  void* stage_out = nullptr;
  size_t stage_out_bytes = 0;
  // Host-mapped error word: kernels whose bounded waits expire set it to a
  // non-zero code instead of hanging; blocking entry points and nimf_sync
  // report it as NIMF_ERR_TIMEOUT and clear it.
  volatile int* host_err = nullptr;
  int* dev_err = nullptr;
};

// Returns NIMF_ERR_TIMEOUT (and clears the word) if a kernel reported an
// expired wait since the last check.  Call after a stream synchronisation.
int check_device_error();

Context* ctx();                        // nullptr before nimf_init
int require_ctx(Context** out);        // NIMF_ERR_STATE if not initialised
int stage_in(size_t bytes, void** p);  // grows the input staging buffer
int stage_out(size_t bytes, void** p); // grows the output staging buffer
int device_alloc(void** p, size_t bytes);
void device_free(void* p);

Weight* lookup(nimf_weight_t h);
nimf_weight_t insert(std::unique_ptr<Weight> w);
void free_weight_storage(Weight* w);

// ----------------------------------------------------------------- launchers
// All launchers validate their arguments, enqueue on `st` and return a status.
int q4g_build(Weight* w, const uint8_t* wq_dev, const float* sc_dev, const float* zp_dev,
              int64_t row_begin, int64_t rows, int64_t n_full, int64_t k, int64_t gs,
              int64_t ngr, cudaStream_t st);
int q4g_gemv(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st);
// Several int4 weights with the same K and group size applied to the same x
// in one persistent launch (their row tiles are streamed back to back).
int q4g_gemv_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                   float* const* ys, cudaStream_t st);
int q4g_dequant(const Q4GWeight& w, float* out, cudaStream_t st);
// The grouped GEMV with its outputs also stored into every rank's buffer
// (the fused all-gather of N-shard outputs, comm.cu): ys[i] is where this
// rank's first row goes in the local full output (row stride ldys[i]).
constexpr int kCommMaxRanks = 8;  // GPUs of one node the multi-GPU paths address
struct GatherSpec {
  int world = 1;
  long long peer_off[kCommMaxRanks] = {};  // byte offset from a local output address to rank q's copy
  unsigned* ctl = nullptr;     // the group's control words (local)
  unsigned long long wait_ns = 0;
};
int q4g_gemv_group_gather(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                          float* const* ys, const int64_t* ldys, const GatherSpec& g,
                          cudaStream_t st);
// Prefill GEMM on tcgen05 (x with many rows); q4g_tc_supported tells whether
// the weight's group size has a tensor-core kernel.
bool q4g_tc_supported(const Q4GWeight& w);
int q4g_gemm_tc(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st);
// Per-device scratch of the tensor-core GEMMs' prepared x (grown outside
// stream capture; calls using it are ordered on one stream).
int tc_prep_buffer(size_t bytes, cudaStream_t st, unsigned char** out);
void release_prep_buffers();
int q4g_gemm_tc_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                      float* const* ys, cudaStream_t st);
// Prefill GEMM with the weights dequantised into fp16 tiles and one
// accumulator over K (q4g_tc16.cu); used when every weight qualifies and the
// mode (nimf_q4_prefill_mode) allows it.
bool q4g_tc16_supported(const Q4GWeight& w);
int q4g_gemm_tc16_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                        float* const* ys, cudaStream_t st);
extern int g_q4_prefill_mode;   // NIMF_Q4_PREFILL_*

int i8_gemv(const I8Weight& w, const float* x, int64_t m, float* y, cudaStream_t st);
int i8_dequant(const I8Weight& w, float* out, cudaStream_t st);

int cf_encode(const float* x, int64_t n, int e, int m, uint8_t* out, cudaStream_t st);
int cf_decode(const uint8_t* buf, int64_t n_items, int e, int m, float* out, cudaStream_t st);
int cf_gemv(const CFWeight& w, const float* x, int64_t m, float* y, cudaStream_t st);
int cf_dequant(const CFWeight& w, float* out, cudaStream_t st);
// min / max of |x| over finite non-zero elements; returns found=0 when none.
int cf_absrange(const float* x, int64_t n, float* min_abs, float* max_abs, int* found,
                cudaStream_t st);
// median (element n_valid/2 of the ascending order) of |x| over finite non-zero x.
int cf_abs_median(const float* x, int64_t n, float* median, int64_t* n_valid, cudaStream_t st);

// Byte-coded float weights on the tensor cores (fw.cu).  fw_build repacks the
// reference codes (raw_dev) into L; the *_special_codes count tells whether a
// one-byte CustomFloat weight decodes exactly like OCP FP8 (count 0).
int fw_build(FWLayout* L, int fmt, const void* raw_dev, const void* bscale_dev,
             const float* rscale_dev, float uscale, int64_t rows, int64_t k, cudaStream_t st);
int fw_count_special_codes(const uint8_t* d, int64_t n, int mbits, int64_t* count,
                           cudaStream_t st);
void fw_free(FWLayout* L);
void fw_release_scratch();
int fw_gemv(const FWLayout& L, const float* x, int64_t m, float* y, cudaStream_t st);
int fw_dequant(const FWLayout& L, float* out, cudaStream_t st);
// Prefill GEMM of a byte-coded float weight on tcgen05 (fw_tc.cu).
int fw_gemm_tc(const FWLayout& L, const float* x, int64_t m, float* y, cudaStream_t st);

// x[m][k] gathered through a column permutation into a per-device scratch
// buffer (gptq.cu); *out points at the gathered rows.
int gather_cols(const float* x, int64_t m, int64_t k, const int32_t* perm, const float** out,
                cudaStream_t st);
void release_perm_buffer();
void release_attn_buffer();  // glue.cu: decode attention's split partials
void release_decode_plans(); // decode.cu: whole-step plans
void release_p2p_groups();   // p2p.cu: IPC buffers and peer mappings of the all-gather groups

int fp4_gemv(const FP4Weight& w, const float* x, int64_t m, float* y, cudaStream_t st);
int fp4_dequant(const FP4Weight& w, float* out, cudaStream_t st);

// Runs a registered weight's matmul on device buffers (any kind).
int weight_matmul_dev(Weight* w, const float* x, int64_t m, float* y, cudaStream_t st);

// ----------------------------------------------------------------- multi-GPU
// Rows [*r0, *r1) of an n-row weight held by `rank` of `world`: whole 16-row
// tiles, sizes within one tile (the host mirror's shard_rows).
void shard_range(int64_t n, int world, int rank, int64_t* r0, int64_t* r1);
// world 1 / rank 0 without a communicator.
int comm_world(int* world, int* rank);
// Shares a cudaMalloc'd buffer with every rank (CUDA IPC handles exchanged
// over the communicator); peers[q] is rank q's buffer as mapped here
// (peers[rank] = local).  Collective: every rank calls it in the same order.
int comm_share_buffer(void* local, void** peers);
void comm_unshare_buffer(void** peers, int world, int rank);
int comm_allgather_bytes(const void* src, size_t bytes, void* dst_host);
int comm_barrier();
// *all_ok = 1 when every rank passed ok != 0 (collective)
int comm_agree(int ok, int* all_ok);
void release_comm();

void release_f32_scratch();     // f32.cu: split-K partials of the fp32 GEMV
int f32_gemm(const float* a, int64_t m, int64_t k, const float* w_nk, int64_t n, float* c,
             cudaStream_t st);
int f32_transpose(const float* b_kn, int64_t k, int64_t n, float* w_nk, cudaStream_t st);

}  // namespace nimf
