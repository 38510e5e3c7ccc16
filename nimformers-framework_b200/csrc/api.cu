// api.cu -- the extern "C" entry points of libnimf_cuda.so (declared in
// include/nimf_cuda.h): error reporting, the per-process device context, the
// device weight registry and the host-buffer drop-ins for backend.nim's be*
// procs.  No entry point falls back to the CPU: a missing device or a failed
// launch is returned as an error status, like gpubackend.nim:46-61 with
// gForbidCpuFallback = true.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "nimf_internal.h"

namespace nimf {

namespace {
thread_local char g_err[1024] = "";
Context g_ctx;
bool g_ready = false;
std::mutex g_mu;
std::unordered_map<nimf_weight_t, std::unique_ptr<Weight>> g_weights;
nimf_weight_t g_next = 1;
// beMatmulQ4 host-array cache: (wq, scales, zeros pointers, k, n, gs, ngr) ->
// the registered handle and a fingerprint of the three arrays' contents.  A
// hit needs the same pointers, shape and fingerprint, so a weight whose
// address is reused by another of the same shape, or scales / zeros changed in
// place, are registered afresh.
using Q4Key = std::tuple<uintptr_t, uintptr_t, uintptr_t, int64_t, int64_t, int64_t, int64_t>;
struct Q4Entry {
  nimf_weight_t handle = 0;
  uint64_t fingerprint = 0;
};
std::map<Q4Key, Q4Entry> g_q4_cache;
int g_q4_check = NIMF_Q4_CACHE_CHECK_FULL;

// 64-bit fingerprint of a byte range: four independent multiply-rotate lanes
// over 8-byte words (about 10 GB/s on one core), then the tail bytes.
uint64_t fp_mix(uint64_t h, uint64_t w) {
  h ^= w * 0x9E3779B97F4A7C15ull;
  h = (h << 27) | (h >> 37);
  return h * 0xD6E8FEB86659FD93ull;
}

uint64_t fingerprint_bytes(const void* p, size_t n, uint64_t seed) {
  const unsigned char* b = (const unsigned char*)p;
  uint64_t l0 = seed ^ 0x243F6A8885A308D3ull, l1 = seed ^ 0x13198A2E03707344ull;
  uint64_t l2 = seed ^ 0xA4093822299F31D0ull, l3 = seed ^ 0x082EFA98EC4E6C89ull;
  size_t i = 0;
  for (; i + 32 <= n; i += 32) {
    uint64_t w[4];
    std::memcpy(w, b + i, 32);
    l0 = fp_mix(l0, w[0]);
    l1 = fp_mix(l1, w[1]);
    l2 = fp_mix(l2, w[2]);
    l3 = fp_mix(l3, w[3]);
  }
  uint64_t h = fp_mix(fp_mix(fp_mix(fp_mix(0, l0), l1), l2), l3);
  for (; i < n; ++i) h = fp_mix(h, (uint64_t)b[i] | ((uint64_t)i << 8));
  return fp_mix(h, (uint64_t)n);
}

// Sampled fingerprint: the first and last 4 KB and one 64-byte block of every
// 4 KB in between.
uint64_t fingerprint_sampled(const void* p, size_t n, uint64_t seed) {
  const unsigned char* b = (const unsigned char*)p;
  if (n <= 16384) return fingerprint_bytes(p, n, seed);
  uint64_t h = fingerprint_bytes(b, 4096, seed);
  h = fp_mix(h, fingerprint_bytes(b + n - 4096, 4096, seed + 1));
  for (size_t o = 4096; o + 64 <= n - 4096; o += 4096)
    h = fp_mix(h, fingerprint_bytes(b + o, 64, o));
  return fp_mix(h, (uint64_t)n);
}

uint64_t q4_fingerprint(const uint8_t* wq, size_t wbytes, const float* sc, const float* zp,
                        size_t sbytes, int mode) {
  if (mode == NIMF_Q4_CACHE_CHECK_NONE) return 0;
  auto f = mode == NIMF_Q4_CACHE_CHECK_SAMPLED ? fingerprint_sampled : fingerprint_bytes;
  uint64_t h = f(wq, wbytes, 1);
  h = fp_mix(h, f(sc, sbytes, 2));
  return fp_mix(h, f(zp, sbytes, 3));
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

Context* ctx() { return g_ready ? &g_ctx : nullptr; }

int check_device_error() {
  if (g_ready && g_ctx.host_err && *g_ctx.host_err != 0) {
    const int code = *g_ctx.host_err;
    *g_ctx.host_err = 0;
    return set_error(NIMF_ERR_TIMEOUT,
                     "a kernel's bounded wait expired (code %d); its output is not valid", code);
  }
  return NIMF_OK;
}

int require_ctx(Context** out) {
  if (!g_ready) return set_error(NIMF_ERR_STATE, "nimf_init() has not been called");
  NIMF_CUDA_TRY(cudaSetDevice(g_ctx.device));
  *out = &g_ctx;
  return NIMF_OK;
}

std::atomic<int64_t> g_alloc_count{0};

int device_alloc(void** p, size_t bytes) {
  *p = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) {
    *p = nullptr;
    return set_error(NIMF_ERR_CUDA, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
  }
  g_alloc_count.fetch_add(1, std::memory_order_relaxed);
  return NIMF_OK;
}

void device_free(void* p) {
  if (p) cudaFree(p);
}

static int grow(void** buf, size_t* have, size_t bytes) {
  if (bytes <= *have && *buf) return NIMF_OK;
  size_t want = std::max<size_t>(bytes, 1 << 20);
  want = std::max(want, *have * 2);
  if (*buf) {
    cudaStreamSynchronize(g_ctx.stream);
    device_free(*buf);
    *buf = nullptr;
    *have = 0;
  }
  NIMF_TRY(device_alloc(buf, want));
  *have = want;
  return NIMF_OK;
}

int stage_in(size_t bytes, void** p) {
  NIMF_TRY(grow(&g_ctx.stage_in, &g_ctx.stage_in_bytes, bytes));
  *p = g_ctx.stage_in;
  return NIMF_OK;
}

int stage_out(size_t bytes, void** p) {
  NIMF_TRY(grow(&g_ctx.stage_out, &g_ctx.stage_out_bytes, bytes));
  *p = g_ctx.stage_out;
  return NIMF_OK;
}

// Pinned host staging for the matmul entry points' PAGEABLE host buffers (a
// Nim seq, a numpy array).  cudaMemcpyAsync on pageable memory goes through
// the driver's own staging and, device to host, waits for the stream: one
// host wait per copy.  Up to kHostStageMax bytes go through these pinned
// buffers instead (a host memcpy each way), so a call waits on its stream
// once.  Pinned buffers, and larger pageable ones, are copied directly.
namespace {
constexpr size_t kHostStageMax = 4u << 20;
struct HostStage {
  void* p = nullptr;
  size_t bytes = 0;
  bool busy = false;   // an async copy from / to it may still be pending
};
HostStage g_hin, g_hout;

bool is_pageable(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();   // not a CUDA-known pointer: treat as pageable
    return true;
  }
  return at.type == cudaMemoryTypeUnregistered;
}

// Makes s hold `bytes` and be free to overwrite.
int host_stage(HostStage& s, size_t bytes) {
  if (s.busy) {
    NIMF_CUDA_TRY(cudaStreamSynchronize(g_ctx.stream));
    s.busy = false;
  }
  if (s.bytes >= bytes && s.p) return NIMF_OK;
  if (s.p) cudaFreeHost(s.p);
  s.p = nullptr;
  s.bytes = 0;
  const size_t want = std::max<size_t>(bytes, 64u << 10);
  NIMF_CUDA_TRY(cudaHostAlloc(&s.p, want, cudaHostAllocDefault));
  s.bytes = want;
  return NIMF_OK;
}

void release_host_stages() {
  for (HostStage* s : {&g_hin, &g_hout}) {
    if (s->p) cudaFreeHost(s->p);
    *s = HostStage();
  }
}

// Host x -> device, through the pinned stage when x is small and pageable.
int copy_in(void* dst_dev, const void* src, size_t bytes, cudaStream_t st) {
  if (bytes == 0) return NIMF_OK;
  if (bytes <= kHostStageMax && is_pageable(src)) {
    NIMF_TRY(host_stage(g_hin, bytes));
    std::memcpy(g_hin.p, src, bytes);
    g_hin.busy = true;
    src = g_hin.p;
  }
  NIMF_CUDA_TRY(cudaMemcpyAsync(dst_dev, src, bytes, cudaMemcpyHostToDevice, st));
  return NIMF_OK;
}

// Device outputs -> host: outs[i] receives bytes[i] from src_dev + offset of
// the outputs before it (the device staging is contiguous).  Synchronises the
// stream.  Pageable outputs whose total fits the pinned stage come back in
// one copy and are spread on the host; otherwise host outputs that follow one
// another go back in one copy each run.
int copy_out_sync(float* const* outs, const size_t* bytes, int count, const void* src_dev,
                  cudaStream_t st) {
  size_t total = 0;
  bool pageable = false;
  for (int i = 0; i < count; ++i) {
    total += bytes[i];
    if (bytes[i] > 0 && !pageable) pageable = is_pageable(outs[i]);
  }
  if (total > 0 && pageable && total <= kHostStageMax) {
    NIMF_TRY(host_stage(g_hout, total));
    NIMF_CUDA_TRY(cudaMemcpyAsync(g_hout.p, src_dev, total, cudaMemcpyDeviceToHost, st));
    g_hout.busy = true;
    NIMF_CUDA_TRY(cudaStreamSynchronize(st));
    g_hout.busy = false;
    g_hin.busy = false;
    size_t off = 0;
    for (int i = 0; i < count; ++i) {
      if (bytes[i] > 0) std::memcpy(outs[i], (const char*)g_hout.p + off, bytes[i]);
      off += bytes[i];
    }
    return NIMF_OK;
  }
  const char* src = (const char*)src_dev;
  for (int i = 0; i < count;) {
    if (bytes[i] == 0) {
      ++i;
      continue;
    }
    size_t n = bytes[i];
    int j = i + 1;
    while (j < count && bytes[j] > 0 && (const char*)outs[j] == (const char*)outs[i] + n)
      n += bytes[j++];
    NIMF_CUDA_TRY(cudaMemcpyAsync(outs[i], src, n, cudaMemcpyDeviceToHost, st));
    src += n;
    i = j;
  }
  NIMF_CUDA_TRY(cudaStreamSynchronize(st));
  g_hin.busy = false;
  return NIMF_OK;
}
}  // namespace

int64_t Weight::rows() const {
  switch (kind) {
    case NIMF_KIND_INT4_ASYM: return q4.rows;
    case NIMF_KIND_INT8: return i8.rows;
    case NIMF_KIND_CUSTOM_FLOAT: return cf.rows;
    case NIMF_KIND_FP4_E2M1: return fp4.rows;
    case NIMF_KIND_F32: return f32.rows;
  }
  return 0;
}

int64_t Weight::k() const {
  switch (kind) {
    case NIMF_KIND_INT4_ASYM: return q4.k;
    case NIMF_KIND_INT8: return i8.k;
    case NIMF_KIND_CUSTOM_FLOAT: return cf.k;
    case NIMF_KIND_FP4_E2M1: return fp4.k;
    case NIMF_KIND_F32: return f32.k;
  }
  return 0;
}

void free_weight_storage(Weight* w) {
  device_free(w->q4.frag);
  device_free(w->q4.sz);
  device_free(w->q4.raw);
  device_free(w->q4.scales);
  device_free(w->q4.zeros);
  device_free(w->i8.q);
  device_free(w->i8.scales);
  device_free(w->cf.data);
  device_free(w->cf.row_scales);
  device_free(w->fp4.packed);
  device_free(w->fp4.bscale);
  device_free(w->f32.w);
  fw_free(&w->fw);
  device_free(w->kperm);
  w->kperm = nullptr;
  w->kperm_host.clear();
  w->q4 = Q4GWeight();
  w->i8 = I8Weight();
  w->cf = CFWeight();
  w->fp4 = FP4Weight();
  w->f32 = F32Weight();
}

Weight* lookup(nimf_weight_t h) {
  auto it = g_weights.find(h);
  return it == g_weights.end() ? nullptr : it->second.get();
}

nimf_weight_t insert(std::unique_ptr<Weight> w) {
  nimf_weight_t h = g_next++;
  g_weights.emplace(h, std::move(w));
  return h;
}

// Temporary device copies of host arrays used while building a weight.
struct TempBuffers {
  std::vector<void*> ptrs;
  ~TempBuffers() {
    for (void* p : ptrs) device_free(p);
  }
  int upload(const void* host, size_t bytes, void** dev, cudaStream_t st) {
    NIMF_TRY(device_alloc(dev, bytes));
    ptrs.push_back(*dev);
    if (bytes) NIMF_CUDA_TRY(cudaMemcpyAsync(*dev, host, bytes, cudaMemcpyHostToDevice, st));
    return NIMF_OK;
  }
};

static int check_rows(int64_t n, int64_t row_begin, int64_t row_end) {
  if (n < 0 || row_begin < 0 || row_end < row_begin || row_end > n)
    return set_error(NIMF_ERR_SHAPE, "row range [%lld, %lld) outside [0, %lld)",
                     (long long)row_begin, (long long)row_end, (long long)n);
  return NIMF_OK;
}

static int64_t fw_bytes(const FWLayout& L) {
  if (L.fmt < 0) return 0;
  return L.n_rt * L.ntk * 512 + (L.fmt == FW_FP4 ? L.n_rt * L.ntk * 64 : 0);
}

static int finish_register(std::unique_ptr<Weight> w, nimf_weight_t* out) {
  NIMF_CUDA_TRY(cudaStreamSynchronize(g_ctx.stream));
  NIMF_CUDA_TRY(cudaGetLastError());
  *out = insert(std::move(w));
  return NIMF_OK;
}

// Byte-coded float weights: decode GEMV for up to 16 rows of x, the tcgen05
// GEMM above (at K=8192, N=28672: the GEMV takes 86 us for 16 rows where the
// GEMM takes 141 us, and the GEMM 135 us for 17).
static int fw_matmul(const FWLayout& L, const float* x, int64_t m, float* y, cudaStream_t st) {
  return m > 16 ? fw_gemm_tc(L, x, m, y, st) : fw_gemv(L, x, m, y, st);
}

// Runs the kernel path of a weight on device buffers.
static int matmul_dev(Weight* w, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (w->kperm && m > 0 && w->k() > 0) {
    const float* xg = nullptr;
    NIMF_TRY(gather_cols(x, m, w->k(), (const int32_t*)w->kperm, &xg, st));
    x = xg;
  }
  switch (w->kind) {
    case NIMF_KIND_INT4_ASYM: return q4g_gemv(w->q4, x, m, y, st);
    case NIMF_KIND_INT8:
      return w->fw.fmt >= 0 ? fw_matmul(w->fw, x, m, y, st) : i8_gemv(w->i8, x, m, y, st);
    case NIMF_KIND_CUSTOM_FLOAT:
      return w->fw.fmt >= 0 ? fw_matmul(w->fw, x, m, y, st) : cf_gemv(w->cf, x, m, y, st);
    case NIMF_KIND_FP4_E2M1:
      return w->fw.fmt >= 0 ? fw_matmul(w->fw, x, m, y, st) : fp4_gemv(w->fp4, x, m, y, st);
    case NIMF_KIND_F32: return f32_gemm(x, m, w->f32.k, (const float*)w->f32.w, w->f32.rows, y, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "weight kind %d has no matmul path", w->kind);
}

int weight_matmul_dev(Weight* w, const float* x, int64_t m, float* y, cudaStream_t st) {
  return matmul_dev(w, x, m, y, st);
}

}  // namespace nimf

using namespace nimf;

extern "C" {

const char* nimf_last_error(void) { return g_err; }

int nimf_device_count(int* count) {
  if (!count) return set_error(NIMF_ERR_ARG, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    return set_error(NIMF_ERR_CUDA, "cudaGetDeviceCount failed: %s", cudaGetErrorString(e));
  }
  *count = n;
  return NIMF_OK;
}

int nimf_init(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_ready) {
    if (device == g_ctx.device) return NIMF_OK;
    return set_error(NIMF_ERR_STATE, "already initialised on device %d (asked %d)", g_ctx.device,
                     device);
  }
  int n = 0;
  NIMF_CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n)
    return set_error(NIMF_ERR_ARG, "device %d not in [0, %d)", device, n);
  NIMF_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  NIMF_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10)
    return set_error(NIMF_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                     device, prop.major, prop.minor);
  g_ctx = Context();
  g_ctx.device = device;
  g_ctx.num_sms = prop.multiProcessorCount;
  NIMF_CUDA_TRY(cudaStreamCreateWithFlags(&g_ctx.stream, cudaStreamNonBlocking));
  void* he = nullptr;
  NIMF_CUDA_TRY(cudaHostAlloc(&he, sizeof(int), cudaHostAllocMapped));
  *(volatile int*)he = 0;
  g_ctx.host_err = (volatile int*)he;
  NIMF_CUDA_TRY(cudaHostGetDevicePointer((void**)&g_ctx.dev_err, he, 0));
  g_ready = true;
  return NIMF_OK;
}

int nimf_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ready) return NIMF_OK;
  cudaSetDevice(g_ctx.device);
  cudaStreamSynchronize(g_ctx.stream);
  for (auto& kv : g_weights) free_weight_storage(kv.second.get());
  g_weights.clear();
  g_q4_cache.clear();
  fw_release_scratch();
  release_perm_buffer();
  release_attn_buffer();
  release_prep_buffers();
  release_decode_plans();
  release_p2p_groups();
  release_comm();
  release_f32_scratch();
  device_free(g_ctx.stage_in);
  device_free(g_ctx.stage_out);
  release_host_stages();
  if (g_ctx.host_err) cudaFreeHost((void*)g_ctx.host_err);
  cudaStreamDestroy(g_ctx.stream);
  g_ctx = Context();
  g_ready = false;
  return NIMF_OK;
}

int nimf_alloc_count(int64_t* count) {
  if (!count) return set_error(NIMF_ERR_ARG, "NULL output");
  *count = g_alloc_count.load(std::memory_order_relaxed);
  return NIMF_OK;
}

int nimf_sync(void) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  NIMF_CUDA_TRY(cudaDeviceSynchronize());
  return check_device_error();
}

// ------------------------------------------------------------------ weights

int nimf_weight_register_q4g(const uint8_t* wq, const float* scales, const float* zeros,
                             int64_t n, int64_t k, int64_t group_size,
                             int64_t n_groups_per_row, int64_t row_begin, int64_t row_end,
                             nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (k < 0) return set_error(NIMF_ERR_SHAPE, "k = %lld < 0", (long long)k);
  NIMF_TRY(check_rows(n, row_begin, row_end));
  const int64_t need = group_size > 0 ? (k + group_size - 1) / group_size : 1;
  if (n_groups_per_row < need)
    return set_error(NIMF_ERR_SHAPE, "n_groups_per_row = %lld < ceil(K/group_size) = %lld",
                     (long long)n_groups_per_row, (long long)need);
  if ((n * k > 0) && (!wq || !scales || !zeros))
    return set_error(NIMF_ERR_ARG, "NULL weight array");
  const int64_t bpr = (k + 1) / 2;
  const int64_t rows = row_end - row_begin;
  auto w = std::make_unique<Weight>();
  w->row_begin = row_begin;
  w->n_full = n;
  w->kind = NIMF_KIND_INT4_ASYM;
  TempBuffers tmp;
  void *dq = nullptr, *ds = nullptr, *dz = nullptr;
  // upload only the shard's rows
  NIMF_TRY(tmp.upload(wq ? wq + row_begin * bpr : nullptr, (size_t)(rows * bpr), &dq, c->stream));
  NIMF_TRY(tmp.upload(scales ? scales + row_begin * n_groups_per_row : nullptr,
                      (size_t)(rows * n_groups_per_row) * 4, &ds, c->stream));
  NIMF_TRY(tmp.upload(zeros ? zeros + row_begin * n_groups_per_row : nullptr,
                      (size_t)(rows * n_groups_per_row) * 4, &dz, c->stream));
  int st = q4g_build(w.get(), (const uint8_t*)dq, (const float*)ds, (const float*)dz, 0, rows, n,
                     k, group_size, n_groups_per_row, c->stream);
  if (st != NIMF_OK) {
    free_weight_storage(w.get());
    return st;
  }
  return finish_register(std::move(w), out);
}

int nimf_weight_register_i8(const int8_t* q, const float* scales, int64_t n_scales, int64_t n,
                            int64_t k, int64_t row_begin, int64_t row_end, nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (k < 0) return set_error(NIMF_ERR_SHAPE, "k < 0");
  NIMF_TRY(check_rows(n, row_begin, row_end));
  if (n_scales != 1 && n_scales != n)
    return set_error(NIMF_ERR_SHAPE, "n_scales = %lld must be 1 or N = %lld", (long long)n_scales,
                     (long long)n);
  if (!scales || ((n * k > 0) && !q)) return set_error(NIMF_ERR_ARG, "NULL weight array");
  const int64_t rows = row_end - row_begin;
  auto w = std::make_unique<Weight>();
  w->row_begin = row_begin;
  w->n_full = n;
  w->kind = NIMF_KIND_INT8;
  I8Weight& d = w->i8;
  d.rows = rows;
  d.k = k;
  d.n_scales = n_scales == 1 ? 1 : rows;
  NIMF_TRY(device_alloc(&d.q, (size_t)(rows * k)));
  NIMF_TRY(device_alloc(&d.scales, (size_t)d.n_scales * 4));
  if (rows * k > 0)
    NIMF_CUDA_TRY(cudaMemcpyAsync(d.q, q + row_begin * k, (size_t)(rows * k),
                                  cudaMemcpyHostToDevice, c->stream));
  NIMF_CUDA_TRY(cudaMemcpyAsync(d.scales, n_scales == 1 ? scales : scales + row_begin,
                                (size_t)d.n_scales * 4, cudaMemcpyHostToDevice, c->stream));
  w->device_bytes = rows * k + d.n_scales * 4;
  {
    int st = fw_build(&w->fw, FW_I8, d.q, nullptr, d.n_scales == 1 ? nullptr : (const float*)d.scales,
                      n_scales == 1 ? scales[0] : 1.0f, rows, k, c->stream);
    if (st != NIMF_OK) {
      free_weight_storage(w.get());
      return st;
    }
    w->device_bytes += fw_bytes(w->fw);
  }
  return finish_register(std::move(w), out);
}

int nimf_weight_register_cf(const uint8_t* data, int e, int m, const float* row_scales,
                            int64_t n, int64_t k, int64_t row_begin, int64_t row_end,
                            nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (e < 0 || m < 0 || 1 + e + m > 64)
    return set_error(NIMF_ERR_UNSUPPORTED, "CustomFloat e=%d m=%d: total bits must be <= 64", e, m);
  if (k < 0) return set_error(NIMF_ERR_SHAPE, "k < 0");
  NIMF_TRY(check_rows(n, row_begin, row_end));
  if ((n * k > 0) && !data) return set_error(NIMF_ERR_ARG, "NULL weight array");
  const int item = (1 + e + m + 7) / 8;
  const int64_t rows = row_end - row_begin;
  auto w = std::make_unique<Weight>();
  w->row_begin = row_begin;
  w->n_full = n;
  w->kind = NIMF_KIND_CUSTOM_FLOAT;
  CFWeight& d = w->cf;
  d.rows = rows;
  d.k = k;
  d.e = e;
  d.m = m;
  d.item = item;
  const size_t nb = (size_t)(rows * k * item);
  NIMF_TRY(device_alloc(&d.data, nb));
  if (nb)
    NIMF_CUDA_TRY(cudaMemcpyAsync(d.data, data + row_begin * k * item, nb, cudaMemcpyHostToDevice,
                                  c->stream));
  w->device_bytes = (int64_t)nb;
  if (row_scales) {
    NIMF_TRY(device_alloc(&d.row_scales, (size_t)rows * 4));
    NIMF_CUDA_TRY(cudaMemcpyAsync(d.row_scales, row_scales + row_begin, (size_t)rows * 4,
                                  cudaMemcpyHostToDevice, c->stream));
    w->device_bytes += rows * 4;
  }
  // one-byte E4M3 / E5M2 codes that decode exactly like OCP FP8: tensor-core GEMV
  if (item == 1 && ((e == 4 && m == 3) || (e == 5 && m == 2))) {
    int64_t special = 0;
    int st = fw_count_special_codes((const uint8_t*)d.data, rows * k, m, &special, c->stream);
    if (st == NIMF_OK && special == 0)
      st = fw_build(&w->fw, e == 4 ? FW_E4M3 : FW_E5M2, d.data, nullptr,
                    (const float*)d.row_scales, 1.0f, rows, k, c->stream);
    if (st != NIMF_OK) {
      free_weight_storage(w.get());
      return st;
    }
    w->device_bytes += fw_bytes(w->fw);
  }
  return finish_register(std::move(w), out);
}

int nimf_weight_register_fp4(const uint8_t* packed, const uint8_t* block_scales,
                             float tensor_scale, int64_t n, int64_t k, int64_t row_begin,
                             int64_t row_end, nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (k < 0) return set_error(NIMF_ERR_SHAPE, "k < 0");
  NIMF_TRY(check_rows(n, row_begin, row_end));
  if ((n * k > 0) && (!packed || !block_scales)) return set_error(NIMF_ERR_ARG, "NULL array");
  const int64_t rows = row_end - row_begin;
  const int64_t bpr = (k + 1) / 2, nb = (k + 15) / 16;
  auto w = std::make_unique<Weight>();
  w->row_begin = row_begin;
  w->n_full = n;
  w->kind = NIMF_KIND_FP4_E2M1;
  FP4Weight& d = w->fp4;
  d.rows = rows;
  d.k = k;
  d.tensor_scale = tensor_scale;
  NIMF_TRY(device_alloc(&d.packed, (size_t)(rows * bpr)));
  NIMF_TRY(device_alloc(&d.bscale, (size_t)(rows * nb)));
  if (rows * bpr > 0)
    NIMF_CUDA_TRY(cudaMemcpyAsync(d.packed, packed + row_begin * bpr, (size_t)(rows * bpr),
                                  cudaMemcpyHostToDevice, c->stream));
  if (rows * nb > 0)
    NIMF_CUDA_TRY(cudaMemcpyAsync(d.bscale, block_scales + row_begin * nb, (size_t)(rows * nb),
                                  cudaMemcpyHostToDevice, c->stream));
  w->device_bytes = rows * bpr + rows * nb;
  {
    int st = fw_build(&w->fw, FW_FP4, d.packed, d.bscale, nullptr, tensor_scale, rows, k, c->stream);
    if (st != NIMF_OK) {
      free_weight_storage(w.get());
      return st;
    }
    w->device_bytes += fw_bytes(w->fw);
  }
  return finish_register(std::move(w), out);
}

int nimf_weight_register_f32(const float* b_kn, int64_t k, int64_t n, nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (k < 0 || n < 0) return set_error(NIMF_ERR_SHAPE, "negative shape");
  if ((n * k > 0) && !b_kn) return set_error(NIMF_ERR_ARG, "NULL weight array");
  auto w = std::make_unique<Weight>();
  w->kind = NIMF_KIND_F32;
  w->f32.rows = n;
  w->f32.k = k;
  // stored as given, [K][N] row-major (beMatmul's b)
  NIMF_TRY(device_alloc(&w->f32.w, (size_t)(k * n) * 4));
  if (k * n > 0)
    NIMF_CUDA_TRY(cudaMemcpyAsync(w->f32.w, b_kn, (size_t)(k * n) * 4, cudaMemcpyHostToDevice,
                                  c->stream));
  w->device_bytes = k * n * 4;
  return finish_register(std::move(w), out);
}

int nimf_weight_free(nimf_weight_t h) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  free_weight_storage(w);
  g_weights.erase(h);
  for (auto it = g_q4_cache.begin(); it != g_q4_cache.end();) {
    if (it->second.handle == h) it = g_q4_cache.erase(it);
    else ++it;
  }
  return NIMF_OK;
}

int nimf_weight_info(nimf_weight_t h, int64_t* n_rows, int64_t* k, int* kind,
                     int64_t* device_bytes) {
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  if (n_rows) *n_rows = w->rows();
  if (k) *k = w->k();
  if (kind) *kind = w->kind;
  if (device_bytes) *device_bytes = w->device_bytes;
  return NIMF_OK;
}

// ------------------------------------------------------------------ matmul

int nimf_matmul_w_dev(nimf_weight_t h, const float* x_dev, int64_t m, float* y_dev,
                      void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  if (m < 0) return set_error(NIMF_ERR_SHAPE, "m < 0");
  if (m == 0 || w->rows() == 0) return NIMF_OK;
  if (!y_dev || (!x_dev && w->k() > 0)) return set_error(NIMF_ERR_ARG, "NULL x or y");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  return matmul_dev(w, x_dev, m, y_dev, st);
}

int nimf_matmul_w(nimf_weight_t h, const float* x, int64_t m, float* y) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  if (m < 0) return set_error(NIMF_ERR_SHAPE, "m < 0");
  const int64_t rows = w->rows(), k = w->k();
  if (m == 0 || rows == 0) return NIMF_OK;
  if (!y || (!x && k > 0)) return set_error(NIMF_ERR_ARG, "NULL x or y");
  void *dx, *dy;
  NIMF_TRY(stage_in((size_t)(m * k) * 4, &dx));
  NIMF_TRY(stage_out((size_t)(m * rows) * 4, &dy));
  NIMF_TRY(copy_in(dx, x, (size_t)(m * k) * 4, c->stream));
  NIMF_TRY(matmul_dev(w, (const float*)dx, m, (float*)dy, c->stream));
  const size_t yb = (size_t)(m * rows) * 4;
  NIMF_TRY(copy_out_sync(&y, &yb, 1, dy, c->stream));
  return check_device_error();
}

int nimf_matmul_w_group_dev(const nimf_weight_t* handles, int count, const float* x_dev,
                            int64_t m, float* const* y_devs, void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (count < 0 || m < 0) return set_error(NIMF_ERR_SHAPE, "negative count or m");
  if (count == 0 || m == 0) return NIMF_OK;
  if (!handles || !y_devs) return set_error(NIMF_ERR_ARG, "NULL handle or output array");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  std::vector<Weight*> ws((size_t)count);
  bool all_q4 = true;
  for (int i = 0; i < count; ++i) {
    ws[i] = lookup(handles[i]);
    if (!ws[i])
      return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)handles[i]);
    if (ws[i]->k() != ws[0]->k())
      return set_error(NIMF_ERR_SHAPE, "grouped matmul: weights have different K");
    if (!y_devs[i] && ws[i]->rows() > 0) return set_error(NIMF_ERR_ARG, "NULL output %d", i);
    all_q4 = all_q4 && ws[i]->kind == NIMF_KIND_INT4_ASYM && ws[i]->q4.gs == ws[0]->q4.gs &&
             ws[i]->q4.fast == ws[0]->q4.fast && !ws[i]->kperm;
  }
  if (!x_dev && ws[0]->k() > 0) return set_error(NIMF_ERR_ARG, "NULL x");
  if (all_q4) {
    std::vector<const Q4GWeight*> qs((size_t)count);
    for (int i = 0; i < count; ++i) qs[i] = &ws[i]->q4;
    return q4g_gemv_group(qs.data(), count, x_dev, m, y_devs, st);
  }
  for (int i = 0; i < count; ++i)
    if (ws[i]->rows() > 0) NIMF_TRY(matmul_dev(ws[i], x_dev, m, y_devs[i], st));
  return NIMF_OK;
}

int nimf_matmul_w_group(const nimf_weight_t* handles, int count, const float* x, int64_t m,
                        float* const* ys) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (count < 0 || m < 0) return set_error(NIMF_ERR_SHAPE, "negative count or m");
  if (count == 0 || m == 0) return NIMF_OK;
  if (!handles || !ys) return set_error(NIMF_ERR_ARG, "NULL handle or output array");
  int64_t k = -1, total = 0;
  std::vector<int64_t> rows((size_t)count);
  for (int i = 0; i < count; ++i) {
    Weight* w = lookup(handles[i]);
    if (!w)
      return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)handles[i]);
    if (k >= 0 && w->k() != k) return set_error(NIMF_ERR_SHAPE, "grouped matmul: different K");
    k = w->k();
    rows[i] = w->rows();
    total += rows[i];
    if (!ys[i] && rows[i] > 0) return set_error(NIMF_ERR_ARG, "NULL output %d", i);
  }
  if (!x && k > 0) return set_error(NIMF_ERR_ARG, "NULL x");
  void *dx, *dy;
  NIMF_TRY(stage_in((size_t)(m * k) * 4, &dx));
  NIMF_TRY(stage_out((size_t)(m * total) * 4, &dy));
  std::vector<float*> yd((size_t)count);
  int64_t off = 0;
  for (int i = 0; i < count; ++i) {
    yd[i] = (float*)dy + off;
    off += m * rows[i];
  }
  NIMF_TRY(copy_in(dx, x, (size_t)(m * k) * 4, c->stream));
  NIMF_TRY(nimf_matmul_w_group_dev(handles, count, (const float*)dx, m, yd.data(), c->stream));
  // The staged outputs are contiguous: they come back in one copy when they
  // are pageable and small, else in one copy per run of host buffers that
  // follow one another (each copy costs a few microseconds of set-up, more
  // than moving one projection's y).
  std::vector<size_t> yb((size_t)count);
  for (int i = 0; i < count; ++i) yb[i] = (size_t)(m * rows[i]) * 4;
  NIMF_TRY(copy_out_sync(ys, yb.data(), count, dy, c->stream));
  return check_device_error();
}

int nimf_dequant_w(nimf_weight_t h, float* out_host) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  const int64_t n = w->rows() * w->k();
  if (n == 0) return NIMF_OK;
  if (!out_host) return set_error(NIMF_ERR_ARG, "out is NULL");
  void* d;
  NIMF_TRY(stage_out((size_t)n * 4, &d));
  float* o = (float*)d;
  switch (w->kind) {
    case NIMF_KIND_INT4_ASYM: NIMF_TRY(q4g_dequant(w->q4, o, c->stream)); break;
    // formats with a tensor-core copy are read back from it, so the bit-exact
    // check covers the layout the GEMV streams
    case NIMF_KIND_INT8:
      NIMF_TRY(w->fw.fmt >= 0 ? fw_dequant(w->fw, o, c->stream) : i8_dequant(w->i8, o, c->stream));
      break;
    case NIMF_KIND_CUSTOM_FLOAT:
      NIMF_TRY(w->fw.fmt >= 0 ? fw_dequant(w->fw, o, c->stream) : cf_dequant(w->cf, o, c->stream));
      break;
    case NIMF_KIND_FP4_E2M1:
      NIMF_TRY(w->fw.fmt >= 0 ? fw_dequant(w->fw, o, c->stream) : fp4_dequant(w->fp4, o, c->stream));
      break;
    case NIMF_KIND_F32:
      NIMF_TRY(f32_transpose((const float*)w->f32.w, w->f32.k, w->f32.rows, o, c->stream));
      break;
    default: return set_error(NIMF_ERR_UNSUPPORTED, "kind %d", w->kind);
  }
  NIMF_CUDA_TRY(cudaMemcpyAsync(out_host, o, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (!w->kperm_host.empty()) {
    // stored column j is input feature kperm[j]: back to the reference order
    const int64_t k = w->k();
    std::vector<float> row((size_t)k);
    for (int64_t r = 0; r < w->rows(); ++r) {
      float* o_r = out_host + r * k;
      std::copy(o_r, o_r + k, row.begin());
      for (int64_t j = 0; j < k; ++j) o_r[w->kperm_host[(size_t)j]] = row[(size_t)j];
    }
  }
  return NIMF_OK;
}

int nimf_matmul_q4(const float* a, const uint8_t* wq, const float* scales, const float* zeros,
                   int64_t m, int64_t k, int64_t n, int64_t group_size, int64_t n_groups_per_row,
                   float* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (m < 0 || k < 0 || n < 0) return set_error(NIMF_ERR_SHAPE, "negative shape");
  if (m == 0 || n == 0) return NIMF_OK;
  if (!wq || !scales || !zeros) return set_error(NIMF_ERR_ARG, "NULL weight array");
  const int64_t bytes = n * ((k + 1) / 2);
  const int64_t sbytes = n * std::max<int64_t>(n_groups_per_row, 0) * (int64_t)sizeof(float);
  const Q4Key key = std::make_tuple((uintptr_t)wq, (uintptr_t)scales, (uintptr_t)zeros, k, n,
                                    group_size, n_groups_per_row);
  const uint64_t fp = q4_fingerprint(wq, (size_t)bytes, scales, zeros, (size_t)sbytes, g_q4_check);
  nimf_weight_t h;
  auto it = g_q4_cache.find(key);
  if (it != g_q4_cache.end() && it->second.fingerprint == fp && lookup(it->second.handle)) {
    h = it->second.handle;
  } else {
    if (it != g_q4_cache.end()) {
      // same arrays, other contents: the old device copy is stale
      const nimf_weight_t old = it->second.handle;
      g_q4_cache.erase(it);
      if (lookup(old)) NIMF_TRY(nimf_weight_free(old));
    }
    NIMF_TRY(nimf_weight_register_q4g(wq, scales, zeros, n, k, group_size, n_groups_per_row, 0, n,
                                      &h));
    g_q4_cache[key] = Q4Entry{h, fp};
  }
  return nimf_matmul_w(h, a, m, out);
}

int nimf_q4_prefill_mode(int mode) {
  if (mode != NIMF_Q4_PREFILL_AUTO && mode != NIMF_Q4_PREFILL_EXACT)
    return set_error(NIMF_ERR_ARG, "q4_prefill_mode: %d is not AUTO (0) or EXACT (1)", mode);
  g_q4_prefill_mode = mode;
  return NIMF_OK;
}

int nimf_q4_cache_set_check(int mode) {
  if (mode != NIMF_Q4_CACHE_CHECK_FULL && mode != NIMF_Q4_CACHE_CHECK_SAMPLED &&
      mode != NIMF_Q4_CACHE_CHECK_NONE)
    return set_error(NIMF_ERR_ARG, "nimf_q4_cache_set_check: mode %d", mode);
  g_q4_check = mode;
  return NIMF_OK;
}

int nimf_q4_cache_size(int64_t* entries) {
  if (!entries) return set_error(NIMF_ERR_ARG, "NULL output");
  *entries = (int64_t)g_q4_cache.size();
  return NIMF_OK;
}

int nimf_weight_cache_clear(void) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  std::vector<nimf_weight_t> hs;
  for (auto& kv : g_q4_cache) hs.push_back(kv.second.handle);
  g_q4_cache.clear();
  for (nimf_weight_t h : hs)
    if (lookup(h)) NIMF_TRY(nimf_weight_free(h));
  return NIMF_OK;
}

int nimf_matmul_f32(const float* a, int64_t m, int64_t k, const float* b, int64_t k2, int64_t n,
                    float* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (k2 != k)
    return set_error(NIMF_ERR_SHAPE, "beMatmul: K = %lld but K2 = %lld", (long long)k,
                     (long long)k2);
  if (m < 0 || k < 0 || n < 0) return set_error(NIMF_ERR_SHAPE, "negative shape");
  if (m == 0 || n == 0) return NIMF_OK;
  if (!out || (k > 0 && (!a || !b))) return set_error(NIMF_ERR_ARG, "NULL array");
  const size_t ba = (size_t)(m * k) * 4, bb = (size_t)(k * n) * 4, bc = (size_t)(m * n) * 4;
  void *din, *dc;
  NIMF_TRY(stage_in(ba + bb + 256, &din));
  NIMF_TRY(stage_out(bc, &dc));
  float* da = (float*)din;
  float* db = (float*)((char*)din + ((ba + 255) / 256) * 256);
  if (ba) NIMF_CUDA_TRY(cudaMemcpyAsync(da, a, ba, cudaMemcpyHostToDevice, c->stream));
  if (bb) NIMF_CUDA_TRY(cudaMemcpyAsync(db, b, bb, cudaMemcpyHostToDevice, c->stream));
  NIMF_TRY(f32_gemm(da, m, k, db, n, (float*)dc, c->stream));
  NIMF_CUDA_TRY(cudaMemcpyAsync(out, dc, bc, cudaMemcpyDeviceToHost, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return NIMF_OK;
}

int nimf_matmul2_f32(const float* a1, int64_t m1, int64_t k1, const float* b1, int64_t k1b,
                     int64_t n1, const float* a2, int64_t m2, int64_t k2, const float* b2,
                     int64_t k2b, int64_t n2, float* out1, float* out2) {
  NIMF_TRY(nimf_matmul_f32(a1, m1, k1, b1, k1b, n1, out1));
  return nimf_matmul_f32(a2, m2, k2, b2, k2b, n2, out2);
}

// ------------------------------------------------------------------ CustomFloat / APF

static int cf_check(int e, int m) {
  if (e < 0 || m < 0) return set_error(NIMF_ERR_ARG, "negative exponent/mantissa bits");
  if (1 + e + m > 64)
    return set_error(NIMF_ERR_UNSUPPORTED,
                     "CustomFloat e=%d m=%d: encodeArray/decodeArray support total_bits <= 64", e,
                     m);
  return NIMF_OK;
}

int nimf_cf_encode_dev(const float* x_dev, int64_t n, int e, int m, uint8_t* out_dev,
                       void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  NIMF_TRY(cf_check(e, m));
  if (n < 0) return set_error(NIMF_ERR_SHAPE, "n < 0");
  if (n == 0) return NIMF_OK;
  if (!x_dev || !out_dev) return set_error(NIMF_ERR_ARG, "NULL buffer");
  return cf_encode(x_dev, n, e, m, out_dev, stream ? (cudaStream_t)stream : c->stream);
}

int nimf_cf_decode_dev(const uint8_t* buf_dev, int64_t nbytes, int e, int m, float* out_dev,
                       void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  NIMF_TRY(cf_check(e, m));
  const int item = (1 + e + m + 7) / 8;
  if (nbytes < 0 || nbytes % item != 0)
    return set_error(NIMF_ERR_SHAPE, "buffer of %lld bytes is not a multiple of itemSize %d",
                     (long long)nbytes, item);
  if (nbytes == 0) return NIMF_OK;
  if (!buf_dev || !out_dev) return set_error(NIMF_ERR_ARG, "NULL buffer");
  return cf_decode(buf_dev, nbytes / item, e, m, out_dev,
                   stream ? (cudaStream_t)stream : c->stream);
}

int nimf_cf_encode(const float* x, int64_t n, int e, int m, uint8_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  NIMF_TRY(cf_check(e, m));
  if (n < 0) return set_error(NIMF_ERR_SHAPE, "n < 0");
  if (n == 0) return NIMF_OK;
  if (!x || !out) return set_error(NIMF_ERR_ARG, "NULL buffer");
  const int item = (1 + e + m + 7) / 8;
  void *dx, *dy;
  NIMF_TRY(stage_in((size_t)n * 4, &dx));
  NIMF_TRY(stage_out((size_t)n * item, &dy));
  NIMF_CUDA_TRY(cudaMemcpyAsync(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
  NIMF_TRY(cf_encode((const float*)dx, n, e, m, (uint8_t*)dy, c->stream));
  NIMF_CUDA_TRY(cudaMemcpyAsync(out, dy, (size_t)n * item, cudaMemcpyDeviceToHost, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return NIMF_OK;
}

int nimf_cf_decode(const uint8_t* buf, int64_t nbytes, int e, int m, float* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  NIMF_TRY(cf_check(e, m));
  const int item = (1 + e + m + 7) / 8;
  if (nbytes < 0 || nbytes % item != 0)
    return set_error(NIMF_ERR_SHAPE, "buffer of %lld bytes is not a multiple of itemSize %d",
                     (long long)nbytes, item);
  if (nbytes == 0) return NIMF_OK;
  if (!buf || !out) return set_error(NIMF_ERR_ARG, "NULL buffer");
  const int64_t n = nbytes / item;
  void *dx, *dy;
  NIMF_TRY(stage_in((size_t)nbytes, &dx));
  NIMF_TRY(stage_out((size_t)n * 4, &dy));
  NIMF_CUDA_TRY(cudaMemcpyAsync(dx, buf, (size_t)nbytes, cudaMemcpyHostToDevice, c->stream));
  NIMF_TRY(cf_decode((const uint8_t*)dx, n, e, m, (float*)dy, c->stream));
  NIMF_CUDA_TRY(cudaMemcpyAsync(out, dy, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return NIMF_OK;
}

// customfloat.nim:149-198.  The reductions (min/max |x|, medians) run on the
// device; the final integer formulas run here in double exactly as the
// reference evaluates them.
int nimf_cf_autoselect(const float* x, int64_t n, const float* grad, int64_t n_grad,
                       double rel_error_tol, int exp_margin, int* exponent_bits,
                       int* mantissa_bits) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (n < 0 || n_grad < 0) return set_error(NIMF_ERR_SHAPE, "negative length");
  if (!exponent_bits || !mantissa_bits) return set_error(NIMF_ERR_ARG, "NULL output");
  if ((n > 0 && !x) || (n_grad > 0 && !grad)) return set_error(NIMF_ERR_ARG, "NULL input");
  float mn = 0.f, mx = 0.f;
  int found = 0;
  void* dx = nullptr;
  if (n > 0) {
    NIMF_TRY(stage_in((size_t)n * 4, &dx));
    NIMF_CUDA_TRY(cudaMemcpyAsync(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
    NIMF_TRY(cf_absrange((const float*)dx, n, &mn, &mx, &found, c->stream));
  }
  // computeRequiredExponentBits (customfloat.nim:149-165)
  int eb = 1;
  if (found) {
    const int64_t max_e = (int64_t)std::floor(std::log2((double)mx));
    const int64_t min_e = (int64_t)std::floor(std::log2((double)mn));
    const int64_t span = (max_e - min_e) + 2 * (int64_t)exp_margin + 2;
    const int64_t r = (int64_t)std::ceil(std::log2((double)std::max<int64_t>(span, 2)));
    eb = (int)std::max<int64_t>(1, r);
  }
  // computeRequiredMantissaBits (customfloat.nim:167-198)
  int mb = 2;
  if (found) {
    const int64_t base = (int64_t)std::ceil(std::log2(1.0 / std::max(rel_error_tol, 1e-12)));
    int64_t extra = 0;
    if (n_grad > 0) {
      float wmed = 0.f, gmed = 0.f;
      int64_t nv = 0, ng = 0;
      NIMF_TRY(cf_abs_median((const float*)dx, n, &wmed, &nv, c->stream));
      void* dg;
      NIMF_TRY(stage_out((size_t)n_grad * 4, &dg));
      NIMF_CUDA_TRY(
          cudaMemcpyAsync(dg, grad, (size_t)n_grad * 4, cudaMemcpyHostToDevice, c->stream));
      NIMF_TRY(cf_abs_median((const float*)dg, n_grad, &gmed, &ng, c->stream));
      if (ng > 0) {
        wmed = std::max(wmed, 1e-12f);
        const double ratio = (double)gmed / (double)wmed;
        if (ratio > 0 && ratio < 1) {
          const int64_t need = (int64_t)std::ceil(-std::log2(ratio));
          extra = std::max<int64_t>(0, need - base);
        }
      }
    }
    mb = (int)std::min<int64_t>(23, std::max<int64_t>(2, base + extra));
  }
  *exponent_bits = eb;
  *mantissa_bits = mb;
  return NIMF_OK;
}

int nimf_apf_cast(const float* x, int64_t n, const float* grad, int64_t n_grad,
                  double rel_error_tol, int exp_margin, int* exponent_bits, int* mantissa_bits,
                  uint8_t* out) {
  NIMF_TRY(nimf_cf_autoselect(x, n, grad, n_grad, rel_error_tol, exp_margin, exponent_bits,
                              mantissa_bits));
  return nimf_cf_encode(x, n, *exponent_bits, *mantissa_bits, out);
}

}  // extern "C"
