// cf.cu -- CustomFloat / APF (customfloat.nim) on the device: element encode
// and decode with the reference's exact bit rules, the reductions behind the
// APF auto-selection, and the GEMV over CustomFloat-encoded weights.
//
// Encode (customfloat.nim:49-78): truncating; exponent overflow, inf and NaN
// give the +-inf pattern (mantissa 0); underflow and zero give a signed zero;
// no subnormals.  Decode (customfloat.nim:80-102): exp == maxExp -> +-inf,
// exp == 0 && mant == 0 -> +-0, otherwise 2^(exp - bias) * 1.mant with the
// float32 exponent clamped to [0, 255].  Items are itemSize = ceil(total/8)
// little-endian bytes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

struct CFmt {
  int e, m, item, bias, max_exp;
  uint64_t mant_mask;
};

CFmt make_fmt(int e, int m) {
  CFmt f;
  f.e = e;
  f.m = m;
  f.item = (1 + e + m + 7) / 8;
  f.bias = e > 0 ? (1 << (e - 1)) - 1 : 0;
  f.max_exp = e > 0 ? (1 << e) - 1 : 0;
  f.mant_mask = m == 0 ? 0ull : ((m >= 64) ? ~0ull : ((1ull << m) - 1));
  return f;
}

__device__ __forceinline__ uint64_t cf_pack(float x, const CFmt f) {
  const uint32_t b = __float_as_uint(x);
  const uint64_t sign = (b >> 31) & 1u;
  const uint32_t exp32 = (b >> 23) & 0xFFu;
  const uint32_t mant32 = b & 0x7FFFFFu;
  const int real_exp = (int)exp32 - 127;
  const bool is_zero = exp32 == 0 && mant32 == 0;
  const bool is_inf_nan = exp32 == 255;
  const int new_exp = real_exp + f.bias;
  const bool overflow = new_exp >= f.max_exp && !is_zero;
  const bool underflow = new_exp <= 0 && !is_zero;
  const uint64_t top = (uint64_t)(f.e + f.m);
  if (is_inf_nan || overflow) return (sign << top) | ((uint64_t)f.max_exp << f.m);
  if (underflow || is_zero) return sign << top;
  const uint64_t mant =
      f.m <= 23 ? (uint64_t)(mant32 >> (23 - f.m)) : ((uint64_t)mant32 << (f.m - 23));
  const uint64_t ne = (uint64_t)min(max(new_exp, 0), f.max_exp);
  return (sign << top) | (ne << f.m) | mant;
}

__device__ __forceinline__ float cf_unpack(uint64_t p, const CFmt f) {
  const uint64_t top = (uint64_t)(f.e + f.m);
  const uint32_t sign = (uint32_t)((p >> top) & 1u);
  const uint64_t ex = (p >> f.m) & (uint64_t)f.max_exp;
  const uint64_t mant = p & f.mant_mask;
  if (ex == (uint64_t)f.max_exp) return __uint_as_float((sign << 31) | 0x7F800000u);
  if (ex == 0 && mant == 0) return __uint_as_float(sign << 31);
  const int e32 = min(max((int)ex - f.bias + 127, 0), 255);
  const uint32_t m32 = f.m <= 23 ? (uint32_t)(mant << (23 - f.m)) : (uint32_t)(mant >> (f.m - 23));
  return __uint_as_float((sign << 31) | ((uint32_t)e32 << 23) | m32);
}

__device__ __forceinline__ uint64_t load_item(const uint8_t* p, int item) {
  uint64_t v = 0;
  for (int b = 0; b < item; ++b) v |= (uint64_t)p[b] << (8 * b);
  return v;
}

constexpr int kChunk = 16;  // elements per thread in the vector kernels

// 16 elements per thread: 4 x 128-bit loads of fp32, 16*item bytes stored as
// item x 128-bit stores (16*item is a multiple of 16).  Requires 16-byte
// aligned x and out.
__global__ void cf_encode_vec(const float* __restrict__ x, int64_t nchunks, const CFmt f,
                              uint8_t* __restrict__ out) {
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const float4* xs = reinterpret_cast<const float4*>(x) + c * 4;
    float v[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 t = __ldg(xs + i);
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
    uint32_t words[32];  // up to 16 * 8 bytes = 32 words
    const int nw = 4 * f.item;
#pragma unroll
    for (int i = 0; i < 32; ++i) words[i] = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint64_t pk = cf_pack(v[i], f);
      const int bit0 = i * f.item * 8;
#pragma unroll 1
      for (int b = 0; b < f.item; ++b) {
        const uint32_t byte = (uint32_t)((pk >> (8 * b)) & 0xFFu);
        const int bit = bit0 + 8 * b;
        words[bit >> 5] |= byte << (bit & 31);
      }
    }
    uint4* o = reinterpret_cast<uint4*>(out + c * 16 * f.item);
    for (int i = 0; i < nw / 4; ++i)
      o[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
  }
}

__global__ void cf_encode_scalar(const float* __restrict__ x, int64_t i0, int64_t n, const CFmt f,
                                 uint8_t* __restrict__ out) {
  for (int64_t i = i0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t pk = cf_pack(x[i], f);
    for (int b = 0; b < f.item; ++b) out[i * f.item + b] = (uint8_t)((pk >> (8 * b)) & 0xFFu);
  }
}

__global__ void cf_decode_vec(const uint8_t* __restrict__ buf, int64_t nchunks, const CFmt f,
                              float* __restrict__ out) {
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    uint32_t words[32];
    const uint4* in = reinterpret_cast<const uint4*>(buf + c * 16 * f.item);
    for (int i = 0; i < f.item; ++i) {
      const uint4 t = __ldg(in + i);
      words[4 * i] = t.x; words[4 * i + 1] = t.y; words[4 * i + 2] = t.z; words[4 * i + 3] = t.w;
    }
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint64_t pk = 0;
      const int bit0 = i * f.item * 8;
#pragma unroll 1
      for (int b = 0; b < f.item; ++b) {
        const int bit = bit0 + 8 * b;
        pk |= (uint64_t)((words[bit >> 5] >> (bit & 31)) & 0xFFu) << (8 * b);
      }
      v[i] = cf_unpack(pk, f);
    }
    float4* o = reinterpret_cast<float4*>(out) + c * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

__global__ void cf_decode_scalar(const uint8_t* __restrict__ buf, int64_t i0, int64_t n,
                                 const CFmt f, float* __restrict__ out) {
  for (int64_t i = i0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = cf_unpack(load_item(buf + i * f.item, f.item), f);
}

// min / max over |x| for finite non-zero x, as float bit patterns (ordered
// like unsigned integers for non-negative floats).
__global__ void absrange_kernel(const float* __restrict__ x, int64_t n, unsigned* mm) {
  unsigned lo = 0x7F800000u, hi = 0u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned b = __float_as_uint(x[i]) & 0x7FFFFFFFu;
    if (b != 0u && b < 0x7F800000u) {
      lo = min(lo, b);
      hi = max(hi, b);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&mm[0], lo);
    atomicMax(&mm[1], hi);
  }
}

// Histogram of an 11/11/10-bit digit of |x| bits for finite non-zero x whose
// higher bits equal `prefix` (radix selection of the median).
__global__ void radix_hist_kernel(const float* __restrict__ x, int64_t n, int shift, int bits,
                                  unsigned prefix, int prefix_shift, unsigned* __restrict__ hist) {
  __shared__ unsigned sh[2048];
  const int nb = 1 << bits;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned b = __float_as_uint(x[i]) & 0x7FFFFFFFu;
    if (b == 0u || b >= 0x7F800000u) continue;
    if (prefix_shift < 32 && (b >> prefix_shift) != prefix) continue;
    atomicAdd(&sh[(b >> shift) & (nb - 1)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nb; i += blockDim.x)
    if (sh[i]) atomicAdd(&hist[i], sh[i]);
}

// Warp per row GEMV over CustomFloat items (any format).
__global__ void cf_gemv_generic(const uint8_t* __restrict__ data, const float* __restrict__ rs,
                                int64_t rows, int64_t k, const CFmt f, const float* __restrict__ x,
                                int m, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = warp; row < rows; row += nwarps) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const uint8_t* rp = data + row * k * f.item;
    for (int64_t c = lane; c < k; c += 32) {
      const float w = cf_unpack(load_item(rp + c * f.item, f.item), f);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < m) acc[i] = fmaf(w, x[i * k + c], acc[i]);
    }
    const float s = rs ? rs[row] : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < m) {
        const float v = warp_sum(acc[i]);
        if (lane == 0) y[i * rows + row] = v * s;
      }
    }
  }
}

__global__ void cf_dequant_kernel(const uint8_t* __restrict__ data, const float* __restrict__ rs,
                                  int64_t rows, int64_t k, const CFmt f, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * k;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = cf_unpack(load_item(data + i * f.item, f.item), f);
    out[i] = rs ? __fmul_rn(v, rs[i / k]) : v;
  }
}

unsigned grid_for(int64_t work, int block) {
  Context* c = ctx();
  const int64_t cap = (int64_t)(c ? c->num_sms : 148) * 8;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, (work + block - 1) / block));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Small per-context device scratch for the reductions.
void* g_scratch = nullptr;
int g_scratch_dev = -1;
int scratch(void** p) {
  Context* c = ctx();
  if (!g_scratch || g_scratch_dev != c->device) {
    NIMF_TRY(device_alloc(&g_scratch, 2048 * sizeof(unsigned)));
    g_scratch_dev = c->device;
  }
  *p = g_scratch;
  return NIMF_OK;
}

}  // namespace

int cf_encode(const float* x, int64_t n, int e, int m, uint8_t* out, cudaStream_t st) {
  const CFmt f = make_fmt(e, m);
  int64_t done = 0;
  if (aligned16(x) && aligned16(out)) {
    const int64_t nch = n / kChunk;
    if (nch > 0) cf_encode_vec<<<grid_for(nch, 256), 256, 0, st>>>(x, nch, f, out);
    done = nch * kChunk;
  }
  if (done < n) cf_encode_scalar<<<grid_for(n - done, 256), 256, 0, st>>>(x, done, n, f, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int cf_decode(const uint8_t* buf, int64_t n, int e, int m, float* out, cudaStream_t st) {
  const CFmt f = make_fmt(e, m);
  int64_t done = 0;
  if (aligned16(buf) && aligned16(out)) {
    const int64_t nch = n / kChunk;
    if (nch > 0) cf_decode_vec<<<grid_for(nch, 256), 256, 0, st>>>(buf, nch, f, out);
    done = nch * kChunk;
  }
  if (done < n) cf_decode_scalar<<<grid_for(n - done, 256), 256, 0, st>>>(buf, done, n, f, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int cf_absrange(const float* x, int64_t n, float* min_abs, float* max_abs, int* found,
                cudaStream_t st) {
  void* s;
  NIMF_TRY(scratch(&s));
  const unsigned init[2] = {0x7F800000u, 0u};
  NIMF_CUDA_TRY(cudaMemcpyAsync(s, init, sizeof(init), cudaMemcpyHostToDevice, st));
  absrange_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, (unsigned*)s);
  NIMF_CUDA_TRY(cudaGetLastError());
  unsigned r[2];
  NIMF_CUDA_TRY(cudaMemcpyAsync(r, s, sizeof(r), cudaMemcpyDeviceToHost, st));
  NIMF_CUDA_TRY(cudaStreamSynchronize(st));
  *found = r[1] != 0u;
  *min_abs = __builtin_bit_cast(float, r[0]);
  *max_abs = __builtin_bit_cast(float, r[1]);
  return NIMF_OK;
}

int cf_abs_median(const float* x, int64_t n, float* median, int64_t* n_valid, cudaStream_t st) {
  void* s;
  NIMF_TRY(scratch(&s));
  unsigned* hist = (unsigned*)s;
  // 31 significant bits of |x|: digits of 11, 11, 9 bits from the top.
  const int shifts[3] = {20, 9, 0};
  const int widths[3] = {11, 11, 9};
  unsigned prefix = 0;
  int prefix_shift = 32;
  int64_t want = -1, total = 0;
  std::vector<unsigned> h(2048);
  for (int pass = 0; pass < 3; ++pass) {
    const int nb = 1 << widths[pass];
    NIMF_CUDA_TRY(cudaMemsetAsync(hist, 0, nb * sizeof(unsigned), st));
    radix_hist_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, shifts[pass], widths[pass], prefix,
                                                        prefix_shift, hist);
    NIMF_CUDA_TRY(cudaGetLastError());
    NIMF_CUDA_TRY(cudaMemcpyAsync(h.data(), hist, nb * sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    NIMF_CUDA_TRY(cudaStreamSynchronize(st));
    if (pass == 0) {
      for (int i = 0; i < nb; ++i) total += h[i];
      *n_valid = total;
      if (total == 0) {
        *median = 0.0f;
        return NIMF_OK;
      }
      want = total / 2;  // Nim: s[s.len div 2] of the ascending sort
    }
    int64_t acc = 0;
    int sel = nb - 1;
    for (int i = 0; i < nb; ++i) {
      if (acc + h[i] > want) { sel = i; break; }
      acc += h[i];
    }
    want -= acc;
    prefix = (prefix << widths[pass]) | (unsigned)sel;
    prefix_shift = shifts[pass];
  }
  *median = __builtin_bit_cast(float, prefix);
  return NIMF_OK;
}

int cf_gemv(const CFWeight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  const CFmt f = make_fmt(w.e, w.m);
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    cf_gemv_generic<<<grid_for(w.rows * 32, 256), 256, 0, st>>>(
        (const uint8_t*)w.data, (const float*)w.row_scales, w.rows, w.k, f, x + m0 * w.k, mc,
        y + m0 * w.rows);
  }
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int cf_dequant(const CFWeight& w, float* out, cudaStream_t st) {
  const CFmt f = make_fmt(w.e, w.m);
  cf_dequant_kernel<<<grid_for(w.rows * w.k, 256), 256, 0, st>>>(
      (const uint8_t*)w.data, (const float*)w.row_scales, w.rows, w.k, f, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

}  // namespace nimf

// ---------------------------------------------------------------------------
// Allocation-free APF format selection on device buffers.
//
// For callers that cannot call cudaMalloc: a host that hands the GPU's whole
// memory to its own allocator (a serving process that reserves it at start-up)
// and forbids any other allocation, or one that must not add allocations while
// a step runs.  The existing nimf_cf_autoselect stages x in buffers the
// library allocates and keeps its reduction scratch in another allocated
// buffer; this variant reads the caller's device buffers and keeps its scratch
// in the fixed array below.  It copies its reductions back to the host and
// synchronises the stream, so a call on a stream that is being captured
// returns NIMF_ERR_STATE without touching the capture.
//
// Scratch: g_noalloc_scratch holds 2 + 2048 32-bit words (8,200 bytes):
// word 0 / 1 are the min / max of |x| (as float bits), words 2.. a radix
// histogram.  Every GPU that loads the library holds it until the process
// exits.  All calls share it, so calls that overlap on the GPU race; each call
// clears what must start at zero before using it.  Element counts are limited
// to 2^31 - 1 (the histogram counts are 32-bit).
namespace nimf {
namespace {

constexpr int kNoAllocWords = 2 + 2048;
constexpr int64_t kNoAllocMaxElems = 2147483647LL;
static __device__ __align__(256) unsigned g_noalloc_scratch[kNoAllocWords];
// Device address of g_noalloc_scratch, per device.  In host code the array's
// name is only a host-side stand-in, never a device address.
unsigned* g_noalloc_addr[64] = {};

__global__ void noalloc_minmax_init(unsigned* s) {
  s[0] = 0x7F800000u;
  s[1] = 0u;
}

// Median of |v| over finite non-zero v (element n_valid/2 of the ascending
// order), by three radix-histogram passes in the scratch histogram.
int noalloc_abs_median(const float* v, int64_t n, unsigned* hist, float* median,
                       int64_t* n_valid, cudaStream_t st) {
  const int shifts[3] = {20, 9, 0};
  const int widths[3] = {11, 11, 9};
  unsigned prefix = 0;
  int prefix_shift = 32;
  int64_t want = -1, total = 0;
  unsigned h[2048];
  for (int pass = 0; pass < 3; ++pass) {
    const int nb = 1 << widths[pass];
    NIMF_CUDA_TRY(cudaMemsetAsync(hist, 0, nb * sizeof(unsigned), st));
    radix_hist_kernel<<<grid_for(n, 256), 256, 0, st>>>(v, n, shifts[pass], widths[pass], prefix,
                                                        prefix_shift, hist);
    NIMF_CUDA_TRY(cudaGetLastError());
    NIMF_CUDA_TRY(cudaMemcpyAsync(h, hist, nb * sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    NIMF_CUDA_TRY(cudaStreamSynchronize(st));
    if (pass == 0) {
      for (int i = 0; i < nb; ++i) total += h[i];
      *n_valid = total;
      if (total == 0) {
        *median = 0.0f;
        return NIMF_OK;
      }
      want = total / 2;
    }
    int64_t acc = 0;
    int sel = nb - 1;
    for (int i = 0; i < nb; ++i) {
      if (acc + h[i] > want) {
        sel = i;
        break;
      }
      acc += h[i];
    }
    want -= acc;
    prefix = (prefix << widths[pass]) | (unsigned)sel;
    prefix_shift = shifts[pass];
  }
  *median = __builtin_bit_cast(float, prefix);
  return NIMF_OK;
}

}  // namespace
}  // namespace nimf

using namespace nimf;

extern "C" int nimf_cf_autoselect_dev_noalloc(const float* x_dev, int64_t n,
                                              const float* grad_dev, int64_t n_grad,
                                              double rel_error_tol, int exp_margin,
                                              int* exponent_bits, int* mantissa_bits,
                                              void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (n < 0 || n_grad < 0) return set_error(NIMF_ERR_SHAPE, "negative length");
  if (n > kNoAllocMaxElems || n_grad > kNoAllocMaxElems)
    return set_error(NIMF_ERR_SHAPE,
                     "nimf_cf_autoselect_dev_noalloc: at most %lld elements per buffer "
                     "(its fixed scratch keeps 32-bit counts); got %lld and %lld",
                     (long long)kNoAllocMaxElems, (long long)n, (long long)n_grad);
  if (!exponent_bits || !mantissa_bits) return set_error(NIMF_ERR_ARG, "NULL output");
  if ((n > 0 && !x_dev) || (n_grad > 0 && !grad_dev)) return set_error(NIMF_ERR_ARG, "NULL input");
  if (c->device < 0 || c->device >= 64) return set_error(NIMF_ERR_STATE, "device index");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "nimf_cf_autoselect_dev_noalloc: the stream is being captured; this call "
                       "reads its reductions back to the host and synchronises the stream");
  }
  // One-time set-up on this device (the device is current): the array's
  // device address.
  if (!g_noalloc_addr[c->device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(NIMF_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_addr[c->device] = (unsigned*)p;
  }
  unsigned* scratch = g_noalloc_addr[c->device];

  float mn = 0.f, mx = 0.f;
  bool found = false;
  if (n > 0) {
    noalloc_minmax_init<<<1, 1, 0, st>>>(scratch);
    absrange_kernel<<<grid_for(n, 256), 256, 0, st>>>(x_dev, n, scratch);
    NIMF_CUDA_TRY(cudaGetLastError());
    unsigned r[2];
    NIMF_CUDA_TRY(cudaMemcpyAsync(r, scratch, sizeof(r), cudaMemcpyDeviceToHost, st));
    NIMF_CUDA_TRY(cudaStreamSynchronize(st));
    found = r[1] != 0u;
    mn = __builtin_bit_cast(float, r[0]);
    mx = __builtin_bit_cast(float, r[1]);
  }
  // computeRequiredExponentBits / computeRequiredMantissaBits
  // (customfloat.nim:149-198), evaluated in double as the reference does.
  int eb = 1, mb = 2;
  if (found) {
    const int64_t max_e = (int64_t)std::floor(std::log2((double)mx));
    const int64_t min_e = (int64_t)std::floor(std::log2((double)mn));
    const int64_t span = (max_e - min_e) + 2 * (int64_t)exp_margin + 2;
    eb = (int)std::max<int64_t>(1, (int64_t)std::ceil(std::log2((double)std::max<int64_t>(span, 2))));
    const int64_t base = (int64_t)std::ceil(std::log2(1.0 / std::max(rel_error_tol, 1e-12)));
    int64_t extra = 0;
    if (n_grad > 0) {
      float wmed = 0.f, gmed = 0.f;
      int64_t nv = 0, ngv = 0;
      NIMF_TRY(noalloc_abs_median(x_dev, n, scratch + 2, &wmed, &nv, st));
      NIMF_TRY(noalloc_abs_median(grad_dev, n_grad, scratch + 2, &gmed, &ngv, st));
      if (ngv > 0) {
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
