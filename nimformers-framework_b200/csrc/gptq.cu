// gptq.cu -- GPTQ-native int4 checkpoints (qweight / qzeros / fp16 scales /
// g_idx, the layout export_to_nimq.py:219-254 dequantize_gptq_linear reads)
// registered as device-resident int4 group weights without an fp32
// round-trip through the exporter.
//
//   w[n][k] = (nib(k, n) - ((z(g_idx[k], n) + 1) & 15)) * float(scale[g_idx[k]][n])
//
// with nib the k % 8-th nibble of qweight[k / 8][n] and z the n % 8-th nibble
// of qzeros[g][n / 8].  This is the int4 group weight's (float(nib) - zp) * sc
// with zp = float((z + 1) & 15) and sc = float(scale): the subtraction is
// exact, so dequantisation is bit-identical to the reference.  Groups that are
// contiguous runs of k (g_idx[k] = k / gs) map onto the int4 layout directly.
// Act-order checkpoints (g_idx a permutation of such runs) are stored with
// their k reordered so that every group is contiguous; the permutation stays
// on the device and x is gathered through it before each matmul.
#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

#include "nimf_internal.h"

namespace nimf {

namespace {

__global__ void gather_cols_kernel(const float* __restrict__ x, int64_t m, int64_t k,
                                   const int32_t* __restrict__ perm, float* __restrict__ out) {
  const int64_t n = m * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k, j = i - r * k;
    out[i] = x[r * k + perm[j]];
  }
}

struct PermBuf {
  int device = -1;
  void* p = nullptr;
  size_t bytes = 0;
};
PermBuf g_pbuf;

}  // namespace

// x[m][k] gathered through perm into a per-device scratch buffer (grown
// outside stream capture; calls using it are ordered on one stream).
int gather_cols(const float* x, int64_t m, int64_t k, const int32_t* perm, const float** out,
                cudaStream_t st) {
  Context* c = ctx();
  const size_t bytes = (size_t)(m * k) * sizeof(float);
  if (g_pbuf.device != c->device || g_pbuf.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "act-order GPTQ weight: its x scratch must grow, which cannot happen during "
                       "stream capture; run the same call once before capturing");
    NIMF_CUDA_TRY(cudaDeviceSynchronize());
    if (g_pbuf.device == c->device) device_free(g_pbuf.p);
    g_pbuf = PermBuf();
    NIMF_TRY(device_alloc(&g_pbuf.p, bytes));
    g_pbuf.device = c->device;
    g_pbuf.bytes = bytes;
  }
  if (m * k > 0) {
    const unsigned blocks = (unsigned)std::max<int64_t>(
        1, std::min<int64_t>((int64_t)c->num_sms * 8, (m * k + 255) / 256));
    gather_cols_kernel<<<blocks, 256, 0, st>>>(x, m, k, perm, (float*)g_pbuf.p);
    NIMF_CUDA_TRY(cudaGetLastError());
  }
  *out = (const float*)g_pbuf.p;
  return NIMF_OK;
}

void release_perm_buffer() {
  device_free(g_pbuf.p);
  g_pbuf = PermBuf();
}

namespace {

float half_to_float(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
  uint32_t bits;
  if (e == 31) {
    bits = s | 0x7F800000u | (m << 13);
  } else if (e == 0) {
    if (m == 0) {
      bits = s;
    } else {  // subnormal: normalise
      int ee = -1;
      uint32_t mm = m;
      do {
        ++ee;
        mm <<= 1;
      } while ((mm & 1024u) == 0);
      bits = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023u) << 13);
    }
  } else {
    bits = s | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_weight_register_gptq(const int32_t* qweight, const int32_t* qzeros,
                              const uint16_t* scales_f16, const int32_t* g_idx,
                              int64_t in_features, int64_t out_features, int64_t n_groups,
                              int64_t row_begin, int64_t row_end, nimf_weight_t* out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  const int64_t K = in_features, N = out_features;
  if (K <= 0 || N <= 0 || K % 8 || N % 8 || n_groups <= 0)
    return set_error(NIMF_ERR_SHAPE, "GPTQ: in_features %lld and out_features %lld must be positive "
                     "multiples of 8, n_groups %lld positive", (long long)K, (long long)N,
                     (long long)n_groups);
  if (row_begin < 0 || row_end < row_begin || row_end > N)
    return set_error(NIMF_ERR_SHAPE, "row range [%lld, %lld) outside [0, %lld)",
                     (long long)row_begin, (long long)row_end, (long long)N);
  if (!qweight || !qzeros || !scales_f16 || !g_idx) return set_error(NIMF_ERR_ARG, "NULL GPTQ array");
  // groups: every k in [0, n_groups), equal group sizes except the last run
  std::vector<int64_t> count((size_t)n_groups, 0);
  for (int64_t k = 0; k < K; ++k) {
    if (g_idx[k] < 0 || g_idx[k] >= n_groups)
      return set_error(NIMF_ERR_SHAPE, "GPTQ: g_idx[%lld] = %d outside [0, %lld)", (long long)k,
                       g_idx[k], (long long)n_groups);
    ++count[(size_t)g_idx[k]];
  }
  std::vector<int32_t> perm((size_t)K);
  std::iota(perm.begin(), perm.end(), 0);
  std::stable_sort(perm.begin(), perm.end(), [&](int32_t a, int32_t b) { return g_idx[a] < g_idx[b]; });
  bool identity = true;
  for (int64_t j = 0; j < K; ++j) identity = identity && perm[(size_t)j] == j;
  const int64_t gs = count[0];
  for (int64_t g = 0; g < n_groups; ++g) {
    const bool last = g == n_groups - 1;
    if (count[(size_t)g] != gs && !(last && count[(size_t)g] > 0 && count[(size_t)g] < gs))
      return set_error(NIMF_ERR_UNSUPPORTED, "GPTQ: group %lld has %lld members, group 0 has %lld",
                       (long long)g, (long long)count[(size_t)g], (long long)gs);
  }
  if ((K + gs - 1) / gs != n_groups)
    return set_error(NIMF_ERR_SHAPE, "GPTQ: %lld groups of %lld cannot cover K = %lld",
                     (long long)n_groups, (long long)gs, (long long)K);
  // host arrays in the int4 group layout, rows [row_begin, row_end), k in
  // permuted order (stored column j holds original k = perm[j])
  const int64_t rows = row_end - row_begin, bpr = (K + 1) / 2;
  std::vector<uint8_t> wq((size_t)(rows * bpr), 0);
  std::vector<float> sc((size_t)(rows * n_groups)), zp((size_t)(rows * n_groups));
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t n = row_begin + r;
    for (int64_t j = 0; j < K; ++j) {
      const int64_t k = perm[(size_t)j];
      const uint32_t nib = ((uint32_t)qweight[(k / 8) * N + n] >> (4 * (k % 8))) & 15u;
      wq[(size_t)(r * bpr + j / 2)] |= (uint8_t)(nib << (4 * (j & 1)));
    }
    for (int64_t g = 0; g < n_groups; ++g) {
      const uint32_t z = (((uint32_t)qzeros[g * (N / 8) + n / 8] >> (4 * (n % 8))) & 15u);
      zp[(size_t)(r * n_groups + g)] = (float)((z + 1) & 15u);
      sc[(size_t)(r * n_groups + g)] = half_to_float(scales_f16[g * N + n]);
    }
  }
  nimf_weight_t h;
  NIMF_TRY(nimf_weight_register_q4g(wq.data(), sc.data(), zp.data(), rows, K, gs, n_groups, 0,
                                    rows, &h));
  {
    Weight* w = lookup(h);
    w->row_begin = row_begin;
    w->n_full = N;
  }
  if (!identity) {
    Weight* w = lookup(h);
    void* d = nullptr;
    int st = device_alloc(&d, (size_t)K * sizeof(int32_t));
    if (st == NIMF_OK) {
      cudaError_t e = cudaMemcpy(d, perm.data(), (size_t)K * sizeof(int32_t), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) st = set_error(NIMF_ERR_CUDA, "GPTQ permutation upload: %s", cudaGetErrorString(e));
    }
    if (st != NIMF_OK) {
      device_free(d);
      nimf_weight_free(h);
      return st;
    }
    w->kperm = d;
    w->kperm_host = perm;
  }
  *out = h;
  return NIMF_OK;
}

}  // extern "C"
