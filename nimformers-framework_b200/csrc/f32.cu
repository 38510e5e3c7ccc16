// f32.cu -- the raw fp32 matmul of beMatmul / beMatmul2 (backend.nim:87-91,
// 112-119 -> gpubackend.nim:584-626): C[M][N] = A[M][K] . B[K][N], row-major,
// fp32 products and fp32 sums, as cpuMatmul (gpubackend.nim:560-582) computes
// them up to the order of the sums.  The reference's CUDA path hands this to
// cuBLAS SGEMM (cuda_runtime.nim:122-152); here two hand-written kernels
// cover it:
//
//   * f32_gemv_kernel (M <= 8): one pass over B, which is the only large
//     operand, so it is HBM-bound.  A block owns 128 columns (32 lanes x one
//     float4) and a K range; its 8 warps take the range's k in turn and sum
//     their partials in warp order in shared memory.  When the column tiles
//     alone would leave SMs idle, K is split over blocks too and a second
//     kernel adds the splits' partials in split order (deterministic).
//   * f32_gemm_kernel (M > 8): 128 x 128 output tile per block of 256
//     threads, 8 x 8 outputs per thread, k-slabs of 8 staged in shared memory
//     (A transposed so a thread's 8 rows are two float4 loads), the next slab
//     loaded into registers while the current one is multiplied.  Each output
//     is one fp32 FMA chain over k ascending.
//
// Both read A and B with bounds checks (zeros outside), so any M, N, K work;
// 16-byte vector loads are used when rows are 16-byte aligned.
#include <algorithm>
#include <cstdint>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr int kGemvCols = 128;   // columns per GEMV block (32 lanes x 4)
constexpr int kGemvWarps = 8;
constexpr int kMaxRowsGemv = 8;

// Partial sums of rows [0, m) of A over k in [k0, k1) for 128 columns.
// part == nullptr: write C directly (single K split).
template <bool VEC>
__global__ void __launch_bounds__(kGemvWarps * 32)
f32_gemv_kernel(const float* __restrict__ a, int m, int64_t k, const float* __restrict__ b,
                int64_t n, float* __restrict__ c, float* __restrict__ part, int64_t kchunk) {
  __shared__ float4 red[kGemvWarps][kMaxRowsGemv][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col = (int64_t)blockIdx.x * kGemvCols + lane * 4;
  const int64_t k0 = (int64_t)blockIdx.y * kchunk;
  const int64_t k1 = min(k, k0 + kchunk);
  float4 acc[kMaxRowsGemv];
#pragma unroll
  for (int r = 0; r < kMaxRowsGemv; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t kk = k0 + warp; kk < k1; kk += kGemvWarps) {
    float4 bv;
    const float* brow = b + kk * n;
    if (VEC && col + 3 < n) {
      bv = __ldg(reinterpret_cast<const float4*>(brow + col));
    } else {
      bv.x = col < n ? __ldg(brow + col) : 0.f;
      bv.y = col + 1 < n ? __ldg(brow + col + 1) : 0.f;
      bv.z = col + 2 < n ? __ldg(brow + col + 2) : 0.f;
      bv.w = col + 3 < n ? __ldg(brow + col + 3) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < kMaxRowsGemv; ++r) {
      if (r < m) {
        const float av = __ldg(a + (int64_t)r * k + kk);
        acc[r].x = fmaf(av, bv.x, acc[r].x);
        acc[r].y = fmaf(av, bv.y, acc[r].y);
        acc[r].z = fmaf(av, bv.z, acc[r].z);
        acc[r].w = fmaf(av, bv.w, acc[r].w);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kMaxRowsGemv; ++r)
    if (r < m) red[warp][r][lane] = acc[r];
  __syncthreads();
  // thread t sums warp partials of (row t / 32, lane t % 32) in warp order
  for (int e = threadIdx.x; e < m * 32; e += blockDim.x) {
    const int r = e >> 5, l = e & 31;
    float4 s = red[0][r][l];
    for (int w = 1; w < kGemvWarps; ++w) {
      const float4 v = red[w][r][l];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    const int64_t cc = (int64_t)blockIdx.x * kGemvCols + l * 4;
    float* dst = part ? part + ((int64_t)blockIdx.y * m + r) * n : c + (int64_t)r * n;
    const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (cc + j < n) dst[cc + j] = sv[j];
  }
}

// c[i] = sum over splits in order of part[s][i]
__global__ void f32_splits_sum_kernel(const float* __restrict__ part, int splits, int64_t count,
                                      float* __restrict__ c) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = part[i];
    for (int j = 1; j < splits; ++j) s += part[(int64_t)j * count + i];
    c[i] = s;
  }
}

constexpr int kBM = 128, kBN = 128, kBK = 8;

template <bool VEC>
__global__ void __launch_bounds__(256)
f32_gemm_kernel(const float* __restrict__ a, int64_t m, int64_t k, const float* __restrict__ b,
                int64_t n, float* __restrict__ c) {
  __shared__ __align__(16) float As[2][kBK][kBM + 4];
  __shared__ __align__(16) float Bs[2][kBK][kBN];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * kBM, n0 = (int64_t)blockIdx.x * kBN;
  // global -> register loaders: A row m0 + tid/2, k columns (tid&1)*4 .. +3;
  // B row k0 + tid/32, columns (tid&31)*4 .. +3
  const int ar = tid >> 1, ak = (tid & 1) * 4;
  const int br = tid >> 5, bc = (tid & 31) * 4;
  float ra[4], rb[4];
  auto load = [&](int64_t k0) {
    const int64_t gm = m0 + ar, gk = k0 + ak;
    if (VEC && gm < m && gk + 3 < k) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(a + gm * k + gk));
      ra[0] = v.x, ra[1] = v.y, ra[2] = v.z, ra[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) ra[j] = (gm < m && gk + j < k) ? __ldg(a + gm * k + gk + j) : 0.f;
    }
    const int64_t gk2 = k0 + br, gn = n0 + bc;
    if (VEC && gk2 < k && gn + 3 < n) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(b + gk2 * n + gn));
      rb[0] = v.x, rb[1] = v.y, rb[2] = v.z, rb[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) rb[j] = (gk2 < k && gn + j < n) ? __ldg(b + gk2 * n + gn + j) : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) As[buf][ak + j][ar] = ra[j];
    *reinterpret_cast<float4*>(&Bs[buf][br][bc]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
  };
  // thread (ty, tx) owns rows {4ty .. 4ty+3, 64+4ty .. 64+4ty+3} and the same
  // pattern of columns, so its shared-memory reads are float4s without
  // conflicts within a quarter warp
  const int ty = tid >> 4, tx = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int64_t nk = (k + kBK - 1) / kBK;
  load(0);
  store(0);
  __syncthreads();
  for (int64_t t = 0; t < nk; ++t) {
    const int buf = (int)(t & 1);
    if (t + 1 < nk) load((t + 1) * kBK);
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + 4 * tx]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (t + 1 < nk) store(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + (i - 4));
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gn = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + (j - 4));
      if (gn < n) c[gm * n + gn] = acc[i][j];
    }
  }
}

// split-K partials of the GEMV path (grown outside stream capture)
struct F32Scratch {
  int device = -1;
  float* part = nullptr;
  size_t bytes = 0;
};
F32Scratch g_f32s[16];

int f32_scratch(size_t bytes, cudaStream_t st, float** out) {
  Context* cx = ctx();
  F32Scratch& s = g_f32s[cx->device & 15];
  if (s.device == cx->device && s.bytes >= bytes) {
    *out = s.part;
    return NIMF_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone)
    return set_error(NIMF_ERR_STATE,
                     "fp32 GEMV: its split-K buffer must grow (%zu bytes), which cannot happen "
                     "during stream capture; run the call once before capturing",
                     bytes);
  NIMF_CUDA_TRY(cudaStreamSynchronize(st));
  if (s.device == cx->device) device_free(s.part);
  s = F32Scratch();
  void* p = nullptr;
  NIMF_TRY(device_alloc(&p, bytes));
  s.device = cx->device;
  s.part = (float*)p;
  s.bytes = bytes;
  *out = s.part;
  return NIMF_OK;
}

}  // namespace

void release_f32_scratch() {
  Context* cx = ctx();
  for (F32Scratch& s : g_f32s) {
    if (s.part && cx && s.device == cx->device) device_free(s.part);
    s = F32Scratch();
  }
}

// C[m][n] = A[m][k] . B[k][n] (row-major), the operation cuda_runtime.nim:147-150
// asks cuBLAS for.
int f32_gemm(const float* a, int64_t m, int64_t k, const float* b_kn, int64_t n, float* c,
             cudaStream_t st) {
  Context* cx = ctx();
  if (m == 0 || n == 0) return NIMF_OK;
  if (k == 0) {
    NIMF_CUDA_TRY(cudaMemsetAsync(c, 0, (size_t)(m * n) * 4, st));
    return NIMF_OK;
  }
  const int sms = cx ? cx->num_sms : 148;
  const bool vec_b = ((reinterpret_cast<uintptr_t>(b_kn) & 15) == 0) && n % 4 == 0;
  if (m <= kMaxRowsGemv) {
    const int64_t ctiles = (n + kGemvCols - 1) / kGemvCols;
    // split K so that about two blocks run per SM, each with >= 64 k per warp
    int64_t splits = std::max<int64_t>(1, (2 * sms + ctiles - 1) / ctiles);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, k / (kGemvWarps * 64)));
    splits = std::min<int64_t>(splits, 64);
    const int64_t kchunk = (k + splits - 1) / splits;
    splits = (k + kchunk - 1) / kchunk;
    if (ctiles > 65535 * 1024LL) return set_error(NIMF_ERR_UNSUPPORTED, "fp32 GEMV: N too large");
    float* part = nullptr;
    if (splits > 1) NIMF_TRY(f32_scratch((size_t)splits * m * n * 4, st, &part));
    dim3 grid((unsigned)ctiles, (unsigned)splits);
    if (vec_b)
      f32_gemv_kernel<true><<<grid, kGemvWarps * 32, 0, st>>>(a, (int)m, k, b_kn, n, c, part, kchunk);
    else
      f32_gemv_kernel<false><<<grid, kGemvWarps * 32, 0, st>>>(a, (int)m, k, b_kn, n, c, part, kchunk);
    NIMF_CUDA_TRY(cudaGetLastError());
    if (splits > 1) {
      const int64_t cnt = m * n;
      const unsigned blocks = (unsigned)std::min<int64_t>((cnt + 255) / 256, (int64_t)sms * 8);
      f32_splits_sum_kernel<<<blocks, 256, 0, st>>>(part, (int)splits, cnt, c);
      NIMF_CUDA_TRY(cudaGetLastError());
    }
    return NIMF_OK;
  }
  const int64_t gx = (n + kBN - 1) / kBN, gy = (m + kBM - 1) / kBM;
  if (gy > 65535) return set_error(NIMF_ERR_UNSUPPORTED, "fp32 GEMM: M too large");
  const bool vec = vec_b && ((reinterpret_cast<uintptr_t>(a) & 15) == 0) && k % 4 == 0;
  dim3 grid((unsigned)gx, (unsigned)gy);
  if (vec) f32_gemm_kernel<true><<<grid, 256, 0, st>>>(a, m, k, b_kn, n, c);
  else f32_gemm_kernel<false><<<grid, 256, 0, st>>>(a, m, k, b_kn, n, c);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

}  // namespace nimf
