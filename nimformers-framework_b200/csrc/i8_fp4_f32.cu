// i8_fp4_f32.cu -- the int8 (quant.nim:51-67) and FP4 E2M1 block-16 (no
// reference counterpart) warp-per-row kernels, and the fp32 weight transpose
// (beMatmul's b, gpubackend.nim:584-604).  The fp32 matmul itself is f32.cu.
//
// int8 and FP4 GEMVs here are warp-per-row kernels that dequantise each weight
// with the reference's rounding and accumulate in fp32.
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

unsigned grid_rows(int64_t rows) {
  Context* c = ctx();
  const int64_t cap = (int64_t)(c ? c->num_sms : 148) * 16;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, (rows * 32 + 255) / 256));
}

unsigned grid_elems(int64_t n) {
  Context* c = ctx();
  const int64_t cap = (int64_t)(c ? c->num_sms : 148) * 8;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, (n + 255) / 256));
}

// ------------------------------------------------------------------ int8
__global__ void i8_gemv_kernel(const int8_t* __restrict__ q, const float* __restrict__ sc,
                               int64_t nsc, int64_t rows, int64_t k, const float* __restrict__ x,
                               int m, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  griddep_wait();
  for (int64_t row = warp; row < rows; row += nwarps) {
    const float s = sc[nsc == 1 ? 0 : row];
    const int8_t* rp = q + row * k;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int64_t c = lane; c < k; c += 32) {
      const float w = __fmul_rn((float)rp[c], s);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < m) acc[i] = fmaf(w, x[i * k + c], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < m) {
        const float v = warp_sum(acc[i]);
        if (lane == 0) y[i * rows + row] = v;
      }
    }
  }
}

__global__ void i8_dequant_kernel(const int8_t* __restrict__ q, const float* __restrict__ sc,
                                  int64_t nsc, int64_t rows, int64_t k, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * k;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn((float)q[i], sc[nsc == 1 ? 0 : i / k]);
}

// ------------------------------------------------------------------ FP4
__device__ __forceinline__ float e2m1_value(uint32_t nib) {
  // {0, .5, 1, 1.5, 2, 3, 4, 6} with sign bit 3
  const uint32_t e = (nib >> 1) & 3u, mbit = nib & 1u;
  float v;
  if (e == 0) v = mbit ? 0.5f : 0.0f;
  else v = __uint_as_float(((e + 126u) << 23) | (mbit << 22));
  return (nib & 8u) ? -v : v;
}

__device__ __forceinline__ float e4m3_ocp_value(uint32_t b) {
  const uint32_t s = b >> 7, e = (b >> 3) & 15u, mm = b & 7u;
  float v;
  if (e == 15 && mm == 7) v = __uint_as_float(0x7FC00000u);
  else if (e == 0) v = (float)mm * 0.001953125f;  // m * 2^-9, exact
  else v = __uint_as_float(((e + 120u) << 23) | (mm << 20));
  return s ? -v : v;
}

__global__ void fp4_gemv_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ bs,
                                float ts, int64_t rows, int64_t k, const float* __restrict__ x,
                                int m, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t bpr = (k + 1) / 2, nb = (k + 15) / 16;
  griddep_wait();
  for (int64_t row = warp; row < rows; row += nwarps) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int64_t c = lane; c < k; c += 32) {
      const uint8_t b = packed[row * bpr + (c >> 1)];
      const uint32_t nib = (c & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
      const float t = __fmul_rn(e4m3_ocp_value(bs[row * nb + (c >> 4)]), ts);
      const float w = __fmul_rn(e2m1_value(nib), t);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < m) acc[i] = fmaf(w, x[i * k + c], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < m) {
        const float v = warp_sum(acc[i]);
        if (lane == 0) y[i * rows + row] = v;
      }
    }
  }
}

__global__ void fp4_dequant_kernel(const uint8_t* __restrict__ packed,
                                   const uint8_t* __restrict__ bs, float ts, int64_t rows,
                                   int64_t k, float* __restrict__ out) {
  const int64_t bpr = (k + 1) / 2, nb = (k + 15) / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * k;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / k, c = i % k;
    const uint8_t b = packed[row * bpr + (c >> 1)];
    const uint32_t nib = (c & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
    const float t = __fmul_rn(e4m3_ocp_value(bs[row * nb + (c >> 4)]), ts);
    out[i] = __fmul_rn(e2m1_value(nib), t);
  }
}

// ------------------------------------------------------------------ fp32
__global__ void transpose_kernel(const float* __restrict__ in, int64_t rows, int64_t cols,
                                 float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}


}  // namespace

int i8_gemv(const I8Weight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    i8_gemv_kernel<<<grid_rows(w.rows), 256, 0, st>>>((const int8_t*)w.q, (const float*)w.scales,
                                                      w.n_scales, w.rows, w.k, x + m0 * w.k, mc,
                                                      y + m0 * w.rows);
  }
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int i8_dequant(const I8Weight& w, float* out, cudaStream_t st) {
  i8_dequant_kernel<<<grid_elems(w.rows * w.k), 256, 0, st>>>(
      (const int8_t*)w.q, (const float*)w.scales, w.n_scales, w.rows, w.k, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int fp4_gemv(const FP4Weight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    fp4_gemv_kernel<<<grid_rows(w.rows), 256, 0, st>>>(
        (const uint8_t*)w.packed, (const uint8_t*)w.bscale, w.tensor_scale, w.rows, w.k,
        x + m0 * w.k, mc, y + m0 * w.rows);
  }
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int fp4_dequant(const FP4Weight& w, float* out, cudaStream_t st) {
  fp4_dequant_kernel<<<grid_elems(w.rows * w.k), 256, 0, st>>>(
      (const uint8_t*)w.packed, (const uint8_t*)w.bscale, w.tensor_scale, w.rows, w.k, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int f32_transpose(const float* b_kn, int64_t k, int64_t n, float* w_nk, cudaStream_t st) {
  if (k == 0 || n == 0) return NIMF_OK;
  dim3 grid((unsigned)((n + 31) / 32), (unsigned)((k + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(b_kn, k, n, w_nk);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

}  // namespace nimf
