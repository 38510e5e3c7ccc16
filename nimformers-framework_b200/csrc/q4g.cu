// q4g.cu -- int4 asymmetric per-group weights (QuantTensor kind 3 with
// groupSize > 0, quant.nim:131-167) on sm_100a: device repack, bit-exact
// dequantisation and the decode GEMV y[M][N] = x[M][K] . W^T.
//
// GEMV design (memory-bound: 0.5 B of weight per multiply-add):
//   * Weights are repacked once at registration into mma.sync m16n8k16
//     A-fragment order: for row tile rt (16 output rows) and k-quad kq (64 k),
//     lane L of a warp owns one uint4 whose word j holds the 8 nibbles that
//     lane needs for k-tile 4*kq+j.  A warp therefore streams 512 contiguous
//     bytes per 128-bit load, and unpacking is 1 SHF + 4 LOP3 + 4 bf16 SUB
//     per 8 nibbles (0x4300|n == bf16(128+n)).
//   * The nibbles (exact small integers in bf16) multiply x on the tensor
//     cores.  x is split into bf16 hi + lo parts (~2^-17 relative), so the
//     products carry fp32-class accuracy; for M <= 4 the hi and lo parts sit
//     in columns [0,4) and [4,8) of the same n=8 MMA, for M <= 8 they take
//     two MMAs.
//   * The asymmetric zero point is applied once per group by the algebra
//     sum_k (n_k - zp) s x_k = s (sum_k n_k x_k - zp sum_k x_k); the per-group
//     sums of x are computed in the CTA prologue.  Only the GEMV accumulation
//     is refactored; the dequantised weights themselves (q4g_dequant below)
//     are bit-identical to the reference.
//   * Split-K over a thread-block cluster: the CTAs of one row band each take
//     a range of groups, stage their slice of x (as ready-to-use B fragments)
//     and their scales/zeros in shared memory, and reduce the partial y
//     through distributed shared memory in rank order (deterministic).
//   * Programmatic dependent launch: weights are prefetched before
//     griddepcontrol.wait, so back-to-back GEMVs overlap prologue and tail.
#include <cooperative_groups.h>

#include <algorithm>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace cg = cooperative_groups;

namespace nimf {

namespace {

constexpr int kWarps = 4;       // row tiles per CTA (one per warp)
constexpr int kPipe = 8;        // 128-bit weight loads in flight per lane
constexpr int kMaxSplits = 8;   // portable cluster size

// Slot s (0..7) of a fragment word holds row  g + 8*(s&1)  and
// k-offset  2t + 8*((s>>1)&1) + ((s>>2)&1)  of the 16x16 tile.
__device__ __forceinline__ int slot_row(int g, int s) { return g + ((s & 1) ? 8 : 0); }
__device__ __forceinline__ int slot_k(int t, int s) {
  return 2 * t + ((s & 2) ? 8 : 0) + ((s & 4) ? 1 : 0);
}

__global__ void q4g_repack_frag(const uint8_t* __restrict__ wq, int64_t bpr, int64_t rows,
                                int64_t k, int64_t kq_total, int64_t total,
                                uint4* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const int64_t q = i >> 5;
  const int64_t kq = q % kq_total;
  const int64_t rt = q / kq_total;
  const int g = lane >> 2, t = lane & 3;
  uint32_t words[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t kt0 = (kq * 4 + j) * 16;
    uint32_t w = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int64_t row = rt * 16 + slot_row(g, s);
      const int64_t col = kt0 + slot_k(t, s);
      uint32_t nib = 0;
      if (row < rows && col < k) {
        const uint8_t b = wq[row * bpr + (col >> 1)];
        nib = (col & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
      }
      w |= nib << (4 * s);
    }
    words[j] = w;
  }
  out[i] = make_uint4(words[0], words[1], words[2], words[3]);
}

__global__ void q4g_repack_sz(const float* __restrict__ sc, const float* __restrict__ zp,
                              int64_t ngr, int64_t rows, int64_t groups, int64_t total,
                              float4* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int gi = (int)(i & 7);
  const int64_t q = i >> 3;
  const int64_t grp = q % groups;
  const int64_t rt = q / groups;
  const int64_t r0 = rt * 16 + gi, r1 = r0 + 8;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r0 < rows) { v.x = sc[r0 * ngr + grp]; v.y = zp[r0 * ngr + grp]; }
  if (r1 < rows) { v.z = sc[r1 * ngr + grp]; v.w = zp[r1 * ngr + grp]; }
  out[i] = v;
}

// out[r][c] = (float(nib) - zp) * sc with the reference's two roundings
// (quant.nim:162: lut[k] = (float32(k) - zp) * sc), read back from the
// fragment layout.
__global__ void q4g_dequant_frag(const uint4* __restrict__ frag, const float4* __restrict__ sz,
                                 int64_t rows, int64_t k, int64_t kq_total, int64_t groups,
                                 int64_t gs, float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * k) return;
  const int64_t row = i / k, col = i % k;
  const int64_t rt = row >> 4;
  const int r = (int)(row & 15);
  const int64_t kt = col >> 4;
  const int kk = (int)(col & 15);
  const int g = r & 7, rhi = r >> 3;
  const int t = (kk & 7) >> 1, khi = kk >> 3, kodd = kk & 1;
  const int lane = g * 4 + t;
  const int s = rhi + 2 * khi + 4 * kodd;
  const uint4 v = frag[((rt * kq_total) + (kt >> 2)) * 32 + lane];
  const uint32_t word = (&v.x)[kt & 3];
  const uint32_t nib = (word >> (4 * s)) & 15u;
  const float4 p = sz[((rt * groups) + col / gs) * 8 + g];
  const float scale = rhi ? p.z : p.x;
  const float zero = rhi ? p.w : p.y;
  out[i] = __fmul_rn(__fsub_rn((float)nib, zero), scale);
}

__global__ void q4g_dequant_raw(const uint8_t* __restrict__ wq, const float* __restrict__ sc,
                                const float* __restrict__ zp, int64_t rows, int64_t k,
                                int64_t gs, int64_t ngr, float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * k) return;
  const int64_t row = i / k, col = i % k;
  const int64_t bpr = (k + 1) / 2;
  const uint8_t b = wq[row * bpr + (col >> 1)];
  const uint32_t nib = (col & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
  const int64_t g = gs > 0 ? col / gs : 0;
  out[i] = __fmul_rn(__fsub_rn((float)nib, zp[row * ngr + g]), sc[row * ngr + g]);
}

struct GemvArgs {
  const uint4* frag;
  const float4* sz;
  const float* x;
  float* y;
  int64_t ldx, ldy;
  int m, k, rows, n_rt;
  int kq_total, kqg, gs, groups, gps;
};

// MODE 1: M <= 4, one MMA per k-tile (hi in columns 0..3, lo in 4..7).
// MODE 2: M <= 8, two MMAs per k-tile (hi and lo each in columns 0..7).
template <int MODE>
__global__ void __launch_bounds__(kWarps * 32)
q4g_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int g0 = split * a.gps;
  const int ng = min(a.gps, a.groups - g0);
  const int kq0 = g0 * a.kqg, nq = ng * a.kqg;
  const int kt0 = kq0 * 4, nkt = nq * 4;
  const int rt = blockIdx.x * kWarps + warp;
  const bool active = rt < a.n_rt;

  constexpr int kFragBytes = MODE == 1 ? 8 : 16;
  unsigned char* p = smem;
  unsigned char* xs = p;                    p += (size_t)a.gps * a.kqg * 4 * 32 * kFragBytes;
  float* sxs = reinterpret_cast<float*>(p); p += (size_t)a.gps * 8 * sizeof(float);
  float4* szs = reinterpret_cast<float4*>(p); p += (size_t)kWarps * a.gps * 8 * sizeof(float4);
  float* part = reinterpret_cast<float*>(p);

  // 1. Start streaming this warp's weights and (async) its scales/zeros.
  uint4 buf[kPipe];
  const uint4* wp = a.frag + ((size_t)(active ? rt : 0) * a.kq_total + kq0) * 32 + lane;
  if (active) {
#pragma unroll
    for (int i = 0; i < kPipe; ++i)
      if (i < nq) buf[i] = ldg_stream(wp + (size_t)i * 32);
    const float4* szg = a.sz + ((size_t)rt * a.groups + g0) * 8;
    for (int i = lane; i < ng * 8; i += 32) cp_async16(&szs[(warp * a.gps) * 8 + i], szg + i);
  }

  // 2. x may be written by the previous kernel in the stream.
  griddep_wait();

  // 3. Stage x[:, this split's k range] as B fragments, and per-group sums.
  for (int e = threadIdx.x; e < nkt * 32; e += blockDim.x) {
    const int ktl = e >> 5, L = e & 31;
    const int n = L >> 2, tt = L & 3;
    const int kb = (kt0 + ktl) * 16 + 2 * tt;
    // MODE 1: columns 0..3 carry the hi part of rows m = n, columns 4..7 the
    // lo part of rows m = n - 4.  MODE 2: column n is row m = n (hi and lo).
    const int mrow = (MODE == 1 && n >= 4) ? n - 4 : n;
    const bool ok = mrow < a.m;
    const float* xr = a.x + (size_t)(ok ? mrow : 0) * a.ldx;
    float v[4];
    v[0] = (ok && kb < a.k) ? __ldg(xr + kb) : 0.0f;
    v[1] = (ok && kb + 1 < a.k) ? __ldg(xr + kb + 1) : 0.0f;
    v[2] = (ok && kb + 8 < a.k) ? __ldg(xr + kb + 8) : 0.0f;
    v[3] = (ok && kb + 9 < a.k) ? __ldg(xr + kb + 9) : 0.0f;
    uint32_t h0, l0, h1, l1;
    split_bf16x2(v[0], v[1], h0, l0);
    split_bf16x2(v[2], v[3], h1, l1);
    if (MODE == 1)
      reinterpret_cast<uint2*>(xs)[e] = n < 4 ? make_uint2(h0, h1) : make_uint2(l0, l1);
    else
      reinterpret_cast<uint4*>(xs)[e] = make_uint4(h0, h1, l0, l1);
  }
  for (int pr = warp; pr < ng * 8; pr += kWarps) {
    const int gl = pr >> 3, n = pr & 7;
    float s = 0.0f;
    if (n < a.m) {
      const float* xr = a.x + (size_t)n * a.ldx;
      const int kb = (g0 + gl) * a.gs;
      for (int kk = lane; kk < a.gs; kk += 32)
        if (kb + kk < a.k) s += __ldg(xr + kb + kk);
      s = warp_sum(s);
    }
    if (lane == 0) sxs[gl * 8 + n] = s;
  }
  cp_async_wait_all();
  __syncthreads();
  griddep_launch_dependents();

  // 4. Main loop: unpack, MMA, per-group scale/zero epilogue.
  float tot[4] = {0.f, 0.f, 0.f, 0.f};
  if (active) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
    const float4* szw = szs + (size_t)warp * a.gps * 8 + g;
    for (int q0 = 0; q0 < nq; q0 += kPipe) {
#pragma unroll
      for (int i = 0; i < kPipe; ++i) {
        const int q = q0 + i;
        if (q < nq) {
          const uint4 w = buf[i];
          if (q + kPipe < nq) buf[i] = ldg_stream(wp + (size_t)(q + kPipe) * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t word = (&w.x)[j];
            const uint32_t a0 = nib2_to_bf16x2(word);
            const uint32_t a1 = nib2_to_bf16x2(word >> 4);
            const uint32_t a2 = nib2_to_bf16x2(word >> 8);
            const uint32_t a3 = nib2_to_bf16x2(word >> 12);
            const int ktl = q * 4 + j;
            if (MODE == 1) {
              const uint2 b = reinterpret_cast<const uint2*>(xs)[ktl * 32 + lane];
              mma_bf16_16816(acc, a0, a1, a2, a3, b.x, b.y);
            } else {
              const uint4 b = reinterpret_cast<const uint4*>(xs)[ktl * 32 + lane];
              mma_bf16_16816(acc, a0, a1, a2, a3, b.x, b.y);
              mma_bf16_16816(acc2, a0, a1, a2, a3, b.z, b.w);
            }
          }
          if ((q + 1) % a.kqg == 0) {
            const int gl = q / a.kqg;
            const float4 s = szw[gl * 8];
            const float2 sx = *reinterpret_cast<const float2*>(&sxs[gl * 8 + 2 * t]);
            if (MODE == 1) {
              // columns 2t, 2t+1: hi part of m = 2t, 2t+1 when t < 2, lo part otherwise
              const float sx0 = t < 2 ? sx.x : 0.0f, sx1 = t < 2 ? sx.y : 0.0f;
              tot[0] = fmaf(s.x, fmaf(-s.y, sx0, acc[0]), tot[0]);
              tot[1] = fmaf(s.x, fmaf(-s.y, sx1, acc[1]), tot[1]);
              tot[2] = fmaf(s.z, fmaf(-s.w, sx0, acc[2]), tot[2]);
              tot[3] = fmaf(s.z, fmaf(-s.w, sx1, acc[3]), tot[3]);
            } else {
              tot[0] = fmaf(s.x, fmaf(-s.y, sx.x, acc[0] + acc2[0]), tot[0]);
              tot[1] = fmaf(s.x, fmaf(-s.y, sx.y, acc[1] + acc2[1]), tot[1]);
              tot[2] = fmaf(s.z, fmaf(-s.w, sx.x, acc[2] + acc2[2]), tot[2]);
              tot[3] = fmaf(s.z, fmaf(-s.w, sx.y, acc[3] + acc2[3]), tot[3]);
#pragma unroll
              for (int c = 0; c < 4; ++c) acc2[c] = 0.f;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[c] = 0.f;
          }
        }
      }
    }
    if (MODE == 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c) tot[c] += __shfl_xor_sync(0xffffffffu, tot[c], 2);
    }
  }

  // 5. Output.  Lane (g, t) holds rows (g, g+8) x columns m = 2t, 2t+1
  //    (MODE 1: only t < 2 carries results).
  const bool lane_has = MODE == 1 ? (t < 2) : true;
  if (nsplit == 1) {
    if (active && lane_has) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int row = rt * 16 + g + ((c & 2) ? 8 : 0);
        const int mm = 2 * t + (c & 1);
        if (row < a.rows && mm < a.m) a.y[(size_t)mm * a.ldy + row] = tot[c];
      }
    }
    return;
  }
  // part[warp][16 rows][8 cols]
  if (lane_has) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int r = g + ((c & 2) ? 8 : 0);
      const int mm = 2 * t + (c & 1);
      part[(warp * 16 + r) * 8 + mm] = active ? tot[c] : 0.0f;
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int rank = (int)cluster.block_rank();
  const int total = kWarps * 16 * 8;
  for (int e = rank * blockDim.x + threadIdx.x; e < total; e += nsplit * blockDim.x) {
    const int mm = e & 7;
    const int rr = e >> 3;  // warp*16 + r
    const int row = blockIdx.x * kWarps * 16 + rr;
    if (mm >= a.m || row >= a.rows) continue;
    float s = 0.0f;
    for (int r = 0; r < nsplit; ++r) s += cluster.map_shared_rank(part, r)[e];
    a.y[(size_t)mm * a.ldy + row] = s;
  }
  cluster.sync();
}

// Any group size (including <= 0, one group per row), any K: one warp per
// output row, reference arithmetic for each dequantised weight.
__global__ void q4g_gemv_generic(const uint8_t* __restrict__ wq, const float* __restrict__ sc,
                                 const float* __restrict__ zp, int64_t rows, int64_t k,
                                 int64_t gs, int64_t ngr, const float* __restrict__ x,
                                 int64_t ldx, int m, float* __restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t bpr = (k + 1) / 2;
  griddep_wait();
  for (int64_t row = warp; row < rows; row += nwarps) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int64_t c = lane; c < k; c += 32) {
      const uint8_t b = wq[row * bpr + (c >> 1)];
      const uint32_t nib = (c & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
      const int64_t gg = gs > 0 ? c / gs : 0;
      const float w = __fmul_rn(__fsub_rn((float)nib, zp[row * ngr + gg]), sc[row * ngr + gg]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < m) acc[i] = fmaf(w, x[i * ldx + c], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < m) {
        const float s = warp_sum(acc[i]);
        if (lane == 0) y[i * ldy + row] = s;
      }
    }
  }
}

inline unsigned grid1d(int64_t n, int block) { return (unsigned)((n + block - 1) / block); }

}  // namespace

int q4g_build(Weight* wt, const uint8_t* wq_dev, const float* sc_dev, const float* zp_dev,
              int64_t row_begin, int64_t rows, int64_t n_full, int64_t k, int64_t gs,
              int64_t ngr, cudaStream_t st) {
  (void)n_full;
  Q4GWeight& w = wt->q4;
  w.rows = rows;
  w.k = k;
  w.gs = gs;
  w.ngr = ngr;
  const int64_t bpr = (k + 1) / 2;
  const uint8_t* src = wq_dev + row_begin * bpr;
  const float* scs = sc_dev + row_begin * ngr;
  const float* zps = zp_dev + row_begin * ngr;
  w.fast = gs > 0 && gs % 64 == 0;
  if (w.fast) {
    w.n_rt = (rows + 15) / 16;
    const int64_t kp = ((k + gs - 1) / gs) * gs;
    w.kq_total = kp / 64;
    w.groups = kp / gs;
    const int64_t nfrag = w.n_rt * w.kq_total * 32;
    const int64_t nsz = w.n_rt * w.groups * 8;
    NIMF_TRY(device_alloc(&w.frag, (size_t)nfrag * 16));
    NIMF_TRY(device_alloc(&w.sz, (size_t)nsz * 16));
    wt->device_bytes = nfrag * 16 + nsz * 16;
    if (nfrag > 0)
      q4g_repack_frag<<<grid1d(nfrag, 256), 256, 0, st>>>(src, bpr, rows, k, w.kq_total, nfrag,
                                                          (uint4*)w.frag);
    if (nsz > 0)
      q4g_repack_sz<<<grid1d(nsz, 256), 256, 0, st>>>(scs, zps, ngr, rows, w.groups, nsz,
                                                      (float4*)w.sz);
    NIMF_CUDA_TRY(cudaGetLastError());
  } else {
    const size_t nb = (size_t)(rows * bpr);
    const size_t ns = (size_t)(rows * ngr) * sizeof(float);
    NIMF_TRY(device_alloc(&w.raw, nb ? nb : 1));
    NIMF_TRY(device_alloc(&w.scales, ns ? ns : 4));
    NIMF_TRY(device_alloc(&w.zeros, ns ? ns : 4));
    if (nb) NIMF_CUDA_TRY(cudaMemcpyAsync(w.raw, src, nb, cudaMemcpyDeviceToDevice, st));
    if (ns) NIMF_CUDA_TRY(cudaMemcpyAsync(w.scales, scs, ns, cudaMemcpyDeviceToDevice, st));
    if (ns) NIMF_CUDA_TRY(cudaMemcpyAsync(w.zeros, zps, ns, cudaMemcpyDeviceToDevice, st));
    wt->device_bytes = (int64_t)(nb + 2 * ns);
  }
  return NIMF_OK;
}

int q4g_dequant(const Q4GWeight& w, float* out, cudaStream_t st) {
  const int64_t n = w.rows * w.k;
  if (n == 0) return NIMF_OK;
  if (w.fast)
    q4g_dequant_frag<<<grid1d(n, 256), 256, 0, st>>>((const uint4*)w.frag, (const float4*)w.sz,
                                                     w.rows, w.k, w.kq_total, w.groups, w.gs,
                                                     out);
  else
    q4g_dequant_raw<<<grid1d(n, 256), 256, 0, st>>>((const uint8_t*)w.raw,
                                                    (const float*)w.scales,
                                                    (const float*)w.zeros, w.rows, w.k, w.gs,
                                                    w.ngr, out);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

namespace {

template <int MODE>
int launch_fast(const Q4GWeight& w, const float* x, int64_t ldx, int mc, float* y, int64_t ldy,
                int num_sms, cudaStream_t st) {
  const int kqg = (int)(w.gs / 64);
  const int bands = (int)((w.n_rt + kWarps - 1) / kWarps);
  const int groups = (int)w.groups;
  const int frag_bytes = MODE == 1 ? 8 : 16;
  const size_t per_group = (size_t)kqg * 4 * 32 * frag_bytes + 8 * sizeof(float) +
                           (size_t)kWarps * 8 * sizeof(float4);
  const size_t fixed = (size_t)kWarps * 16 * 8 * sizeof(float);
  const size_t budget = 96 * 1024;
  const int gps_max = (int)std::max<size_t>(1, (budget - fixed) / per_group);
  const int target_ctas = 4 * num_sms;
  int s = std::max((groups + gps_max - 1) / gps_max, (target_ctas + bands - 1) / bands);
  s = std::min(s, std::min(kMaxSplits, groups));
  s = std::max(s, 1);
  int gps = (groups + s - 1) / s;
  if (gps > gps_max)
    return set_error(NIMF_ERR_UNSUPPORTED, "q4g gemv: K=%lld too large for the split-K staging",
                     (long long)w.k);
  s = (groups + gps - 1) / gps;
  const size_t smem = fixed + per_group * (size_t)gps;

  GemvArgs a;
  a.frag = (const uint4*)w.frag;
  a.sz = (const float4*)w.sz;
  a.x = x;
  a.y = y;
  a.ldx = ldx;
  a.ldy = ldy;
  a.m = mc;
  a.k = (int)w.k;
  a.rows = (int)w.rows;
  a.n_rt = (int)w.n_rt;
  a.kq_total = (int)w.kq_total;
  a.kqg = kqg;
  a.gs = (int)w.gs;
  a.groups = groups;
  a.gps = gps;

  auto kern = q4g_gemv_kernel<MODE>;
  static bool attr_done = false;
  if (!attr_done) {
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)budget + 1024));
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)bands, (unsigned)s, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 1;
  attrs[0].val.clusterDim.y = (unsigned)s;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NIMF_OK;
}

}  // namespace

int q4g_gemv(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  Context* c = ctx();
  const int num_sms = c ? c->num_sms : 148;
  if (m <= 0 || w.rows <= 0) return NIMF_OK;
  if (w.k == 0) {
    for (int64_t i = 0; i < m; ++i)
      NIMF_CUDA_TRY(cudaMemsetAsync(y + i * w.rows, 0, (size_t)w.rows * sizeof(float), st));
    return NIMF_OK;
  }
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    const float* xc = x + m0 * w.k;
    float* yc = y + m0 * w.rows;
    if (w.fast) {
      if (mc <= 4) NIMF_TRY(launch_fast<1>(w, xc, w.k, mc, yc, w.rows, num_sms, st));
      else NIMF_TRY(launch_fast<2>(w, xc, w.k, mc, yc, w.rows, num_sms, st));
    } else {
      const int block = 256;
      const int64_t want = (w.rows * 32 + block - 1) / block;
      const unsigned grid = (unsigned)std::min<int64_t>(want, (int64_t)num_sms * 16);
      q4g_gemv_generic<<<grid, block, 0, st>>>((const uint8_t*)w.raw, (const float*)w.scales,
                                               (const float*)w.zeros, w.rows, w.k, w.gs, w.ngr,
                                               xc, w.k, mc, yc, w.rows);
      NIMF_CUDA_TRY(cudaGetLastError());
    }
  }
  return NIMF_OK;
}

}  // namespace nimf
