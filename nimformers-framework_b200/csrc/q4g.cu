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

#ifndef NIMF_Q4G_CONSUMERS
#define NIMF_Q4G_CONSUMERS 16
#endif
#ifndef NIMF_Q4G_STAGES
#define NIMF_Q4G_STAGES 32
#endif
#ifndef NIMF_Q4G_SMEM_KB
#define NIMF_Q4G_SMEM_KB 200
#endif
#ifndef NIMF_Q4G_CTAS_PER_SM
#define NIMF_Q4G_CTAS_PER_SM 1
#endif
constexpr int kCons = NIMF_Q4G_CONSUMERS;       // consumer warps per CTA
constexpr int kStages = NIMF_Q4G_STAGES;        // max units (16 rows x 512 k) in the ring
constexpr int kCtasPerSm = NIMF_Q4G_CTAS_PER_SM;
constexpr int kMaxSplits = 8;                   // portable cluster size
constexpr size_t kSmemBudget = (size_t)NIMF_Q4G_SMEM_KB * 1024;
constexpr int kMaxTilesPerCluster = 48;         // partial-y rows a cluster keeps in shared memory

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
  int* err;            // host-mapped error word (1: a bounded wait expired)
  int64_t ldx, ldy;
  int m, k, rows, n_rt;
  int kq_total, groups;
  int gps;             // quantisation groups per k-split (the last split may have fewer)
  int n_clusters;      // clusters in the grid; cluster size = number of k-splits
  int tchunk;          // max row tiles per cluster (sizes the partial-y buffers)
  int ns;              // stages in the weight ring (a multiple of kCons)
  int vec4;            // x rows 16-byte aligned
};

// A stage holds one row tile's slice of this CTA's k-split (packed weights,
// then the scale/zero pairs of its groups), moved by two bulk copies.  It is
// consumed as chunks of kChunkQ k-quads (512 k), one chunk per warp-unit.
constexpr int kChunkQ = 8;
constexpr int kIssuers = 4;  // producer lanes issuing stages round-robin

template <int MODE>
__host__ __device__ constexpr int xfrag_bytes() { return MODE == 1 ? 8 : 16; }

// Shared-memory layout of one CTA:
//   full/empty[kStages] mbarriers
//   ring[ns][stage]          row-tile slices of the k-split
//   xs   [k-tiles][cols][4]  compact B fragments of x (only columns that carry rows)
//   sxs  [gps][2][8]         per-group sums of the bf16 hi / lo parts of x
//   psum [2][M][64-k chunks] chunk sums used to build sxs
//   part [tchunk*nchunk][16][8] per-unit partial y, then summed per row tile
struct SmemLayout {
  size_t ring, stage, xs, sxs, psum, part, total;
};

__host__ __device__ inline SmemLayout q4g_smem_layout(int mode, int kqg, int gps, int m, int ns,
                                                      int tchunk) {
  SmemLayout L;
  const int cg = kChunkQ / kqg;                       // groups per chunk
  const int nchunk = (gps + cg - 1) / cg;
  L.stage = (size_t)gps * kqg * 512 + (size_t)gps * 128;  // a row tile's k-split
  L.ring = ((size_t)2 * kStages * sizeof(uint64_t) + 127) / 128 * 128;  // after the barriers
  L.xs = L.ring + L.stage * ns;
  const int cols = mode == 1 ? 2 * m : m;             // B columns holding data
  L.sxs = L.xs + (size_t)gps * kqg * 4 * cols * 4 * xfrag_bytes<1>() * (mode == 1 ? 1 : 2);
  L.psum = L.sxs + (size_t)gps * 16 * sizeof(float);
  const size_t nch = 2 * (((size_t)gps * kqg * 16 + 31) / 32);
  L.part = L.psum + 2 * (size_t)m * nch * sizeof(float);
  L.part = (L.part + 15) & ~(size_t)15;
  L.total = L.part + (size_t)tchunk * nchunk * 16 * 8 * sizeof(float);
  return L;
}

// One CTA = k-split `rank` of the row tiles of its cluster.  Warp kCons is the
// producer (one lane streams units with bulk copies); consumer warp w handles
// units (row tile i, chunk c) with (i * ncn + c) % kCons == w (ncn = nominal
// chunks per row tile, the same on every rank); stage
// i % ns of a row tile therefore always serves the same warps (ns is a multiple
// of kCons / gcd(ncn, kCons)),
// so no warp ever waits more than one phase ahead on a stage barrier.
// MODE 1: M <= 4, one MMA per k-tile (hi parts of x in columns 0..3, lo in 4..7).
// MODE 2: M <= 8, two MMAs per k-tile (hi and lo each in columns 0..7).
// KQG: k-quads (64 k) per quantisation group (group size 64 * KQG).
template <int MODE, int KQG>
__global__ void __launch_bounds__((kCons + 1) * 32, 1)
q4g_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int GS = 64 * KQG;
  constexpr int CG = kChunkQ / KQG;  // groups per chunk
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int nsplit = (int)cluster.num_blocks();
  const int cid = blockIdx.x / nsplit;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const int base = a.n_rt / a.n_clusters, rem = a.n_rt % a.n_clusters;
  const int rt0 = cid * base + min(cid, rem);
  const int nrt = base + (cid < rem ? 1 : 0);
  const int g0 = rank * a.gps;
  const int ng = max(0, min(a.gps, a.groups - g0));
  const int nchunk = (ng + CG - 1) / CG;          // chunks this rank actually has
  const int ncn = (a.gps + CG - 1) / CG;           // nominal chunks (same on every rank)
  const int nunits = nrt * ncn;
  const int NS = a.ns;
  const int cols = MODE == 1 ? 2 * a.m : a.m;

  const SmemLayout Ls = q4g_smem_layout(MODE, KQG, a.gps, a.m, NS, a.tchunk);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  unsigned char* ring = smem + Ls.ring;
  unsigned char* xs = smem + Ls.xs;
  float* sxs = reinterpret_cast<float*>(smem + Ls.sxs);
  float* psum = reinterpret_cast<float*>(smem + Ls.psum);
  float* part = reinterpret_cast<float*>(smem + Ls.part);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nchunk > 0 ? nchunk : 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kCons) {
    // ---------------- producer.  Weights do not depend on earlier kernels, so
    // this runs without griddepcontrol.wait and overlaps the previous kernel.
    // Lanes 0..kIssuers-1 own the stages s = lane (mod kIssuers).
    griddep_launch_dependents();
    if (lane < kIssuers) {
      bool ok = true;
      const uint32_t wb = (uint32_t)ng * KQG * 512u, zb = (uint32_t)ng * 128u;
      int issued_last = -1;
      for (int i = lane; i < nrt; i += kIssuers) {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
          ok = false;
          break;
        }
        const int rt = rt0 + i;
        unsigned char* dst = ring + (size_t)s * Ls.stage;
        mbar_arrive_expect_tx(&full[s], wb + zb);
        bulk_g2s(dst, a.frag + ((size_t)rt * a.kq_total + (size_t)g0 * KQG) * 32, wb, &full[s]);
        bulk_g2s(dst + (size_t)a.gps * KQG * 512, a.sz + ((size_t)rt * a.groups + g0) * 8, zb,
                 &full[s]);
        issued_last = i;
      }
      // drain: this lane's last copies land before the CTA may exit
      if (ok) {
        for (int i = issued_last; i >= 0 && i > issued_last - NS; i -= kIssuers)
          if (!mbar_wait(&full[i % NS], (i / NS) & 1)) ok = false;
      }
      if (!ok && a.err) atomicExch(a.err, 1);
    }
    __syncwarp();
  } else {
    // ---------------- consumers: stage x as compact B fragments + group sums
    griddep_wait();  // x may be written by the previous kernel in the stream
    {
      const int kb0 = g0 * GS;
      const int f4 = (ng * GS) >> 2;
      const int f4p = (f4 + 31) & ~31;
      const int nch = f4p >> 4;
      uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
      constexpr int kUnroll = 4;
      for (int it0 = threadIdx.x; it0 < a.m * f4p; it0 += kCons * 32 * kUnroll) {
        float4 vv[kUnroll];
#pragma unroll
        for (int r = 0; r < kUnroll; ++r) {  // issue all loads first
          const int it = it0 + r * kCons * 32;
          const int mrow = it / f4p, f = it - mrow * f4p;
          const int k = kb0 + 4 * f;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (it < a.m * f4p && f < f4) {
            const float* xr = a.x + (size_t)mrow * a.ldx + k;
            if (a.vec4 && k + 3 < a.k) {
              v = __ldg(reinterpret_cast<const float4*>(xr));
            } else {
              v.x = k < a.k ? __ldg(xr) : 0.f;
              v.y = k + 1 < a.k ? __ldg(xr + 1) : 0.f;
              v.z = k + 2 < a.k ? __ldg(xr + 2) : 0.f;
              v.w = k + 3 < a.k ? __ldg(xr + 3) : 0.f;
            }
          }
          vv[r] = v;
        }
#pragma unroll
        for (int r = 0; r < kUnroll; ++r) {
          const int it = it0 + r * kCons * 32;
          if (it >= a.m * f4p) break;  // uniform across the warp (f4p % 32 == 0)
          const int mrow = it / f4p, f = it - mrow * f4p;
          const float4 v = vv[r];
          float sh = 0.f, sl = 0.f;
          if (f < f4) {
            uint32_t h01, l01, h23, l23;
            split_bf16x2(v.x, v.y, h01, l01);
            split_bf16x2(v.z, v.w, h23, l23);
            sh = (bf16x2_lo(h01) + bf16x2_hi(h01)) + (bf16x2_lo(h23) + bf16x2_hi(h23));
            sl = (bf16x2_lo(l01) + bf16x2_hi(l01)) + (bf16x2_lo(l23) + bf16x2_hi(l23));
            // k offsets 4j..4j+3 of a 16-k tile feed lanes t = 2(j&1), 2(j&1)+1,
            // fragment word j>>1 (k 0..7 -> b0, k 8..15 -> b1)
            const int ktl = f >> 2, j = f & 3;
            const int t0 = 2 * (j & 1), word = j >> 1;
            if (MODE == 1) {
              // compact columns: hi of row m at m, lo of row m at M + m
              const size_t eh = ((size_t)ktl * cols + mrow) * 4 + t0;
              const size_t el = ((size_t)ktl * cols + a.m + mrow) * 4 + t0;
              xw[eh * 2 + word] = h01;
              xw[(eh + 1) * 2 + word] = h23;
              xw[el * 2 + word] = l01;
              xw[(el + 1) * 2 + word] = l23;
            } else {
              const size_t e = ((size_t)ktl * cols + mrow) * 4 + t0;
              xw[e * 4 + word] = h01;
              xw[(e + 1) * 4 + word] = h23;
              xw[e * 4 + 2 + word] = l01;
              xw[(e + 1) * 4 + 2 + word] = l23;
            }
          }
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) {
            sh += __shfl_xor_sync(0xffffffffu, sh, o);
            sl += __shfl_xor_sync(0xffffffffu, sl, o);
          }
          if ((lane & 15) == 0) {
            psum[mrow * nch + (f >> 4)] = sh;
            psum[(a.m + mrow) * nch + (f >> 4)] = sl;
          }
        }
      }
      named_barrier(1, kCons * 32);
      for (int e = threadIdx.x; e < ng * 16; e += kCons * 32) {
        const int gl = e >> 4, part_lo = (e >> 3) & 1, n = e & 7;
        float s = 0.f;
        if (n < a.m) {
          const float* ps = psum + (part_lo * a.m + n) * nch + gl * KQG;
#pragma unroll
          for (int c = 0; c < KQG; ++c) s += ps[c];
        }
        sxs[e] = s;
      }
      named_barrier(1, kCons * 32);
    }
    griddep_launch_dependents();

    // lane (n = g, t) carries B column n
    const int mcol = MODE == 1 ? (g & 3) : g;
    const bool bvalid = mcol < a.m;
    const int ccol = MODE == 1 ? (g < 4 ? mcol : a.m + mcol) : mcol;  // compact column
    const int sx_off = MODE == 1 ? (t < 2 ? 2 * t : 2 * t + 4) : 2 * t;
    const bool lane_has = MODE == 1 ? (t < 2) : true;
    const uint2* xs2 = reinterpret_cast<const uint2*>(xs) + ccol * 4 + t;
    const uint4* xs4 = reinterpret_cast<const uint4*>(xs) + ccol * 4 + t;

    for (int u = warp; u < nunits; u += kCons) {
      const int i = u / ncn, c = u - i * ncn;
      if (c >= nchunk) continue;  // the last k-split may have fewer chunks
      const int s = i % NS;
      const int cg0 = c * CG, ncg = min(CG, ng - cg0);
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      if (!mbar_wait(&full[s], (i / NS) & 1)) {
        if (lane == 0 && a.err) atomicExch(a.err, 1);
      } else {
        const unsigned char* st = ring + (size_t)s * Ls.stage;
        const uint4* wq = reinterpret_cast<const uint4*>(st + (size_t)c * kChunkQ * 512) + lane;
        const float4* szp =
            reinterpret_cast<const float4*>(st + (size_t)a.gps * KQG * 512 + (size_t)cg0 * 128) + g;
        // one accumulator set per group of the chunk: CG independent MMA chains
        float acc[CG][4], acc2[MODE == 2 ? CG : 1][4];
#pragma unroll
        for (int gl = 0; gl < CG; ++gl)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[gl][q] = 0.f;
            acc2[MODE == 2 ? gl : 0][q] = 0.f;
          }
#pragma unroll
        for (int gl = 0; gl < CG; ++gl) {
          if (gl < ncg) {
#pragma unroll
            for (int qq = 0; qq < KQG; ++qq) {
              const int ql = gl * KQG + qq;                // quad within the chunk
              const uint4 w = wq[ql * 32];
              const int kt0 = (cg0 * KQG + ql) * 4;        // k-tile within the CTA range
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const uint32_t word = jj == 0 ? w.x : (jj == 1 ? w.y : (jj == 2 ? w.z : w.w));
                const uint32_t a0 = lop3_and_or(word, 0x000F000Fu, 0x43004300u);
                const uint32_t a1 = lop3_and_or(word >> 4, 0x000F000Fu, 0x43004300u);
                const uint32_t a2 = lop3_and_or(word >> 8, 0x000F000Fu, 0x43004300u);
                const uint32_t a3 = lop3_and_or(word >> 12, 0x000F000Fu, 0x43004300u);
                const int kt = kt0 + jj;
                if (MODE == 1) {
                  uint2 b = make_uint2(0u, 0u);
                  if (bvalid) b = xs2[(size_t)kt * cols * 4];
                  mma_bf16_16816(acc[gl], a0, a1, a2, a3, b.x, b.y);
                } else {
                  uint4 b = make_uint4(0u, 0u, 0u, 0u);
                  if (bvalid) b = xs4[(size_t)kt * cols * 4];
                  mma_bf16_16816(acc[gl], a0, a1, a2, a3, b.x, b.y);
                  mma_bf16_16816(acc2[MODE == 2 ? gl : 0], a0, a1, a2, a3, b.z, b.w);
                }
              }
            }
          }
        }
        // per-group epilogues: sum_k (n - zp) x = acc - (128 + zp) sum_k x
#pragma unroll
        for (int gl = 0; gl < CG; ++gl) {
          if (gl < ncg) {
            const float4 sp = szp[gl * 8];
            const float zg = 128.0f + sp.y, zg8 = 128.0f + sp.w;
            const int glc = cg0 + gl;                      // group within the CTA range
            const float2 sx = *reinterpret_cast<const float2*>(&sxs[glc * 16 + sx_off]);
            if (MODE == 1) {
              tot[0] = fmaf(sp.x, fmaf(-zg, sx.x, acc[gl][0]), tot[0]);
              tot[1] = fmaf(sp.x, fmaf(-zg, sx.y, acc[gl][1]), tot[1]);
              tot[2] = fmaf(sp.z, fmaf(-zg8, sx.x, acc[gl][2]), tot[2]);
              tot[3] = fmaf(sp.z, fmaf(-zg8, sx.y, acc[gl][3]), tot[3]);
            } else {
              const float2 sl = *reinterpret_cast<const float2*>(&sxs[glc * 16 + 8 + sx_off]);
              const int g2 = MODE == 2 ? gl : 0;
              tot[0] = fmaf(sp.x, fmaf(-zg, sx.x, acc[gl][0]) + fmaf(-zg, sl.x, acc2[g2][0]), tot[0]);
              tot[1] = fmaf(sp.x, fmaf(-zg, sx.y, acc[gl][1]) + fmaf(-zg, sl.y, acc2[g2][1]), tot[1]);
              tot[2] = fmaf(sp.z, fmaf(-zg8, sx.x, acc[gl][2]) + fmaf(-zg8, sl.x, acc2[g2][2]), tot[2]);
              tot[3] = fmaf(sp.z, fmaf(-zg8, sx.y, acc[gl][3]) + fmaf(-zg8, sl.y, acc2[g2][3]), tot[3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (MODE == 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) tot[q] += __shfl_xor_sync(0xffffffffu, tot[q], 2);
      }
      if (lane_has) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = g + ((q & 2) ? 8 : 0);
          const int mm = 2 * t + (q & 1);
          part[((size_t)u * 16 + r) * 8 + mm] = tot[q];
        }
      }
    }
  }
  // sum the chunks of each row tile locally (chunk order) into the now idle
  // ring, then over the cluster's k-splits (rank order): deterministic.
  __syncthreads();
  float* sums = reinterpret_cast<float*>(ring);
  for (int e = threadIdx.x; e < nrt * 128; e += blockDim.x) {
    const int i = e >> 7, r = e & 127;
    float s = 0.f;
    for (int c = 0; c < nchunk; ++c) s += part[((size_t)(i * ncn + c)) * 128 + r];
    sums[e] = s;
  }
  cluster.sync();
  const int total = nrt * 128;
  for (int e = rank * blockDim.x + threadIdx.x; e < total; e += nsplit * blockDim.x) {
    const int mm = e & 7;
    const int row = rt0 * 16 + (e >> 3);
    if (mm >= a.m || row >= a.rows) continue;
    float s = 0.0f;
    for (int r = 0; r < nsplit; ++r) s += cluster.map_shared_rank(sums, r)[e];
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
  w.fast = gs == 64 || gs == 128 || gs == 256;
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

// Launches the GEMV over row tiles [rt_begin, rt_begin + n_rt) of w.
template <int MODE, int KQG>
int launch_fast(const Q4GWeight& w, int64_t rt_begin, int n_rt, const float* x, int64_t ldx,
                int mc, float* y, int64_t ldy, int num_sms, cudaStream_t st) {
  Context* c = ctx();
  const int groups = (int)w.groups;
  const int slots = num_sms * kCtasPerSm;
  auto kern = q4g_gemv_kernel<MODE, KQG>;
  static int attr_dev = -1;
  static int max_active[kMaxSplits + 1];
  if (c && attr_dev != c->device) {
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBudget));
    // clusters of each size that fit on the GPU at once (GPC boundaries make
    // this less than SMs / size for sizes that do not divide a GPC)
    for (int cs = 1; cs <= kMaxSplits; ++cs) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3((unsigned)(cs * 64), 1, 1);
      q.blockDim = dim3((kCons + 1) * 32, 1, 1);
      q.dynamicSmemBytes = kSmemBudget;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = (unsigned)cs;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      q.attrs = at;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) n = slots / cs;
      max_active[cs] = n;
    }
    cudaGetLastError();
    attr_dev = c->device;
  }
  // Pick the k-split count (= cluster size): feasible shared memory with at
  // least kCons ring stages (row-tile slices); score = estimated time relative to
  // a balanced full-GPU run (SM utilisation x row-tile balance).
  int best_s = -1, best_gps = 0, best_nclu = 1, best_ns = 0;
  double best_score = 1e30;
  for (int s = 1; s <= kMaxSplits; ++s) {
    const int gps = (groups + s - 1) / s;
    const int ss = (groups + gps - 1) / gps;
    if (ss != s) continue;
    const int act = (c && attr_dev == c->device) ? max_active[ss] : slots / ss;
    const int nclu = std::max(1, std::min(n_rt, act));
    const int tchunk = (n_rt + nclu - 1) / nclu;
    const SmemLayout L0 = q4g_smem_layout(MODE, KQG, gps, mc, 0, tchunk);
    if (L0.total >= kSmemBudget) continue;
    const size_t stage = L0.stage;
    // stage i % ns serves warps (i * nchunk + c) % kCons: keep ns a multiple of
    // that period so every stage always serves the same warps
    const int nchunk = (gps + kChunkQ / KQG - 1) / (kChunkQ / KQG);
    int gcdv = kCons, bb = nchunk;
    while (bb) { const int tmp = gcdv % bb; gcdv = bb; bb = tmp; }
    const int period = std::max(kCons / gcdv, kIssuers);
    int ns = (int)((kSmemBudget - L0.total) / stage);
    ns = std::min(ns, kStages) / period * period;
    if (ns < std::max(period, 4) || (size_t)ns * stage < (size_t)tchunk * 512) continue;
    const double util = std::min(1.0, (double)ss * nclu / slots);
    const double balance = (double)tchunk * nclu / n_rt;
    const double score = balance / util;
    if (score < best_score - 1e-9) {
      best_score = score;
      best_s = ss;
      best_gps = gps;
      best_nclu = nclu;
      best_ns = ns;
    }
  }
  if (best_s < 0)
    return set_error(NIMF_ERR_UNSUPPORTED, "q4g gemv: K=%lld, M=%d does not fit the staging",
                     (long long)w.k, mc);
  const int s = best_s, gps = best_gps, n_clusters = best_nclu, ns = best_ns;
  const int tchunk = (n_rt + n_clusters - 1) / n_clusters;
  const SmemLayout L = q4g_smem_layout(MODE, KQG, gps, mc, ns, tchunk);

  GemvArgs a;
  a.frag = (const uint4*)w.frag + (size_t)rt_begin * w.kq_total * 32;
  a.sz = (const float4*)w.sz + (size_t)rt_begin * w.groups * 8;
  a.x = x;
  a.y = y + rt_begin * 16;
  a.err = c ? c->dev_err : nullptr;
  a.ldx = ldx;
  a.ldy = ldy;
  a.m = mc;
  a.k = (int)w.k;
  a.rows = (int)std::min<int64_t>((int64_t)n_rt * 16, w.rows - rt_begin * 16);
  a.n_rt = n_rt;
  a.kq_total = (int)w.kq_total;
  a.groups = groups;
  a.gps = gps;
  a.n_clusters = n_clusters;
  a.tchunk = tchunk;
  a.ns = ns;
  a.vec4 = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 4 == 0);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_clusters * s), 1, 1);
  cfg.blockDim = dim3((kCons + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = (unsigned)s;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NIMF_OK;
}

// Row tiles per launch are capped so a cluster holds at most kMaxTilesPerCluster
// partial row tiles in shared memory.
template <int MODE, int KQG>
int launch_rows(const Q4GWeight& w, const float* x, int64_t ldx, int mc, float* y, int64_t ldy,
                int num_sms, cudaStream_t st) {
  const int64_t cap = (int64_t)kMaxTilesPerCluster * std::max(1, num_sms * kCtasPerSm / kMaxSplits);
  for (int64_t r0 = 0; r0 < w.n_rt; r0 += cap) {
    const int n = (int)std::min<int64_t>(cap, w.n_rt - r0);
    NIMF_TRY((launch_fast<MODE, KQG>(w, r0, n, x, ldx, mc, y, ldy, num_sms, st)));
  }
  return NIMF_OK;
}

template <int MODE>
int launch_mode(const Q4GWeight& w, const float* x, int64_t ldx, int mc, float* y, int64_t ldy,
                int num_sms, cudaStream_t st) {
  switch (w.gs) {
    case 64: return launch_rows<MODE, 1>(w, x, ldx, mc, y, ldy, num_sms, st);
    case 128: return launch_rows<MODE, 2>(w, x, ldx, mc, y, ldy, num_sms, st);
    case 256: return launch_rows<MODE, 4>(w, x, ldx, mc, y, ldy, num_sms, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "q4g fast path: group size %lld", (long long)w.gs);
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
      if (mc <= 4) NIMF_TRY(launch_mode<1>(w, xc, w.k, mc, yc, w.rows, num_sms, st));
      else NIMF_TRY(launch_mode<2>(w, xc, w.k, mc, yc, w.rows, num_sms, st));
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
