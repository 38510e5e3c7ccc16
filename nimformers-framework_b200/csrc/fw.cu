// fw.cu -- tensor-core GEMV for the byte-coded float weight formats:
//   int8 symmetric (quant.nim:51-67, per-tensor or per-row scale),
//   one-byte CustomFloat E4M3 = CustomFloat(4,3) and E5M2 = CustomFloat(5,2)
//     (customfloat.nim:49-102, quant.nim:243,254; optional per-row scale),
//   FP4 E2M1 with an OCP-E4M3 scale per 16 k and a tensor scale (extension).
//
// Every weight value of these formats is exactly representable in fp16:
// int8 (|q| <= 127), E4M3 / E5M2 codes whose reference decoding equals the
// OCP decoding (all codes except exponent field all-ones, which the reference
// decodes as inf, and exponent 0 with a non-zero mantissa, which the reference
// decodes as 2^-bias (1.m); the encoder never emits either), and the product
// e2m1 x e4m3 (at most 6 significant bits, magnitude in [2^-10, 2688]).  So
// the weights are decoded exactly into fp16 mma.sync A fragments.  For M <= 4
// x is split into fp16 hi + lo parts after a per-row power-of-two scale
// (x ~= (hi + lo) 2^-p to about 2^-22 relative) and both parts share one MMA
// (hi in columns 0..3, lo in 4..7); for 5 <= M <= 16 x is one fp16 term, the
// x precision of the tensor-core GEMM (fw_tc.cu: about 2e-4 of max|y|), which
// halves the MMAs and B loads per weight tile.  Products accumulate in fp32;
// the per-row / tensor scales are applied once per output in fp32.
//
// Layout (built once at registration, the reference bytes are kept too):
//   frag  [n_rt][ntk][32 lanes] uint4 -- one 512-byte tile per 16 rows x TK k
//         (TK = 32 for one-byte codes, 64 for FP4).  Lane (g, t) holds the A
//         fragments of mma.m16n8k16 for rows g, g+8 of every 16-k subtile j:
//         one-byte codes: word 2j   = {(g, 2t..2t+1), (g+8, 2t..2t+1)}
//                         word 2j+1 = {(g, 2t+8..2t+9), (g+8, 2t+8..2t+9)}
//                         (k relative to the subtile, the lower k in the lower byte)
//         FP4:            word j, byte p = register a_p of subtile j
//                         (p: 0 (g, 2t..), 1 (g+8, 2t..), 2 (g, 2t+8..), 3 (g+8, 2t+8..)),
//                         the lower k in the low nibble.
//   sfrag (FP4) [n_rt][ntk][8 g] uint2 -- byte 2j + h = block scale of row
//         g + 8h for subtile j.
//
// Kernel: one CTA of 16 warps per SM.  A CTA owns a balanced range of row
// tiles and one k-split; its x slice is staged in shared memory as hi/lo fp16
// rows, permuted within every 16 k so that a lane's two B registers are one
// 8-byte load.  The CTA's (row tile, 8-tile chunk) units are cut into 16
// equal contiguous ranges, one per warp; each warp streams its chunks with
// 128-bit loads (the next chunk is in flight while the current one is
// multiplied), keeps one accumulator per row tile and parks it in shared
// memory when the row tile changes.  The partials of a row tile are summed in
// warp order (deterministic).  With several k-splits, each split writes its
// partial to a scratch buffer and the last CTA of a row group to arrive sums
// the splits in order.
#include <cuda_fp16.h>

#include <algorithm>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr int kFwWarps = 16;
constexpr int kFwThreads = kFwWarps * 32;
constexpr int kChunkTiles = 8;             // tiles per load batch of a warp
constexpr size_t kFwXBudget = 160 * 1024;  // shared memory for the x slice
constexpr int kFwMaxM = 16;
constexpr size_t kFwSmemMax = 220 * 1024;  // dynamic shared memory per CTA

__host__ __device__ constexpr int fw_tk(int fmt) { return fmt == FW_FP4 ? 64 : 32; }

// ------------------------------------------------------------------ conversions
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t v16) {
  uint32_t r;
  const unsigned short h = (unsigned short)v16;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e5m2x2(uint32_t v16) {
  uint32_t r;
  const unsigned short h = (unsigned short)v16;
  asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}
// Two e2m1 codes in the low byte of v (lower k in the low nibble) -> f16x2.
__device__ __forceinline__ uint32_t cvt_e2m1x2(uint32_t v) {
  uint32_t r;
  const unsigned short h = (unsigned short)(v & 0xFFu);
  asm("{ .reg .b8 lo, hi;\n"
      "  mov.b16 {lo, hi}, %1;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, lo; }"
      : "=r"(r)
      : "h"(h));
  return r;
}
// Two int8 codes in bytes b and b+1 of w -> f16x2 (exact): the biased byte
// q + 128 becomes the low mantissa byte of 1024 + (q + 128), then 1152 is
// subtracted.
template <int B>
__device__ __forceinline__ uint32_t cvt_s8x2(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(u), "r"(0x64646464u), "r"(B == 0 ? 0x4140u : 0x4342u));
  const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&r), __half2half2(__ushort_as_half(0x6480)));
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// A fragments (4 registers) of subtile j of one lane's 16-byte tile slice.
template <int FMT>
__device__ __forceinline__ void tile_a(const uint4& w, uint32_t sw, int j, uint32_t (&a)[4]) {
  const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
  if (FMT == FW_FP4) {
    // block scales of rows g and g+8 for this subtile, broadcast per row
    const uint32_t s2 = cvt_e4m3x2(sw);
    uint32_t sg, sg8;
    asm("prmt.b32 %0, %1, %1, 0x1010;" : "=r"(sg) : "r"(s2));
    asm("prmt.b32 %0, %1, %1, 0x3232;" : "=r"(sg8) : "r"(s2));
    // the word's four bytes (registers a0..a3 of the subtile) are split once
    uint32_t c[4];
    asm("{ .reg .b8 b0, b1, b2, b3;\n"
        "  mov.b32 {b0, b1, b2, b3}, %4;\n"
        "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
        "  cvt.rn.f16x2.e2m1x2 %3, b3; }"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(wd[j]));
    a[0] = hmul2_u(c[0], sg);
    a[1] = hmul2_u(c[1], sg8);
    a[2] = hmul2_u(c[2], sg);
    a[3] = hmul2_u(c[3], sg8);
  } else {
    const uint32_t w0 = wd[2 * j], w1 = wd[2 * j + 1];
    if (FMT == FW_I8) {
      a[0] = cvt_s8x2<0>(w0);
      a[1] = cvt_s8x2<1>(w0);
      a[2] = cvt_s8x2<0>(w1);
      a[3] = cvt_s8x2<1>(w1);
    } else if (FMT == FW_E4M3) {
      a[0] = cvt_e4m3x2(w0);
      a[1] = cvt_e4m3x2(w0 >> 16);
      a[2] = cvt_e4m3x2(w1);
      a[3] = cvt_e4m3x2(w1 >> 16);
    } else {
      a[0] = cvt_e5m2x2(w0);
      a[1] = cvt_e5m2x2(w0 >> 16);
      a[2] = cvt_e5m2x2(w1);
      a[3] = cvt_e5m2x2(w1 >> 16);
    }
  }
}

// ------------------------------------------------------------------ repack
// One thread per (tile, lane) 16-byte slot of frag (and, for FP4 with lane
// t == 0, the 8-byte scale slot of row pair g).  Rows >= rows and k >= K are
// zero codes (and zero scales), so padded rows and columns add nothing.
template <int FMT>
__global__ void fw_repack_kernel(const uint8_t* __restrict__ raw, const uint8_t* __restrict__ bs,
                                 int64_t rows, int64_t k, int64_t ntk, int64_t total,
                                 uint4* __restrict__ frag, uint2* __restrict__ sfrag) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  constexpr int TK = fw_tk(FMT);
  const int lane = (int)(i & 31);
  const int64_t tile = i >> 5;
  const int64_t kt = tile % ntk, rt = tile / ntk;
  const int g = lane >> 2, t = lane & 3;
  uint32_t wd[4] = {0u, 0u, 0u, 0u};
  if (FMT == FW_FP4) {
    const int64_t bpr = (k + 1) / 2;
    for (int j = 0; j < 4; ++j)
      for (int p = 0; p < 4; ++p)
        for (int e = 0; e < 2; ++e) {
          const int64_t row = rt * 16 + g + 8 * (p & 1);
          const int64_t col = kt * TK + 16 * j + 2 * t + 8 * (p >> 1) + e;
          uint32_t nib = 0;
          if (row < rows && col < k) {
            const uint8_t b = raw[row * bpr + (col >> 1)];
            nib = (col & 1) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
          }
          wd[j] |= nib << (8 * p + 4 * e);
        }
    if (t == 0) {
      const int64_t nb = (k + 15) / 16;
      uint32_t s[2] = {0u, 0u};
      for (int j = 0; j < 4; ++j)
        for (int h = 0; h < 2; ++h) {
          const int64_t row = rt * 16 + g + 8 * h;
          const int64_t blk = kt * 4 + j;
          const uint32_t v = (row < rows && blk < nb) ? (uint32_t)bs[row * nb + blk] : 0u;
          const int byte = 2 * j + h;
          s[byte >> 2] |= v << (8 * (byte & 3));
        }
      sfrag[tile * 8 + g] = make_uint2(s[0], s[1]);
    }
  } else {
    for (int wi = 0; wi < 4; ++wi)
      for (int byte = 0; byte < 4; ++byte) {
        const int j = wi >> 1;
        const int ri = 2 * (wi & 1) + (byte >> 1);  // A register a0..a3
        const int e = byte & 1;
        const int64_t row = rt * 16 + g + 8 * (ri & 1);
        const int64_t col = kt * TK + 16 * j + 2 * t + 8 * (ri >> 1) + e;
        const uint32_t v = (row < rows && col < k) ? (uint32_t)raw[row * k + col] : 0u;
        wd[wi] |= v << (8 * byte);
      }
  }
  frag[i] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
}

// Counts one-byte CustomFloat codes whose reference decoding differs from the
// OCP decoding of the tensor-core conversion: exponent field all ones
// (reference: +-inf) or zero with a non-zero mantissa (reference: 2^-bias (1.m)).
__global__ void fw_count_special(const uint8_t* __restrict__ d, int64_t n, int mbits,
                                 unsigned* __restrict__ bad) {
  unsigned c = 0;
  const unsigned emask = (0x7Fu >> mbits), mmask = (1u << mbits) - 1u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned b = d[i];
    const unsigned e = (b >> mbits) & emask, mm = b & mmask;
    c += (e == emask || (e == 0 && mm != 0)) ? 1u : 0u;
  }
  if (c) atomicAdd(bad, c);
}

// ------------------------------------------------------------------ dequant
// Bit-exact dequantisation read back from the tensor-core layout through the
// same conversion instructions the GEMV uses, with the reference's roundings:
// int8 q * scale (quant.nim:64), CustomFloat value (* row scale), FP4
// e2m1 * (e4m3 * tensor scale).
template <int FMT>
__global__ void fw_dequant_kernel(const uint4* __restrict__ frag, const uint2* __restrict__ sfrag,
                                  const float* __restrict__ rscale, float uscale, int64_t rows,
                                  int64_t k, int64_t ntk, float* __restrict__ out) {
  constexpr int TK = fw_tk(FMT);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * k;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / k, col = i % k;
    const int64_t rt = row >> 4, kt = col / TK;
    const int r = (int)(row & 15), g = r & 7, hr = r >> 3;
    const int kk = (int)(col % TK);
    const int j = kk >> 4, k16 = kk & 15;
    const int hi8 = k16 >> 3, t = (k16 & 7) >> 1, e = k16 & 1;
    const int ri = hr + 2 * hi8;
    const int lane = 4 * g + t;
    const uint4 w = frag[(rt * ntk + kt) * 32 + lane];
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    float v;
    if (FMT == FW_FP4) {
      const uint32_t byte = (wd[j] >> (8 * ri)) & 0xFFu;
      const uint32_t h2 = cvt_e2m1x2(byte);
      const float q = __half2float(__ushort_as_half((unsigned short)(e ? (h2 >> 16) : (h2 & 0xFFFFu))));
      const uint2 sv = sfrag[(rt * ntk + kt) * 8 + g];
      const uint32_t sw = (j < 2 ? sv.x : sv.y) >> (16 * (j & 1));
      const uint32_t s2 = cvt_e4m3x2(sw);
      const float sc = __half2float(__ushort_as_half((unsigned short)(hr ? (s2 >> 16) : (s2 & 0xFFFFu))));
      v = __fmul_rn(q, __fmul_rn(sc, uscale));
    } else {
      const uint32_t word = wd[2 * j + (ri >> 1)];
      const uint32_t pair = (word >> (16 * (ri & 1))) & 0xFFFFu;
      uint32_t h2;
      if (FMT == FW_I8) h2 = cvt_s8x2<0>(pair);
      else if (FMT == FW_E4M3) h2 = cvt_e4m3x2(pair);
      else h2 = cvt_e5m2x2(pair);
      v = __half2float(__ushort_as_half((unsigned short)(e ? (h2 >> 16) : (h2 & 0xFFFFu))));
      const float s = rscale ? rscale[row] : uscale;
      if (FMT == FW_I8 || rscale) v = __fmul_rn(v, s);
    }
    out[i] = v;
  }
}

// ------------------------------------------------------------------ GEMV
struct FwArgs {
  const uint4* frag;
  const uint2* sfrag;
  const float* rscale;  // per-row epilogue scale (nullable: uscale for all rows)
  float uscale;
  const float* x;
  float* y;
  float* part;          // k-split partials [S][M][rows]
  unsigned* cnt;        // k-split arrival counters [G] (zero between launches)
  int64_t ldx, ldy;
  int m, rows, k;
  int n_rt, ntk;
  int S, ks_tiles, G;
  int xstride;          // halves per staged x row (slice + 16 pad)
  int nseg;             // partial slots per warp
  int vec4;             // x rows 16-byte aligned
};

// x scale: 2^p with max|x| 2^p in [2^14, 2^15), so hi and lo stay normal fp16.
__device__ __forceinline__ int fw_xscale_pow(unsigned maxbits) {
  if (maxbits == 0u) return 0;
  const int E = (int)((maxbits >> 23) & 0xFFu);
  return max(-126, min(126, 141 - E));
}

// Shared memory: xmax[16] | x hi [M][xstride] | x lo [M][xstride] (M <= 4 only) | partials.
// x terms staged per row: hi and lo for M <= 4, hi alone above.
__host__ __device__ inline int fw_xterms(int m) { return m <= 4 ? 2 : 1; }
__host__ __device__ inline size_t fw_smem_bytes(int m, int xstride, int nseg) {
  return 64 + (size_t)fw_xterms(m) * m * xstride * 2 + (size_t)kFwWarps * nseg * 16 * m * 4 + 16;
}

template <int FMT, int MODE>
__global__ void __launch_bounds__(kFwThreads, 1) fw_gemv_kernel(const FwArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int TK = fw_tk(FMT);
  constexpr int SUB = TK / 16;                       // 16-k subtiles per tile
  // B column blocks per MMA step: M <= 4 puts hi and lo of x rows 0..3 in
  // one block; M <= 8 (16) multiplies x rows 0..7 (and 8..15) as one fp16
  // term, the x precision of the GEMM path (about 2e-4 of max|y|)
  constexpr int NB = MODE == 3 ? 2 : 1;
  constexpr int NACC = MODE == 3 ? 2 : 1;
  // byte codes, MODE 1 / 2: two accumulator sets, alternating by 16-k
  // subtile, so that consecutive MMAs of a warp do not wait on each other;
  // summed at flush (FP4 is bound by its decode and has no registers left)
  constexpr int NPAR = (MODE == 3 || FMT == FW_FP4) ? 1 : 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int grp = blockIdx.x, split = blockIdx.y;
  const int base = a.n_rt / a.G, rem = a.n_rt % a.G;
  const int rt0 = grp * base + min(grp, rem);
  const int nrt = base + (grp < rem ? 1 : 0);
  const int kt0 = split * a.ks_tiles;
  const int nkt = max(0, min(a.ks_tiles, a.ntk - kt0));
  const int kbeg = kt0 * TK, klen = nkt * TK;
  const int cpr = (nkt + kChunkTiles - 1) / kChunkTiles;  // chunks per row tile
  const int C = nrt * cpr;
  const int c0 = (int)((int64_t)warp * C / kFwWarps);
  const int c1 = (int)((int64_t)(warp + 1) * C / kFwWarps);

  unsigned* xmax = reinterpret_cast<unsigned*>(smem);
  __half* xh = reinterpret_cast<__half*>(smem + 64);
  __half* xl = xh + (size_t)a.m * a.xstride;
  float* wpart = reinterpret_cast<float*>((MODE == 1 ? xl : xh) + (size_t)a.m * a.xstride);

  // first chunk of weights: issued before waiting on the previous kernel
  auto load_chunk = [&](int rl, int ch, uint4 (&wv)[kChunkTiles], uint2 (&sv)[kChunkTiles]) {
    const int kt = kt0 + ch * kChunkTiles;
    const int nt = min(kChunkTiles, kt0 + nkt - kt);
    const size_t tile0 = (size_t)(rt0 + rl) * a.ntk + kt;
    const uint4* src = a.frag + tile0 * 32 + lane;
#pragma unroll
    for (int j = 0; j < kChunkTiles; ++j)
      if (j < nt) wv[j] = ldg_stream(src + (size_t)j * 32);
    if (FMT == FW_FP4) {
      const uint2* ss = a.sfrag + tile0 * 8 + g;
#pragma unroll
      for (int j = 0; j < kChunkTiles; ++j)
        if (j < nt) sv[j] = ldg_stream2(ss + (size_t)j * 8);
    }
  };
  // the chunk after the next one is pulled into L2 by one bulk prefetch, so
  // the register loads of the next chunk find their lines in L2
  auto prefetch_chunk = [&](int rl, int ch) {
    const int kt = kt0 + ch * kChunkTiles;
    const int nt = min(kChunkTiles, kt0 + nkt - kt);
    const size_t tile0 = (size_t)(rt0 + rl) * a.ntk + kt;
    if (lane == 0) {
      bulk_prefetch_l2(a.frag + tile0 * 32, (uint32_t)nt * 512u);
      if (FMT == FW_FP4) bulk_prefetch_l2(a.sfrag + tile0 * 8, (uint32_t)nt * 64u);
    }
  };
  uint4 wv[kChunkTiles], nv[kChunkTiles];
  uint2 sv[kChunkTiles], nsv[kChunkTiles];
  // chunk c = rl cpr + ch: (rl, ch) of chunks c, c + 1 and c + 2 advance
  // without divisions
  auto next_rc = [&](int& rl, int& ch) {
    if (++ch == cpr) {
      ch = 0;
      ++rl;
    }
  };
  int rl0 = cpr > 0 ? c0 / cpr : 0, ch0 = c0 - rl0 * cpr;
  int rl1 = rl0, ch1 = ch0;
  next_rc(rl1, ch1);
  int rl2 = rl1, ch2 = ch1;
  next_rc(rl2, ch2);
  griddep_launch_dependents();
  if (c0 + 1 < c1) prefetch_chunk(rl1, ch1);
  if (c0 < c1) load_chunk(rl0, ch0, wv, sv);

  if (threadIdx.x < 16) xmax[threadIdx.x] = 0u;
  __syncthreads();
  griddep_wait();  // x may be written by the previous kernel in the stream

  // ---- stage x[:, kbeg : kbeg + klen) as hi / lo fp16 rows (permuted per 16 k)
  const int f4 = klen >> 2;
  // x item (mrow, j): float4 f = threadIdx.x + 512 j of row mrow; fpt items
  // per row, M fpt per thread, stepped as (mrow, j) without divisions.  A
  // warp's 32 lanes share (mrow, j) (512 is a multiple of 32), so the row
  // maxima reduce per warp; float4 past the slice load as zeros.
  const int fpt = (f4 + kFwThreads - 1) / kFwThreads;
  const int nit = a.m * fpt;
  auto load_x = [&](int mrow, int j) -> float4 {
    const int f = threadIdx.x + j * kFwThreads;
    const int k = kbeg + 4 * f;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (f < f4) {
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
    return v;
  };
  auto row_max = [&](int mrow, const float4& v) {
    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) atomicMax(&xmax[mrow], __float_as_uint(mx));
  };
  auto stage = [&](int mrow, int j, const float4& v) {
    const int f = threadIdx.x + j * kFwThreads;
    if (f >= f4) return;
    const float sc = ldexpf(1.0f, fw_xscale_pow(xmax[mrow]));
    const float xv[4] = {v.x * sc, v.y * sc, v.z * sc, v.w * sc};
    __half hv[4], lv[4];
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      hv[bb] = __float2half_rn(xv[bb]);
      lv[bb] = MODE == 1 ? __float2half_rn(xv[bb] - __half2float(hv[bb])) : __float2half_rn(0.f);
    }
    // k = 4f .. 4f+3 within the slice: positions in the permuted 16-k block
    const int kk = (4 * f) & 15, blk = (4 * f) >> 4;
    const int p0 = 4 * ((kk & 7) >> 1) + 2 * (kk >> 3);  // pair (k, k+1)
    const int p1 = 4 * (((kk + 2) & 7) >> 1) + 2 * ((kk + 2) >> 3);  // pair (k+2, k+3)
    __half* hr = xh + (size_t)mrow * a.xstride + blk * 16;
    __half* lr = xl + (size_t)mrow * a.xstride + blk * 16;
    *reinterpret_cast<__half2*>(hr + p0) = __halves2half2(hv[0], hv[1]);
    *reinterpret_cast<__half2*>(hr + p1) = __halves2half2(hv[2], hv[3]);
    if (MODE == 1) {
      *reinterpret_cast<__half2*>(lr + p0) = __halves2half2(lv[0], lv[1]);
      *reinterpret_cast<__half2*>(lr + p1) = __halves2half2(lv[2], lv[3]);
    }
  };
  auto next_item = [&](int& mrow, int& j) {
    if (++j == fpt) {
      j = 0;
      ++mrow;
    }
  };
  // Pass 1 finds each row's max|x|, pass 2 converts x into the staged fp16
  // rows; each pass issues a batch of loads before using any.  When a
  // thread's share is at most kXR float4, pass 1 keeps it in registers and
  // pass 2 reads nothing again (one L2 round trip and one read of x per CTA).
  constexpr int kXR = FMT == FW_FP4 ? 8 : 16;   // FP4 has fewer registers to spare
  if (nit <= kXR) {
    float4 v[kXR];
    int mr = 0, jj = 0;
#pragma unroll
    for (int r = 0; r < kXR; ++r) {
      v[r] = r < nit ? load_x(mr, jj) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < nit) next_item(mr, jj);
    }
    mr = 0, jj = 0;
#pragma unroll
    for (int r = 0; r < kXR; ++r) {
      if (r < nit) {
        row_max(mr, v[r]);
        next_item(mr, jj);
      }
    }
    __syncthreads();
    mr = 0, jj = 0;
#pragma unroll
    for (int r = 0; r < kXR; ++r) {
      if (r < nit) {
        stage(mr, jj, v[r]);
        next_item(mr, jj);
      }
    }
  } else {
    constexpr int kXB = 8;
    for (int pass = 0; pass < 2; ++pass) {
      int mr = 0, jj = 0;
      for (int i0 = 0; i0 < nit; i0 += kXB) {
        float4 v[kXB];
        int m0 = mr, j0 = jj;
#pragma unroll
        for (int r = 0; r < kXB; ++r) {
          v[r] = i0 + r < nit ? load_x(mr, jj) : make_float4(0.f, 0.f, 0.f, 0.f);
          if (i0 + r < nit) next_item(mr, jj);
        }
#pragma unroll
        for (int r = 0; r < kXB; ++r) {
          if (i0 + r < nit) {
            if (pass == 0) row_max(m0, v[r]);
            else stage(m0, j0, v[r]);
            next_item(m0, j0);
          }
        }
      }
      __syncthreads();
    }
  }
  __syncthreads();

  // B operand row of each column block for this lane (nullptr: zero column)
  const __half* bp[NB];
#pragma unroll
  for (int cb = 0; cb < NB; ++cb) {
    int xr;
    bool lo;
    if (MODE == 1) { xr = g & 3; lo = g >= 4; }
    else if (MODE == 2) { xr = g; lo = false; }
    else { xr = g + 8 * cb; lo = false; }
    bp[cb] = xr < a.m ? (lo ? xl : xh) + (size_t)xr * a.xstride + 4 * t : nullptr;
  }

  float acc[NACC * NPAR][4];
  int cur = -1;
  const int slot0 = cpr > 0 ? c0 / cpr : 0;
  auto flush = [&](int rl) {
    float v[NACC][4];
#pragma unroll
    for (int q = 0; q < NACC; ++q)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[q][e] = NPAR == 2 ? acc[2 * q][e] + acc[2 * q + 1][e] : acc[q][e];
    if (MODE == 1) {
      // columns 4..7 hold the lo parts of x rows 0..3
#pragma unroll
      for (int e = 0; e < 4; ++e) v[0][e] += __shfl_xor_sync(0xffffffffu, v[0][e], 2);
    }
    float* dst = wpart + ((size_t)warp * a.nseg + (rl - slot0)) * 16 * a.m;
#pragma unroll
    for (int q = 0; q < NACC; ++q) {
      const int mb = 8 * q + 2 * t;
      if (MODE == 1 && t >= 2) continue;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int mcol = mb + e;
        if (mcol < a.m) {
          dst[g * a.m + mcol] = v[q][e];
          dst[(g + 8) * a.m + mcol] = v[q][2 + e];
        }
      }
    }
  };

#pragma unroll 1
  for (int c = c0; c < c1; ++c) {
    const int rl = rl0, ch = ch0;
    if (rl != cur) {
      if (cur >= 0) flush(cur);
      cur = rl;
#pragma unroll
      for (int q = 0; q < NACC * NPAR; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[q][e] = 0.f;
    }
    if (c + 2 < c1) prefetch_chunk(rl2, ch2);
    if (c + 1 < c1) load_chunk(rl1, ch1, nv, nsv);
    rl0 = rl1, ch0 = ch1;
    rl1 = rl2, ch1 = ch2;
    next_rc(rl2, ch2);
    const int nt = min(kChunkTiles, nkt - ch * kChunkTiles);
    // B rows of this chunk's first 16-k subtile (then constant offsets)
    const __half* bq[NB];
#pragma unroll
    for (int cb = 0; cb < NB; ++cb) bq[cb] = bp[cb] ? bp[cb] + (size_t)ch * kChunkTiles * SUB * 16 : nullptr;
#pragma unroll
    for (int j = 0; j < kChunkTiles; ++j) {
      if (j < nt) {
#pragma unroll
        for (int sub = 0; sub < SUB; ++sub) {
          const uint32_t swv = FMT == FW_FP4 ? ((sub < 2 ? sv[j].x : sv[j].y) >> (16 * (sub & 1))) : 0u;
          uint32_t af[4];
          tile_a<FMT>(wv[j], swv, sub, af);
#pragma unroll
          for (int cb = 0; cb < NB; ++cb) {
            uint2 b = make_uint2(0u, 0u);
            if (bq[cb]) b = *reinterpret_cast<const uint2*>(bq[cb] + (j * SUB + sub) * 16);
            mma_f16_16816(acc[MODE == 3 ? (cb & 1) : (NPAR == 2 ? (sub & 1) : 0)], af[0], af[1], af[2], af[3], b.x, b.y);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kChunkTiles; ++j) {
      wv[j] = nv[j];
      if (FMT == FW_FP4) sv[j] = nsv[j];
    }
  }
  if (cur >= 0) flush(cur);
  __syncthreads();

  // ---- sum the warps' partials of each row tile in warp order; the row
  // tiles [s0, s1] each warp touched are worked out once per CTA
  __shared__ int wrange[kFwWarps][2];
  if (threadIdx.x < kFwWarps) {
    const int w = threadIdx.x;
    const int w0 = (int)((int64_t)w * C / kFwWarps), w1 = (int)((int64_t)(w + 1) * C / kFwWarps);
    wrange[w][0] = w1 > w0 ? w0 / cpr : 1;
    wrange[w][1] = w1 > w0 ? (w1 - 1) / cpr : 0;
  }
  __syncthreads();
  const int items = nrt * 16 * a.m;
  for (int idx = threadIdx.x; idx < items; idx += kFwThreads) {
    const int rl = idx / (16 * a.m), r = (idx / a.m) & 15, mcol = idx % a.m;
    float v = 0.f;
    for (int w = 0; w < kFwWarps; ++w) {
      const int s0 = wrange[w][0], s1 = wrange[w][1];
      if (rl < s0 || rl > s1) continue;
      v += wpart[((size_t)w * a.nseg + (rl - s0)) * 16 * a.m + r * a.m + mcol];
    }
    const int row = (rt0 + rl) * 16 + r;
    if (row >= a.rows) continue;
    v *= ldexpf(1.0f, -fw_xscale_pow(xmax[mcol]));
    if (a.S == 1) {
      a.y[(size_t)mcol * a.ldy + row] = v * (a.rscale ? a.rscale[row] : a.uscale);
    } else {
      a.part[((size_t)split * a.m + mcol) * a.rows + row] = v;
    }
  }
  if (a.S == 1) return;

  // ---- k-split: the last CTA of this row group sums the splits in order
  __shared__ unsigned last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&a.cnt[grp], 1u) == (unsigned)(a.S - 1) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // kFix outputs per thread per pass, all their split partials loaded before
  // any is added (the adds stay in split order)
  constexpr int kFix = 4;
  const int nfix = nrt * 16 * a.m;
  for (int i0 = threadIdx.x; i0 < nfix; i0 += kFwThreads * kFix) {
    int rowv[kFix], colv[kFix];
#pragma unroll
    for (int u = 0; u < kFix; ++u) {
      const int idx = i0 + u * kFwThreads;
      const int rl = idx / (16 * a.m), r = (idx / a.m) & 15;
      colv[u] = idx % a.m;
      rowv[u] = (idx < nfix && (rt0 + rl) * 16 + r < a.rows) ? (rt0 + rl) * 16 + r : -1;
    }
    float v[kFix];
#pragma unroll
    for (int u = 0; u < kFix; ++u) v[u] = 0.f;
    for (int s0 = 0; s0 < a.S; s0 += 4) {
      float pv[kFix][4];
#pragma unroll
      for (int u = 0; u < kFix; ++u)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          pv[u][q] = (rowv[u] >= 0 && s0 + q < a.S)
                         ? __ldcg(&a.part[((size_t)(s0 + q) * a.m + colv[u]) * a.rows + rowv[u]])
                         : 0.f;
#pragma unroll
      for (int u = 0; u < kFix; ++u)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (s0 + q < a.S) v[u] += pv[u][q];
    }
#pragma unroll
    for (int u = 0; u < kFix; ++u)
      if (rowv[u] >= 0)
        a.y[(size_t)colv[u] * a.ldy + rowv[u]] = v[u] * (a.rscale ? a.rscale[rowv[u]] : a.uscale);
  }
  if (threadIdx.x == 0) a.cnt[grp] = 0u;
}

// Launch plan of one fw GEMV.
struct FwPlan {
  int S, ks_tiles, G, xstride, nseg;
  size_t smem;
};

FwPlan fw_plan_budget(const FWLayout& L, int m, int num_sms, size_t xbudget) {
  FwPlan p;
  const int TK = fw_tk(L.fmt);
  const int ntk = (int)L.ntk, n_rt = (int)L.n_rt;
  // k-tiles whose staged x rows fit the budget (whole chunks of tiles)
  const int64_t kmax = (int64_t)(xbudget / ((size_t)2 * fw_xterms(m) * m)) - 16;
  int ks_cap = (int)std::max<int64_t>(kChunkTiles, kmax / TK / kChunkTiles * kChunkTiles);
  int S = (ntk + ks_cap - 1) / ks_cap;
  // few row tiles: split k further so that every SM has work
  if (n_rt * S < num_sms) {
    const int want = std::min((ntk + kChunkTiles - 1) / kChunkTiles, num_sms / std::max(1, n_rt));
    S = std::max(S, want);
  }
  S = std::max(1, S);
  int ks = (ntk + S - 1) / S;
  ks = (ks + kChunkTiles - 1) / kChunkTiles * kChunkTiles;
  S = std::max(1, (ntk + ks - 1) / ks);
  p.S = S;
  p.ks_tiles = ks;
  p.G = std::max(1, std::min(n_rt, num_sms / S));
  p.xstride = ks * TK + 16;
  // partial slots per warp: row tiles one warp's chunk range can touch
  const int nrt_max = (n_rt + p.G - 1) / p.G;
  const int cpr = (ks + kChunkTiles - 1) / kChunkTiles;
  const int C = nrt_max * cpr;
  int nseg = 1;
  for (int w = 0; w < kFwWarps; ++w) {
    const int w0 = (int)((int64_t)w * C / kFwWarps), w1 = (int)((int64_t)(w + 1) * C / kFwWarps);
    if (w1 > w0) nseg = std::max(nseg, (w1 - 1) / cpr - w0 / cpr + 1);
  }
  p.nseg = nseg;
  p.smem = fw_smem_bytes(m, p.xstride, nseg);
  return p;
}

// The x budget shrinks (more k-splits) until x and the partial slots fit.
FwPlan fw_plan(const FWLayout& L, int m, int num_sms) {
  FwPlan p = fw_plan_budget(L, m, num_sms, kFwXBudget);
  for (size_t b = kFwXBudget / 2; p.smem > kFwSmemMax && b >= 8192; b /= 2)
    p = fw_plan_budget(L, m, num_sms, b);
  return p;
}

template <int FMT, int MODE>
int fw_launch_t(const FwArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = fw_gemv_kernel<FMT, MODE>;
  static bool attr_set = false;
  if (!attr_set) {
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFwSmemMax));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kFwThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NIMF_OK;
}

template <int FMT>
int fw_launch_fmt(const FwArgs& a, int mode, dim3 grid, size_t smem, cudaStream_t st) {
  switch (mode) {
    case 1: return fw_launch_t<FMT, 1>(a, grid, smem, st);
    case 2: return fw_launch_t<FMT, 2>(a, grid, smem, st);
    default: return fw_launch_t<FMT, 3>(a, grid, smem, st);
  }
}

// k-split scratch (partials and arrival counters), per process and device;
// launches that use it must be ordered on one stream.
struct FwScratch {
  int device = -1;
  float* part = nullptr;
  size_t part_bytes = 0;
  unsigned* cnt = nullptr;
  size_t cnt_n = 0;
};
FwScratch g_fws;

int fw_scratch(size_t part_bytes, size_t cnt_n, cudaStream_t st, float** part, unsigned** cnt) {
  Context* c = ctx();
  const bool grow = g_fws.device != c->device || g_fws.part_bytes < part_bytes || g_fws.cnt_n < cnt_n;
  if (grow) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "byte-format GEMV: its k-split scratch must grow, which cannot happen "
                       "during stream capture; run the same call once before capturing");
  }
  if (g_fws.device != c->device) {
    // buffers of another device: free them with that device current
    if (g_fws.device >= 0 && (g_fws.part || g_fws.cnt)) {
      int cur = 0;
      NIMF_CUDA_TRY(cudaGetDevice(&cur));
      NIMF_CUDA_TRY(cudaSetDevice(g_fws.device));
      cudaDeviceSynchronize();
      device_free(g_fws.part);
      device_free(g_fws.cnt);
      NIMF_CUDA_TRY(cudaSetDevice(cur));
    }
    g_fws = FwScratch();
  }
  if (g_fws.part_bytes < part_bytes) {
    device_free(g_fws.part);
    g_fws.part = nullptr;
    g_fws.part_bytes = 0;
    void* p;
    NIMF_TRY(device_alloc(&p, part_bytes));
    g_fws.part = (float*)p;
    g_fws.part_bytes = part_bytes;
  }
  if (g_fws.cnt_n < cnt_n) {
    device_free(g_fws.cnt);
    g_fws.cnt = nullptr;
    g_fws.cnt_n = 0;
    void* p;
    NIMF_TRY(device_alloc(&p, cnt_n * sizeof(unsigned)));
    NIMF_CUDA_TRY(cudaMemsetAsync(p, 0, cnt_n * sizeof(unsigned), st));
    g_fws.cnt = (unsigned*)p;
    g_fws.cnt_n = cnt_n;
  }
  g_fws.device = c->device;
  *part = g_fws.part;
  *cnt = g_fws.cnt;
  return NIMF_OK;
}

}  // namespace

void fw_release_scratch() {
  device_free(g_fws.part);
  device_free(g_fws.cnt);
  g_fws = FwScratch();
}

int fw_build(FWLayout* L, int fmt, const void* raw_dev, const void* bscale_dev, const float* rscale_dev,
             float uscale, int64_t rows, int64_t k, cudaStream_t st) {
  *L = FWLayout();
  if (rows == 0 || k == 0) return NIMF_OK;
  const int TK = fw_tk(fmt);
  const int64_t n_rt = (rows + 15) / 16, ntk = (k + TK - 1) / TK;
  if (n_rt > INT32_MAX / 2 || ntk > INT32_MAX / 64) return NIMF_OK;  // generic path only
  FWLayout l;
  l.fmt = fmt;
  l.rows = rows;
  l.k = k;
  l.n_rt = n_rt;
  l.ntk = ntk;
  l.rscale = rscale_dev;
  l.uscale = uscale;
  const int64_t total = n_rt * ntk * 32;
  NIMF_TRY(device_alloc(&l.frag, (size_t)total * 16));
  if (fmt == FW_FP4) {
    int st2 = device_alloc(&l.sfrag, (size_t)(n_rt * ntk * 8) * 8);
    if (st2 != NIMF_OK) {
      device_free(l.frag);
      return st2;
    }
  }
  const unsigned blocks = (unsigned)((total + 255) / 256);
  const uint8_t* raw = (const uint8_t*)raw_dev;
  switch (fmt) {
    case FW_I8: fw_repack_kernel<FW_I8><<<blocks, 256, 0, st>>>(raw, nullptr, rows, k, ntk, total, (uint4*)l.frag, nullptr); break;
    case FW_E4M3: fw_repack_kernel<FW_E4M3><<<blocks, 256, 0, st>>>(raw, nullptr, rows, k, ntk, total, (uint4*)l.frag, nullptr); break;
    case FW_E5M2: fw_repack_kernel<FW_E5M2><<<blocks, 256, 0, st>>>(raw, nullptr, rows, k, ntk, total, (uint4*)l.frag, nullptr); break;
    default:
      fw_repack_kernel<FW_FP4><<<blocks, 256, 0, st>>>(raw, (const uint8_t*)bscale_dev, rows, k, ntk,
                                                      total, (uint4*)l.frag, (uint2*)l.sfrag);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    device_free(l.frag);
    device_free(l.sfrag);
    return set_error(NIMF_ERR_CUDA, "fw repack launch failed: %s", cudaGetErrorString(e));
  }
  *L = l;
  return NIMF_OK;
}

int fw_count_special_codes(const uint8_t* d, int64_t n, int mbits, int64_t* count, cudaStream_t st) {
  *count = 0;
  if (n == 0) return NIMF_OK;
  void* p;
  NIMF_TRY(stage_out(sizeof(unsigned), &p));
  NIMF_CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(unsigned), st));
  Context* c = ctx();
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((int64_t)c->num_sms * 8, (n + 255) / 256));
  fw_count_special<<<blocks, 256, 0, st>>>(d, n, mbits, (unsigned*)p);
  NIMF_CUDA_TRY(cudaGetLastError());
  unsigned h = 0;
  NIMF_CUDA_TRY(cudaMemcpyAsync(&h, p, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  NIMF_CUDA_TRY(cudaStreamSynchronize(st));
  *count = h;
  return NIMF_OK;
}

void fw_free(FWLayout* L) {
  device_free(L->frag);
  device_free(L->sfrag);
  *L = FWLayout();
}

int fw_dequant(const FWLayout& L, float* out, cudaStream_t st) {
  if (L.rows * L.k == 0) return NIMF_OK;
  Context* c = ctx();
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((int64_t)c->num_sms * 8, (L.rows * L.k + 255) / 256));
  const uint4* f = (const uint4*)L.frag;
  switch (L.fmt) {
    case FW_I8: fw_dequant_kernel<FW_I8><<<blocks, 256, 0, st>>>(f, nullptr, L.rscale, L.uscale, L.rows, L.k, L.ntk, out); break;
    case FW_E4M3: fw_dequant_kernel<FW_E4M3><<<blocks, 256, 0, st>>>(f, nullptr, L.rscale, L.uscale, L.rows, L.k, L.ntk, out); break;
    case FW_E5M2: fw_dequant_kernel<FW_E5M2><<<blocks, 256, 0, st>>>(f, nullptr, L.rscale, L.uscale, L.rows, L.k, L.ntk, out); break;
    default:
      fw_dequant_kernel<FW_FP4><<<blocks, 256, 0, st>>>(f, (const uint2*)L.sfrag, L.rscale, L.uscale, L.rows, L.k, L.ntk, out);
  }
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int fw_gemv(const FWLayout& L, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (m <= 0 || L.rows == 0) return NIMF_OK;
  if (L.k == 0) {
    NIMF_CUDA_TRY(cudaMemsetAsync(y, 0, (size_t)(m * L.rows) * 4, st));
    return NIMF_OK;
  }
  if (L.k > INT32_MAX || L.rows > INT32_MAX) return set_error(NIMF_ERR_UNSUPPORTED, "fw GEMV size exceeds int32");
  Context* c = ctx();
  for (int64_t m0 = 0; m0 < m; m0 += kFwMaxM) {
    const int mc = (int)std::min<int64_t>(kFwMaxM, m - m0);
    const int mode = mc <= 4 ? 1 : (mc <= 8 ? 2 : 3);
    const FwPlan p = fw_plan(L, mc, c->num_sms);
    if (p.smem > kFwSmemMax)
      return set_error(NIMF_ERR_UNSUPPORTED, "fw GEMV plan needs %zu bytes of shared memory", p.smem);
    FwArgs a = {};
    a.frag = (const uint4*)L.frag;
    a.sfrag = (const uint2*)L.sfrag;
    a.rscale = L.rscale;
    a.uscale = L.uscale;
    a.x = x + m0 * L.k;
    a.y = y + m0 * L.rows;
    a.ldx = L.k;
    a.ldy = L.rows;
    a.m = mc;
    a.rows = (int)L.rows;
    a.k = (int)L.k;
    a.n_rt = (int)L.n_rt;
    a.ntk = (int)L.ntk;
    a.S = p.S;
    a.ks_tiles = p.ks_tiles;
    a.G = p.G;
    a.xstride = p.xstride;
    a.nseg = p.nseg;
    a.vec4 = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (L.k & 3) == 0) ? 1 : 0;
    if (p.S > 1)
      NIMF_TRY(fw_scratch((size_t)p.S * mc * L.rows * 4, (size_t)p.G, st, &a.part, &a.cnt));
    const dim3 grid((unsigned)p.G, (unsigned)p.S);
    switch (L.fmt) {
      case FW_I8: NIMF_TRY(fw_launch_fmt<FW_I8>(a, mode, grid, p.smem, st)); break;
      case FW_E4M3: NIMF_TRY(fw_launch_fmt<FW_E4M3>(a, mode, grid, p.smem, st)); break;
      case FW_E5M2: NIMF_TRY(fw_launch_fmt<FW_E5M2>(a, mode, grid, p.smem, st)); break;
      default: NIMF_TRY(fw_launch_fmt<FW_FP4>(a, mode, grid, p.smem, st));
    }
  }
  return NIMF_OK;
}

}  // namespace nimf
