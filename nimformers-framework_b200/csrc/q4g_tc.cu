// q4g_tc.cu -- int4 group-quantised weights (quant.nim:131-167) times a
// prefill-sized x (more than 16 rows) on the 5th-generation tensor cores:
// tcgen05.mma kind::f16 with fp32 accumulators in tensor memory (TMEM).
//
// Per quantisation group g of a channel c (scale sc, zero point zp):
//   y[r][c] += sc * D[c][r],
//   D[c][r] = sum_{k in g} (64 + nib[c][k]) * xh[r][k] - (64 + zp) * S[r][g]
//           = sum_{k in g} (nib[c][k] - zp) * xh[r][k],
// with nib the raw nibbles, xh = fp16(x * 2^e_r) (x rounded once to fp16
// after a per-row power-of-two scale that puts the row's largest magnitude
// in [128, 256)) and S[r][g] the fp32 sum of the row's xh in the group.  The
// tensor core computes all of D: 64 + nib is exact in fp16, and the
// zero-point term is one more K=16 step whose operands split 64 + zp and S
// into two fp16 parts each (hi + lo, 22 significant bits), giving
// zh*Sh + zh*Sl + zl*Sh.  y is multiplied by 2^-e_r at the end.  The only
// approximation is x's fp16 rounding (relative 2^-11 per element).
//
// One CTA computes y[128 rows of x][128 output channels], M=128 (channels) x
// N=npad (x rows of the tile, rounded up to 16) x K=16 MMAs.  Operand A lives
// in TMEM, written by unpack warps with tcgen05.st (no generic-to-async proxy
// fence on the critical path); operand B comes from shared memory in the
// canonical K-major layout.  Per group the accumulators go to one of two
// TMEM buffers and the epilogue warps add sc * D while the tensor core fills
// the other one.  The MMA and producer warps stay converged and issue from
// one elected lane.
//
// Warps: 0 producer (bulk copy of the prepared x tile, tensor-map load of the
// packed weights), 1 TMEM owner and MMA issuer, 2-9 unpack in two sets of 4
// taking alternate groups (thread = output channel = TMEM lane), 10-17
// epilogue (warp w reads TMEM lanes 32 (w % 4) .. + 31 = output channels,
// for x rows 64 ((w - 10) / 4) .. + 63).
// Every wait is bounded; on expiry the kernel records an error, lets the
// other roles run out and still frees its TMEM.
#include <algorithm>

#include "tc_util.cuh"

namespace nimf {

namespace {

constexpr int kTcRows = 128;      // x rows per CTA tile
constexpr int kTcChan = 128;      // output channels per CTA tile (8 row tiles)
constexpr int kTcUnpWarps = 8;    // two sets of 4 (TMEM lane quarters), alternate groups
constexpr int kTcEpiWarps = 8;    // 4 TMEM lane quarters x 2 row halves
constexpr int kTcEpi0 = 2 + kTcUnpWarps;   // first epilogue warp
constexpr int kTcThreads = (kTcEpi0 + kTcEpiWarps) * 32;
#ifndef NIMF_TC_ROTATE
#define NIMF_TC_ROTATE 1
#endif
#ifndef NIMF_TC_WAIT
#define NIMF_TC_WAIT 0
#endif
// wait style of every role (mbar_wait_t)
constexpr int kTcWait = NIMF_TC_WAIT;
// x tile preparation.  Each prepared tile (mt, g) holds kTcRows rows of
// RB = 2 gs + 32 bytes of K-major fp16 in the canonical layout:
//   gs values fp16(x * scale[row]) in the MMA's K order (within every aligned
//   4 k the positions hold k offsets 0, 2, 1, 3: the order in which the
//   unpack warps pair a fragment word's nibbles), then the zero-point step
//   [Sh, Sl, Sh, 0 x 13] with S the fp32 sum of the row's fp16 values,
//   Sh = fp16(S), Sl = fp16(S - Sh).
// Rows past m and k past K are zero.  Thread = (row, 8 consecutive k); the
// gs / 8 threads of a row are consecutive lanes.  Block = 256 threads =
// 2048 / gs rows of one tile and group; grid = (tiles x kTcRows / rows per
// block, groups).
__global__ void __launch_bounds__(256) q4g_tc_prep_x(const float* __restrict__ x, int64_t ldx,
                                                     int m, int k, int gs,
                                                     const float* __restrict__ scale,
                                                     unsigned char* __restrict__ out) {
  const int cg = gs >> 3;                       // threads per row (8 or 16)
  const int rpb = 256 / cg;                     // rows per block
  const int g = blockIdx.y, groups = gridDim.y;
  const int grow = blockIdx.x * rpb + (int)threadIdx.x / cg;  // row over all tiles
  const int c8 = (int)threadIdx.x % cg;
  const int mt = grow / kTcRows, r = grow % kTcRows;
  const int rb = 2 * gs + 32;
  unsigned char* base = out + ((size_t)mt * groups + g) * kTcRows * rb;
  griddep_wait();  // scale comes from the previous kernel
  const bool rv = grow < m;
  const float sf = rv ? __ldg(scale + grow) : 0.f;
  const int c = c8 * 8;
  const float* xr = x + (size_t)(rv ? grow : 0) * ldx + (size_t)g * gs + c;
  const int kvalid = rv ? max(0, min(8, k - g * gs - c)) : 0;
  float v[8];
  if (kvalid == 8 && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0)) {
    const float4 p = __ldg(reinterpret_cast<const float4*>(xr));
    const float4 q = __ldg(reinterpret_cast<const float4*>(xr + 4));
    v[0] = p.x; v[1] = p.z; v[2] = p.y; v[3] = p.w;
    v[4] = q.x; v[5] = q.z; v[6] = q.y; v[7] = q.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = (j & 4) + ((j & 1) << 1) + ((j >> 1) & 1);  // 0,2,1,3 within 4
      v[j] = i < kvalid ? __ldg(xr + i) : 0.f;
    }
  }
  uint32_t h[4];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 p = __floats2half2_rn(v[2 * j] * sf, v[2 * j + 1] * sf);
    const float2 q = __half22float2(p);
    sum += q.x + q.y;
    h[j] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(base + canon_off(r, 2 * c, rb)) = make_uint4(h[0], h[1], h[2], h[3]);
  for (int o = cg >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (c8 == 0) {
    const __half sh = __float2half_rn(sum);
    const __half sl = __float2half_rn(sum - __half2float(sh));
    const uint32_t hs = __half_as_ushort(sh), ls = __half_as_ushort(sl);
    *reinterpret_cast<uint4*>(base + canon_off(r, 2 * gs, rb)) = make_uint4(hs | (ls << 16), hs, 0u, 0u);
    *reinterpret_cast<uint4*>(base + canon_off(r, 2 * gs + 16, rb)) = make_uint4(0u, 0u, 0u, 0u);
  }
  griddep_launch_dependents();
}

// One launch covers up to kTcMaxW weights that share x (a grouped call):
// channel tile blockIdx.y belongs to weight i for nt0[i] <= blockIdx.y < nt0[i+1].
constexpr int kTcMaxW = 4;
struct TcW {
  const float4* sz;      // scale/zero pairs, row tile 0
  float* y;              // [m][ldy]
  int64_t ldy;
  int rows, n_rt;
};
struct TcArgs {
  TcW w[kTcMaxW];
  int nt0[kTcMaxW];
  int nw;
  const unsigned char* xp;  // prepared x, [mt][g]
  const float* xinv;     // per-row 2^-e of x's scale
  int m, groups;
  int* err;
};
// the weights' fragments as 2-D tensors of 4-byte elements, one row per row
// tile (kq_total * 128 elements); box = 8 row tiles x one group
struct TcMaps {
  CUtensorMap m[kTcMaxW];
};

// Shared memory (offsets from the 1024-aligned base) and TMEM columns
template <int KQG>
struct TcLayout {
  static constexpr int GS = 64 * KQG;
  static constexpr int RB = 2 * GS + 32;                             // bytes per x row
  static constexpr int XB = kTcRows * RB;                            // one prepared x tile
  static constexpr int WBYTES = 8 * KQG * 512;                       // packed weights
  static constexpr int STAGES = KQG == 1 ? 8 : 4;
  static constexpr int XOFF = 1024;                                  // after the barriers
  static constexpr int WOFF = XOFF + STAGES * XB;
  static constexpr int TOTAL = WOFF + STAGES * WBYTES;
  static constexpr int KSTEPS = GS / 16 + 1;                         // + zero-point step
  // TMEM: accumulators [0, 2 kTcRows) (two buffers), then ABUF unpacked
  // weight tiles of AW columns (2 fp16 of K per column; the last 8 hold the
  // zero-point step)
  static constexpr uint32_t ACOL = 2 * kTcRows;
  static constexpr uint32_t AW = GS / 2 + 8;
  static constexpr int ABUF = (int)((kTmemCols - ACOL) / AW) < 4 ? (int)((kTmemCols - ACOL) / AW) : 4;
  static_assert(ABUF >= 2, "TMEM columns");
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

template <int KQG>
__global__ void __launch_bounds__(kTcThreads, 1)
    q4g_tc_kernel(const TcArgs a, const __grid_constant__ TcMaps maps) {
  using L = TcLayout<KQG>;
  constexpr int GS = L::GS;
  constexpr int NS = L::STAGES, NA = L::ABUF;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw;
  uint64_t* sfull = reinterpret_cast<uint64_t*>(smem);    // producer -> MMA, unpack
  uint64_t* sempty = sfull + NS;                           // MMA + 4 unpack warps -> producer
  uint64_t* afull = sempty + NS;                           // [NA] unpack -> MMA
  uint64_t* aempty = afull + NA;                           // [NA] MMA -> unpack
  uint64_t* tfull = aempty + NA;                           // [2] MMA -> epilogue
  uint64_t* tempty = tfull + 2;                            // [2] epilogue -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockIdx.x = x tile (fastest, so the CTAs reading one weight tile run
  // together and it comes from DRAM once), blockIdx.y = channel tile
  int wsel = 0;
  for (int i = 1; i < a.nw; ++i)
    if ((int)blockIdx.y >= a.nt0[i]) wsel = i;
  const TcW W = a.w[wsel];
  const CUtensorMap* wmap = &maps.m[wsel];
  const int nt = (int)blockIdx.y - a.nt0[wsel], mt = blockIdx.x;
  const int G = a.groups;
  const int rt0 = nt * 8;
  const int nrt = max(0, min(8, W.n_rt - rt0));
  // x rows of this tile, rounded up to the MMA's N granule
  const int nrows = min(kTcRows, a.m - mt * kTcRows);
  const int npad = (nrows + 15) & ~15;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], 1 + 4);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&afull[b], 4);
      mbar_init(&aempty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kTcEpiWarps);
    }
    *failed = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    if (a.err) atomicExch(a.err, code);
    *reinterpret_cast<volatile int*>(failed) = 1;
  };
  auto stop = [&]() { return *reinterpret_cast<volatile int*>(failed) != 0; };

  if (warp == 0) {
    // ---------------- producer: per group, the x tile's npad rows and the 8
    // row tiles' packed nibbles (one tensor-map box; rows past the weight
    // read 0)
    const uint32_t xbytes = (uint32_t)npad * L::RB;
    int last = -1;
    for (int g = 0; g < G; ++g) {
      const int s = g % NS;
      // lane 0 decides for the warp, so its lanes leave the loop together
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && (g < NS || mbar_wait_t<kTcWait>(&sempty[s], ((g / NS) - 1) & 1))) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0 && !stop()) fail(3);
        break;
      }
      unsigned char* xs = smem + L::XOFF + s * L::XB;
      unsigned char* ws = smem + L::WOFF + s * L::WBYTES;
      const unsigned char* src = a.xp + ((size_t)mt * G + g) * L::XB;
      if (g == 0) griddep_wait();  // the prepared x comes from the previous kernel
      if (elect_one()) {
        mbar_arrive_expect_tx(&sfull[s], xbytes + L::WBYTES);
        bulk_g2s(xs, src, xbytes, &sfull[s]);
        tma_load_2d(ws, wmap, g * KQG * 128, rt0, &sfull[s]);
      }
      __syncwarp();
      last = g;
    }
    // the last copies land before the CTA may exit
    if (lane == 0 && last >= 0) {
      for (int g = max(0, last - NS + 1); g <= last; ++g)
        if (!mbar_wait_t<kTcWait>(&sfull[g % NS], (g / NS) & 1)) fail(3);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the converged warp computes the operands,
    // one elected lane issues
    const uint32_t idesc = idesc_n(npad);
    const uint64_t bdesc0 = smem_desc(smem + L::XOFF, 128, L::RB * 8);
    for (int g = 0; g < G; ++g) {
      const int s = g % NS, b = g & 1, ab = g % NA;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kTcWait>(&sfull[s], (g / NS) & 1) &&
              mbar_wait_t<kTcWait>(&afull[ab], (g / NA) & 1) &&
              (g < 2 || mbar_wait_t<kTcWait>(&tempty[b], ((g >> 1) - 1) & 1)))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(4);
        break;
      }
      tc_fence_after();
      // descriptor start address in 16-byte units: stage offset, 256 B per k step
      const uint64_t bd = bdesc0 + (uint64_t)((s * L::XB) >> 4);
      const uint32_t td = tmem + (uint32_t)b * kTcRows;
      const uint32_t ta = tmem + L::ACOL + (uint32_t)ab * L::AW;
#pragma unroll
      for (int kk = 0; kk < L::KSTEPS; ++kk)
        if (elect_one()) umma_f16_ts(td, ta + (uint32_t)kk * 8u, bd + (uint64_t)(kk * 16), idesc, kk > 0 ? 1u : 0u);
      if (elect_one()) {
        umma_commit(&aempty[ab]);
        umma_commit(&tfull[b]);
        umma_commit(&sempty[s]);
      }
      __syncwarp();
    }
  } else if (warp < kTcEpi0) {
    // ---------------- unpack: packed nibbles (fragment order) -> fp16 rows of
    // A in TMEM.  Thread = output channel r (TMEM lane; a warp owns lanes
    // 32 (warp % 4) .. + 31); rows g8 and g8 + 8 of a row tile share a
    // fragment word (low / high nibble of each byte).  Word wi of fragment
    // lane (g8, t) of quad qq holds k = qq*64 + 16 wi + 4 t + b, b = 0..3;
    // its column pair (qq*32 + wi*8 + 2t, + 1) holds k offsets (0, 2), (1, 3).
    // A nibble n moved to fp16 mantissa bits 4..7 under exponent 2^6 reads
    // 64 + n.
    const int r = (warp & 3) * 32 + lane;
    const int uset = (warp - 2) >> 2;
    const int rl = r >> 4, g8 = r & 7, rot = NIMF_TC_ROTATE ? (g8 >> 1) : 0;
    const bool hi = (r & 8) != 0;
    const int sh0 = hi ? 0 : 4, sh1 = hi ? 8 : 4;  // bytes 0, 2: left; bytes 1, 3: right
    const int rt = min(rt0 + rl, W.n_rt - 1);
    const float4* szp = W.sz + (size_t)rt * a.groups * 8 + g8;
    float4 zn = uset < G ? __ldg(szp + (size_t)uset * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g = uset; g < G; g += 2) {
      const int s = g % NS, ab = g % NA;
      const float4 zz = zn;
      if (g + 2 < G) zn = __ldg(szp + (size_t)(g + 2) * 8);
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kTcWait>(&sfull[s], (g / NS) & 1) &&
              (g < NA || mbar_wait_t<kTcWait>(&aempty[ab], ((g / NA) - 1) & 1)))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(5);
        break;
      }
      tc_fence_after();
      const uint4* wsrc = reinterpret_cast<const uint4*>(smem + L::WOFF + s * L::WBYTES);
      const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + L::ACOL + (uint32_t)ab * L::AW;
#pragma unroll
      for (int qq = 0; qq < KQG; ++qq) {
        // load j reads fragment lane (g8, (j + rot) & 3): the 8 g8 of a warp
        // then hit 8 different 16-byte bank groups
        uint4 u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          u[j] = make_uint4(0u, 0u, 0u, 0u);
          if (rl < nrt) u[j] = wsrc[(rl * KQG + qq) * 32 + g8 * 4 + ((j + rot) & 3)];
        }
        // back to fragment order, u[t] <- u[(t - rot) & 3], with selects
        // (per-lane branches here stall the warps on branch resolution)
        if (NIMF_TC_ROTATE) {
          const bool r1 = (rot & 1) != 0, r2 = (rot & 2) != 0;
          auto sel = [](bool c, const uint4& x, const uint4& y) {
            return make_uint4(c ? x.x : y.x, c ? x.y : y.y, c ? x.z : y.z, c ? x.w : y.w);
          };
          const uint4 v0 = sel(r1, u[3], u[0]), v1 = sel(r1, u[0], u[1]);
          const uint4 v2 = sel(r1, u[1], u[2]), v3 = sel(r1, u[2], u[3]);
          u[0] = sel(r2, v2, v0);
          u[1] = sel(r2, v3, v1);
          u[2] = sel(r2, v0, v2);
          u[3] = sel(r2, v1, v3);
        }
        uint32_t col[32];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t wv[4] = {u[t].x, u[t].y, u[t].z, u[t].w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            col[wi * 8 + 2 * t] = ((wv[wi] << sh0) & 0x00F000F0u) | 0x54005400u;
            col[wi * 8 + 2 * t + 1] = ((wv[wi] >> sh1) & 0x00F000F0u) | 0x54005400u;
          }
        }
        tmem_st32(ta + (uint32_t)qq * 32u, col);
      }
      {
        // zero-point step: (-zh, -zh), (-zl, 0) against (Sh, Sl), (Sh, 0)
        const float z = (hi ? zz.w : zz.y) + 64.0f;
        const __half zh = __float2half_rn(z);
        const __half zl = __float2half_rn(z - __half2float(zh));
        const uint32_t nzh = (uint32_t)__half_as_ushort(zh) ^ 0x8000u;
        const uint32_t nzl = (uint32_t)__half_as_ushort(zl) ^ 0x8000u;
        const uint32_t zc[8] = {nzh | (nzh << 16), nzl, 0u, 0u, 0u, 0u, 0u, 0u};
        tmem_st8(ta + (uint32_t)(GS / 2), zc);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[ab]);
        mbar_arrive(&sempty[s]);
      }
    }
  } else {
    // ---------------- epilogue: thread = output channel (TMEM lane), 64 x rows
    const int quad = warp & 3, rh = (warp - kTcEpi0) >> 2;
    const int ch = quad * 32 + lane;              // channel within the tile
    const int rt = rt0 + (ch >> 4), r16 = ch & 15;
    const bool cvalid = rt < W.n_rt && rt * 16 + r16 < W.rows;
    const bool act0 = rh * 64 < npad, act1 = rh * 64 + 32 < npad;  // warp-uniform
    const float4* szp = W.sz + ((size_t)min(rt, W.n_rt - 1) * a.groups) * 8 + (r16 & 7);
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    griddep_wait();
    // scales one group ahead (their global load off the critical path)
    float4 zn = G > 0 ? __ldg(szp) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g = 0; g < G; ++g) {
      const int b = g & 1;
      const float4 zz = zn;
      if (g + 1 < G) zn = __ldg(szp + (size_t)(g + 1) * 8);
      const float sc = (r16 >> 3) ? zz.z : zz.x;
      int ok = 1;
      if (lane == 0) ok = (!stop() && mbar_wait_t<kTcWait>(&tfull[b], (g >> 1) & 1)) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(6);
        break;
      }
      tc_fence_after();
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)b * kTcRows + rh * 64;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 0 ? act0 : act1) {
          uint32_t d0[16], d1[16];
          tmem_ld16(tl + h * 32, d0);
          tmem_ld16(tl + h * 32 + 16u, d1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            acc[h * 32 + i] = fmaf(sc, __uint_as_float(d0[i]), acc[h * 32 + i]);
            acc[h * 32 + 16 + i] = fmaf(sc, __uint_as_float(d1[i]), acc[h * 32 + 16 + i]);
          }
        }
      }
      // the buffer may be refilled
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (cvalid && act0 && !stop()) {
      const int n = rt * 16 + r16;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int row = mt * kTcRows + rh * 64 + i;
        if (row < a.m) W.y[(size_t)row * W.ldy + n] = acc[i] * __ldg(a.xinv + row);
      }
    }
  }
  // every role is done; outstanding MMAs finished before the last tfull
  // phase, which the epilogue waited for (or the kernel failed, in which case
  // the MMA warp waits here for its own last commit)
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && stop() && G > 0) mbar_wait_t<kTcWait>(&tfull[(G - 1) & 1], ((G - 1) >> 1) & 1);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int weight_tensor_map(const Q4GWeight& w, int kqg, CUtensorMap* tm) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(NIMF_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)w.kq_total * 128, (cuuint64_t)w.n_rt};
  const cuuint64_t strides[1] = {(cuuint64_t)w.kq_total * 512};
  const cuuint32_t box[2] = {(cuuint32_t)kqg * 128, 8};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, w.frag, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(NIMF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NIMF_OK;
}

template <int KQG>
int launch_tc(const Q4GWeight* const* ws, int count, const float* x, int m, float* const* ys,
              cudaStream_t st) {
  using L = TcLayout<KQG>;
  Context* c = ctx();
  const Q4GWeight& w0 = *ws[0];
  const int G = (int)w0.groups;
  const int64_t ldx = w0.k;
  const int mts = (m + kTcRows - 1) / kTcRows;
  if (G > 65535) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: %d groups (max 65535)", G);
  // scratch: the prepared tiles, then scale[m] and inv[m]
  const size_t tiles = ((size_t)mts * G * L::XB + 255) & ~(size_t)255;
  const size_t mpad = (size_t)mts * kTcRows;
  unsigned char* xp = nullptr;
  NIMF_TRY(tc_prep_buffer(tiles + 2 * mpad * sizeof(float), st, &xp));
  float* scale = reinterpret_cast<float*>(xp + tiles);
  float* inv = scale + mpad;
  static int attr_dev = -1;
  auto kern = q4g_tc_kernel<KQG>;
  if (c && attr_dev != c->device) {
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr_dev = c->device;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)m, 1, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, tc_rowscale, x, ldx, m, (int)w0.k, scale, inv));
  }
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(mpad * L::GS / 2048), (unsigned)G, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4g_tc_prep_x, x, ldx, m, (int)w0.k, L::GS,
                                     (const float*)scale, xp));
  }
  // one launch per kTcMaxW weights, all reading the same prepared x
  for (int i0 = 0; i0 < count; i0 += kTcMaxW) {
    TcArgs a = {};
    TcMaps maps;
    int nts = 0;
    a.nw = 0;
    for (int i = i0; i < count && i < i0 + kTcMaxW; ++i) {
      const Q4GWeight& w = *ws[i];
      TcW& t = a.w[a.nw];
      t.sz = (const float4*)w.sz;
      t.y = ys[i];
      t.ldy = w.rows;
      t.rows = (int)w.rows;
      t.n_rt = (int)w.n_rt;
      a.nt0[a.nw] = nts;
      NIMF_TRY(weight_tensor_map(w, KQG, &maps.m[a.nw]));
      nts += (int)((w.rows + kTcChan - 1) / kTcChan);
      ++a.nw;
    }
    if (nts > 65535)
      return set_error(NIMF_ERR_SHAPE, "prefill GEMM: %d channel tiles in one launch (max 65535)", nts);
    for (int i = a.nw; i < kTcMaxW; ++i) a.nt0[i] = nts;
    a.xp = xp;
    a.xinv = inv;
    a.m = m;
    a.groups = G;
    a.err = c ? c->dev_err : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)mts, (unsigned)nts, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, maps));
  }
  return NIMF_OK;
}

}  // namespace

// x-preparation scratch, one buffer per device, grown outside stream capture
struct PrepBuf {
  int device = -1;
  void* p = nullptr;
  size_t bytes = 0;
};
constexpr int kPrepDevices = 64;
PrepBuf g_prep[kPrepDevices];

void release_prep_buffers() {
  int cur = -1;
  cudaGetDevice(&cur);
  for (PrepBuf& b : g_prep) {
    if (b.p) {
      cudaSetDevice(b.device);
      cudaDeviceSynchronize();
      device_free(b.p);
    }
    b = PrepBuf();
  }
  if (cur >= 0) cudaSetDevice(cur);
}

int tc_prep_buffer(size_t bytes, cudaStream_t st, unsigned char** out) {
  Context* c = ctx();
  const int dev = c ? c->device : 0;
  if (dev < 0 || dev >= kPrepDevices)
    return set_error(NIMF_ERR_STATE, "prefill GEMM: device index %d", dev);
  PrepBuf& b = g_prep[dev];
  if (b.device != dev || b.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "prefill GEMM: its x scratch must grow, which cannot happen during "
                       "stream capture; run the same call once before capturing");
    NIMF_CUDA_TRY(cudaDeviceSynchronize());
    if (b.device == dev) device_free(b.p);
    b.p = nullptr;
    NIMF_TRY(device_alloc(&b.p, bytes));
    b.device = dev;
    b.bytes = bytes;
  }
  *out = (unsigned char*)b.p;
  return NIMF_OK;
}

// Group sizes 64 and 128 (256 would need more shared memory than a CTA has),
// zero points within the fp16 split (others use the CUDA-core path).
bool q4g_tc_supported(const Q4GWeight& w) {
  return w.fast && w.tc_zp_ok && (w.gs == 64 || w.gs == 128) && w.rows > 0 && w.k > 0;
}

// ws[0..count) share x (same K and group size, all q4g_tc_supported, rows > 0)
int q4g_gemm_tc_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                      float* const* ys, cudaStream_t st) {
  if (m <= 0 || count <= 0) return NIMF_OK;
  if (m > 0x7fffffff / 2) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: M = %lld", (long long)m);
  for (int i = 1; i < count; ++i)
    if (ws[i]->gs != ws[0]->gs || ws[i]->k != ws[0]->k)
      return set_error(NIMF_ERR_SHAPE, "prefill GEMM: grouped weights differ in K or group size");
  switch (ws[0]->gs) {
    case 64: return launch_tc<1>(ws, count, x, (int)m, ys, st);
    case 128: return launch_tc<2>(ws, count, x, (int)m, ys, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "prefill GEMM: group size %lld", (long long)ws[0]->gs);
}

int q4g_gemm_tc(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (w.rows <= 0) return NIMF_OK;
  const Q4GWeight* ws[1] = {&w};
  float* ys[1] = {y};
  return q4g_gemm_tc_group(ws, 1, x, m, ys, st);
}

}  // namespace nimf
