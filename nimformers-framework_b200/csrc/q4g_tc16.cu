// q4g_tc16.cu -- int4 group-quantised weights (quant.nim:131-167) times a
// prefill-sized x on the 5th-generation tensor cores, with the weights
// dequantised into fp16 tiles so that one TMEM accumulator runs over the
// whole of K (no per-group epilogue).
//
// Per output channel c and quantisation group g (scale sc, zero point zp),
// the unpack warps turn every nibble n into the fp16 value
//   a[c][k] = fp16(fma(n, sc 2^e, -zp sc 2^e))   ~ (n - zp) sc 2^e
// (quant.nim's dequantisation, rounded once more to fp16; 2^e is a per-weight
// power of two chosen at registration that puts the largest magnitude in
// [2^13, 2^14)) and write them straight into TMEM as operand A; x is rounded
// once to fp16 after a per-row power-of-two scale (xh = fp16(x 2^e_r)).  The
// tensor core accumulates D[c][r] = sum_k a[c][k] xh[r][k] in fp32 over all
// of K, and the epilogue writes y[r][c] = D[c][r] 2^-e 2^-e_r once.  The two
// fp16 roundings give about 3e-4 of max|y| at K = 4096 (simulated against
// float64), under the 1e-3 bar; bf16 tiles would give 2.4e-3.
//
// Compared with the exact-nibble GEMM (q4g_tc.cu), whose fp32 epilogue
// applies each group's scale to a fresh accumulator, the per-group chain is
// gone and an x tile of NR = 256 rows feeds each weight tile: per 128 x 256 x
// 128 block the tensor core works 1,024 cycles against about 512 issue slots
// of unpack per sub-partition.
//
// One CTA computes y[NR rows of x][128 output channels]: per group, one
// bulk copy of the prepared x tile and one tensor-map load of the 8 row
// tiles' packed nibbles into a ring stage, GS/16 MMAs of M=128 x N=npad x
// K=16 (kind::f16, A from TMEM, B from shared memory, K-major canonical).
// Warps: 0 producer, 1 TMEM owner and MMA issuer, 2-9 unpack (two sets of 4
// taking alternate groups; thread = output channel = TMEM lane), 10-17
// epilogue (warp w: TMEM lanes 32 (w % 4) .., x rows NR/2 ((w - 10) / 4) ..).
// Every wait is bounded; on expiry the kernel records an error, lets the
// other roles run out and still frees its TMEM after its last commit.
#include <algorithm>

#include "tc_util.cuh"

namespace nimf {

namespace {

constexpr int kT6Chan = 128;                    // output channels per CTA tile (8 row tiles)
constexpr int kT6UnpWarps = 8;
constexpr int kT6EpiWarps = 8;
constexpr int kT6Epi0 = 2 + kT6UnpWarps;
constexpr int kT6Threads = (kT6Epi0 + kT6EpiWarps) * 32;
constexpr int kT6Wait = 0;                      // mbar_wait_t style of every role
constexpr int kT6MaxW = 4;                      // weights per (grouped) launch

template <int KQG, int NR>
struct T6Layout {
  static constexpr int GS = 64 * KQG;
  static constexpr int RB = 2 * GS;                    // bytes per prepared x row (one group)
  static constexpr int XB = NR * RB;                   // one prepared x tile
  static constexpr int WBYTES = 8 * KQG * 512;         // packed weights of 8 row tiles
  // two rings: the weights (small; the unpack warps run ahead on them) and
  // the x tiles (large; the MMA's B operand)
  static constexpr int NSW = 4;
  static constexpr int FIT = (227 * 1024 - 1024 - NSW * WBYTES) / XB;
  static constexpr int NSX = FIT < 8 ? FIT : 8;
  static constexpr int XOFF = 1024;
  static constexpr int WOFF = XOFF + NSX * XB;
  static constexpr int TOTAL = WOFF + NSW * WBYTES;
  static constexpr int KSTEPS = GS / 16;
  static constexpr uint32_t ACOL = NR;                 // accumulator columns
  static constexpr uint32_t AW = GS / 2;               // columns of one A tile
  static constexpr int ABUF = (int)((kTmemCols - ACOL) / AW) < 4 ? (int)((kTmemCols - ACOL) / AW) : 4;
  static_assert(NSX >= 2, "shared memory");
  static_assert(ABUF >= 2, "TMEM columns");
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

// x tile preparation: tile (mt, g) holds NR rows of GS fp16 values
// fp16(x * scale[row]) in the canonical K-major layout, within every aligned
// 4 k in the order 0, 2, 1, 3 (the order in which the unpack warps pair a
// fragment word's bytes).  Rows past m and k past K are zero.  Thread = (row,
// 8 consecutive k); block = 256 threads = 2048 / GS rows of one tile and
// group; grid = (tiles * NR / rows per block, groups).
__global__ void __launch_bounds__(256) q4g_tc16_prep_x(const float* __restrict__ x, int64_t ldx,
                                                       int m, int k, int gs, int nr,
                                                       const float* __restrict__ scale,
                                                       unsigned char* __restrict__ out) {
  const int cg = gs >> 3;
  const int rpb = 256 / cg;
  const int g = blockIdx.y, groups = gridDim.y;
  const int grow = blockIdx.x * rpb + (int)threadIdx.x / cg;
  const int c8 = (int)threadIdx.x % cg;
  const int mt = grow / nr, r = grow % nr;
  const int rb = 2 * gs;
  unsigned char* base = out + ((size_t)mt * groups + g) * (size_t)nr * rb;
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
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 p = __floats2half2_rn(v[2 * j] * sf, v[2 * j + 1] * sf);
    h[j] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(base + canon_off(r, 2 * c, rb)) = make_uint4(h[0], h[1], h[2], h[3]);
  griddep_launch_dependents();
}

struct T6W {
  const float4* sz;      // scale/zero pairs, row tile 0
  float* y;              // [m][ldy]
  int64_t ldy;
  int rows, n_rt;
  float wscale;          // 2^e of the weight's fp16 tiles
  float winv;            // 2^-e
};
struct T6Args {
  T6W w[kT6MaxW];
  int nt0[kT6MaxW];
  int nw;
  const unsigned char* xp;  // prepared x, [mt][g]
  const float* xinv;        // per-row 2^-e_r of x's scale
  int m, groups;
  int* err;
};
struct T6Maps {
  CUtensorMap m[kT6MaxW];
};

// Two nibbles of m (bits 0..3 of bytes b0 and b1) -> the fp16 pair
// {lo: fp16(fma(n0, sc, nzs)), hi: fp16(fma(n1, sc, nzs))}: byte permutes make
// the floats 2^23 + n, one packed subtraction gives n exactly, one packed fma
// the dequantised values, one conversion packs them (5 instructions a pair).
__device__ __forceinline__ uint32_t nib2_h2(uint32_t m, uint32_t sel0, uint32_t sel1,
                                            unsigned long long sc2, unsigned long long nzs2) {
  const uint32_t f0 = __byte_perm(m, 0x4B000000u, sel0);
  const uint32_t f1 = __byte_perm(m, 0x4B000000u, sel1);
  unsigned long long v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(f0), "r"(f1));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(0xCB000000CB000000ull));   // - 2^23 each
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(v) : "l"(sc2), "l"(nzs2));
  uint32_t lo, hi, h;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "r"(hi), "r"(lo));
  return h;
}
__device__ __forceinline__ unsigned long long f32x2_splat(float v) {
  const uint32_t b = __float_as_uint(v);
  return ((unsigned long long)b << 32) | b;
}
__device__ __forceinline__ uint4 sel4(bool c, const uint4& a, const uint4& b) {
  return make_uint4(c ? a.x : b.x, c ? a.y : b.y, c ? a.z : b.z, c ? a.w : b.w);
}

template <int KQG, int NR>
__global__ void __launch_bounds__(kT6Threads, 1)
    q4g_tc16_kernel(const T6Args a, const __grid_constant__ T6Maps maps) {
  using L = T6Layout<KQG, NR>;
  constexpr int NSX = L::NSX, NSW = L::NSW, NA = L::ABUF;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem);    // producer -> MMA (x tile)
  uint64_t* xempty = xfull + NSX;                          // MMA -> producer
  uint64_t* wfull = xempty + NSX;                          // producer -> unpack (weights)
  uint64_t* wempty = wfull + NSW;                          // 4 unpack warps -> producer
  uint64_t* afull = wempty + NSW;                          // [NA] unpack -> MMA
  uint64_t* aempty = afull + NA;                           // [NA] MMA -> unpack
  uint64_t* tfull = aempty + NA;                           // MMA -> epilogue (once)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int wsel = 0;
  for (int i = 1; i < a.nw; ++i)
    if ((int)blockIdx.y >= a.nt0[i]) wsel = i;
  const T6W W = a.w[wsel];
  const CUtensorMap* wmap = &maps.m[wsel];
  const int nt = (int)blockIdx.y - a.nt0[wsel], mt = blockIdx.x;
  const int G = a.groups;
  const int rt0 = nt * 8;
  const int nrt = max(0, min(8, W.n_rt - rt0));
  const int nrows = min(NR, a.m - mt * NR);
  const int npad = (nrows + 15) & ~15;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < NSW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 4);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&afull[b], 4);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(tfull, 1);
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
    // ---------------- producer: the weights of up to NSW groups ahead of the
    // x tile in flight (weights do not depend on the previous kernel, so the
    // first ones go out before griddep_wait)
    const uint32_t xbytes = (uint32_t)npad * L::RB;
    int xlast = -1, wnext = 0;
    bool bad = false;
    for (int g = 0; g < G && !bad; ++g) {
      while (wnext < G && wnext < g + NSW) {
        const int sw = wnext % NSW;
        int ok = 1;
        if (lane == 0)
          ok = (!stop() && (wnext < NSW || mbar_wait_t<kT6Wait>(&wempty[sw], ((wnext / NSW) - 1) & 1))) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          bad = true;
          break;
        }
        if (elect_one()) {
          mbar_arrive_expect_tx(&wfull[sw], L::WBYTES);
          tma_load_2d(smem + L::WOFF + sw * L::WBYTES, wmap, wnext * KQG * 128, rt0, &wfull[sw]);
        }
        __syncwarp();
        ++wnext;
      }
      if (bad) break;
      const int s = g % NSX;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && (g < NSX || mbar_wait_t<kT6Wait>(&xempty[s], ((g / NSX) - 1) & 1))) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        bad = true;
        break;
      }
      const unsigned char* src = a.xp + ((size_t)mt * G + g) * L::XB;
      if (g == 0) griddep_wait();  // the prepared x comes from the previous kernel
      if (elect_one()) {
        mbar_arrive_expect_tx(&xfull[s], xbytes);
        bulk_g2s(smem + L::XOFF + s * L::XB, src, xbytes, &xfull[s]);
      }
      __syncwarp();
      xlast = g;
    }
    if (bad && lane == 0 && !stop()) fail(3);
    // the last copies land before the CTA may exit
    if (lane == 0) {
      for (int g = max(0, xlast - NSX + 1); g <= xlast; ++g)
        if (!mbar_wait_t<kT6Wait>(&xfull[g % NSX], (g / NSX) & 1)) fail(3);
      for (int g = max(0, wnext - NSW); g < wnext; ++g)
        if (!mbar_wait_t<kT6Wait>(&wfull[g % NSW], (g / NSW) & 1)) fail(3);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one accumulator over all groups
    const uint32_t idesc = idesc_n(npad);
    const uint64_t bdesc0 = smem_desc(smem + L::XOFF, 128, L::RB * 8);
    int issued = 0;
    for (int g = 0; g < G; ++g) {
      const int s = g % NSX, ab = g % NA;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kT6Wait>(&xfull[s], (g / NSX) & 1) &&
              mbar_wait_t<kT6Wait>(&afull[ab], (g / NA) & 1))
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
      const uint32_t ta = tmem + L::ACOL + (uint32_t)ab * L::AW;
#pragma unroll
      for (int kk = 0; kk < L::KSTEPS; ++kk)
        if (elect_one())
          umma_f16_ts(tmem, ta + (uint32_t)kk * 8u, bd + (uint64_t)(kk * 16), idesc,
                      (g > 0 || kk > 0) ? 1u : 0u);
      if (elect_one()) {
        umma_commit(&aempty[ab]);
        umma_commit(&xempty[s]);
      }
      __syncwarp();
      issued = g + 1;
    }
    if (elect_one()) umma_commit(tfull);   // every MMA issued so far is done -> epilogue
    __syncwarp();
    (void)issued;
  } else if (warp < kT6Epi0) {
    // ---------------- unpack: packed nibbles (fragment order) -> fp16 rows of
    // A in TMEM.  Thread = output channel r (TMEM lane); rows g8 and g8 + 8
    // of a row tile share a fragment word (low / high nibble of each byte).
    // Word wi of fragment lane (g8, t) of quad qq holds k = qq*64 + 16 wi +
    // 4 t + b, b = 0..3; its column pair (qq*32 + wi*8 + 2t, + 1) holds k
    // offsets (0, 2), (1, 3).
    const int r = (warp & 3) * 32 + lane;
    const int uset = (warp - 2) >> 2;
    const int rl = r >> 4, g8 = r & 7;
    const int rot = g8 >> 1;
    const bool hi = (r & 8) != 0;
    const int rt = min(rt0 + rl, W.n_rt - 1);
    const float4* szp = W.sz + (size_t)rt * a.groups * 8 + g8;
    // this set's scale/zero pairs one group ahead, so their global load is
    // not on the unpack's critical path
    float4 zn = uset < G ? __ldg(szp + (size_t)uset * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
    const bool r1 = (rot & 1) != 0, r2 = (rot & 2) != 0;
    for (int g = uset; g < G; g += 2) {
      const int s = g % NSW, ab = g % NA;
      const float4 zz = zn;
      if (g + 2 < G) zn = __ldg(szp + (size_t)(g + 2) * 8);
      const float sc = (hi ? zz.z : zz.x) * W.wscale;
      const float nzs = -(hi ? zz.w : zz.y) * sc;
      const unsigned long long sc2 = f32x2_splat(sc), nzs2 = f32x2_splat(nzs);
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kT6Wait>(&wfull[s], (g / NSW) & 1) &&
              (g < NA || mbar_wait_t<kT6Wait>(&aempty[ab], ((g / NA) - 1) & 1)))
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
        // (a per-lane branch here stalled the warps on branch resolution)
        {
          const uint4 v0 = sel4(r1, u[3], u[0]), v1 = sel4(r1, u[0], u[1]);
          const uint4 v2 = sel4(r1, u[1], u[2]), v3 = sel4(r1, u[2], u[3]);
          u[0] = sel4(r2, v2, v0);
          u[1] = sel4(r2, v3, v1);
          u[2] = sel4(r2, v0, v2);
          u[3] = sel4(r2, v1, v3);
        }
        uint32_t col[32];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t wv[4] = {u[t].x, u[t].y, u[t].z, u[t].w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t mm = (hi ? (wv[wi] >> 4) : wv[wi]) & 0x0F0F0F0Fu;
            col[wi * 8 + 2 * t] = nib2_h2(mm, 0x7540u, 0x7542u, sc2, nzs2);       // k offsets 0, 2
            col[wi * 8 + 2 * t + 1] = nib2_h2(mm, 0x7541u, 0x7543u, sc2, nzs2);   // k offsets 1, 3
          }
        }
        tmem_st32(ta + (uint32_t)qq * 32u, col);
      }
      // the group's weights are in registers / TMEM: their slot is free
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ab]);
    }
  } else {
    // ---------------- epilogue: thread = output channel (TMEM lane), NR/2 x rows
    const int quad = warp & 3, rh = (warp - kT6Epi0) >> 2;
    const int ch = quad * 32 + lane;              // channel within the tile
    const int rt = rt0 + (ch >> 4), r16 = ch & 15;
    const bool cvalid = rt < W.n_rt && rt * 16 + r16 < W.rows;
    const int n = rt * 16 + r16;
    constexpr int HALF = NR / 2;
    griddep_wait();
    int ok = 1;
    if (lane == 0) ok = (!stop() && mbar_wait_t<kT6Wait>(tfull, 0)) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {
      if (lane == 0 && !stop()) fail(6);
    } else {
      tc_fence_after();
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(rh * HALF);
#pragma unroll 1
      for (int c0 = 0; c0 < HALF; c0 += 16) {
        if (rh * HALF + c0 >= npad) break;        // warp-uniform
        uint32_t d[16];
        tmem_ld16(tl + (uint32_t)c0, d);
        tmem_wait_ld();
        if (cvalid) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int row = mt * NR + rh * HALF + c0 + i;
            if (row < a.m)
              W.y[(size_t)row * W.ldy + n] = __uint_as_float(d[i]) * W.winv * __ldg(a.xinv + row);
          }
        }
      }
    }
  }
  // every role is done; the MMAs finished before tfull completed, which the
  // epilogue waited for (or the kernel failed, in which case the MMA warp
  // waits here for the commit it made after its last MMA)
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && stop()) mbar_wait_t<kT6Wait>(tfull, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int t6_tensor_map(const Q4GWeight& w, int kqg, CUtensorMap* tm) {
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

template <int KQG, int NR>
int launch_t6(const Q4GWeight* const* ws, int count, const float* x, int m, float* const* ys,
              cudaStream_t st) {
  using L = T6Layout<KQG, NR>;
  Context* c = ctx();
  const Q4GWeight& w0 = *ws[0];
  const int G = (int)w0.groups;
  const int64_t ldx = w0.k;
  const int mts = (m + NR - 1) / NR;
  if (G > 65535) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: %d groups (max 65535)", G);
  // scratch: the prepared tiles, then scale[m] and inv[m]
  const size_t tiles = ((size_t)mts * G * L::XB + 255) & ~(size_t)255;
  const size_t mpad = (size_t)mts * NR;
  unsigned char* xp = nullptr;
  NIMF_TRY(tc_prep_buffer(tiles + 2 * mpad * sizeof(float), st, &xp));
  float* scale = reinterpret_cast<float*>(xp + tiles);
  float* inv = scale + mpad;
  static int attr_dev = -1;
  auto kern = q4g_tc16_kernel<KQG, NR>;
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
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4g_tc16_prep_x, x, ldx, m, (int)w0.k, L::GS, NR,
                                     (const float*)scale, xp));
  }
  for (int i0 = 0; i0 < count; i0 += kT6MaxW) {
    T6Args a = {};
    T6Maps maps;
    int nts = 0;
    a.nw = 0;
    for (int i = i0; i < count && i < i0 + kT6MaxW; ++i) {
      const Q4GWeight& w = *ws[i];
      T6W& t = a.w[a.nw];
      t.sz = (const float4*)w.sz;
      t.y = ys[i];
      t.ldy = w.rows;
      t.rows = (int)w.rows;
      t.n_rt = (int)w.n_rt;
      t.wscale = ldexpf(1.0f, w.tc16_exp);
      t.winv = ldexpf(1.0f, -w.tc16_exp);
      a.nt0[a.nw] = nts;
      NIMF_TRY(t6_tensor_map(w, KQG, &maps.m[a.nw]));
      nts += (int)((w.rows + kT6Chan - 1) / kT6Chan);
      ++a.nw;
    }
    if (nts > 65535)
      return set_error(NIMF_ERR_SHAPE, "prefill GEMM: %d channel tiles in one launch (max 65535)", nts);
    for (int i = a.nw; i < kT6MaxW; ++i) a.nt0[i] = nts;
    a.xp = xp;
    a.xinv = inv;
    a.m = m;
    a.groups = G;
    a.err = c ? c->dev_err : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)mts, (unsigned)nts, 1);
    cfg.blockDim = dim3(kT6Threads, 1, 1);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, maps));
  }
  return NIMF_OK;
}

}  // namespace

bool q4g_tc16_supported(const Q4GWeight& w) {
  return w.fast && w.tc16_ok && (w.gs == 64 || w.gs == 128) && w.rows > 0 && w.k > 0;
}

// ws[0..count) share x (same K and group size, all q4g_tc16_supported)
int q4g_gemm_tc16_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                        float* const* ys, cudaStream_t st) {
  if (m <= 0 || count <= 0) return NIMF_OK;
  if (m > 0x7fffffff / 2) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: M = %lld", (long long)m);
  for (int i = 1; i < count; ++i)
    if (ws[i]->gs != ws[0]->gs || ws[i]->k != ws[0]->k)
      return set_error(NIMF_ERR_SHAPE, "prefill GEMM: grouped weights differ in K or group size");
  // 256-row x tiles unless the grid would then fill under half of the SMs
  // (the unpack of a weight tile is then shared by twice the MMA work)
  Context* c = ctx();
  const int sms = c ? c->num_sms : 148;
  int64_t ctiles = 0;
  for (int i = 0; i < count; ++i) ctiles += (ws[i]->rows + kT6Chan - 1) / kT6Chan;
  const bool wide = m > 128 && ctiles * ((m + 255) / 256) >= sms / 2;
  switch (ws[0]->gs) {
    case 64:
      return wide ? launch_t6<1, 256>(ws, count, x, (int)m, ys, st)
                  : launch_t6<1, 128>(ws, count, x, (int)m, ys, st);
    case 128:
      return wide ? launch_t6<2, 256>(ws, count, x, (int)m, ys, st)
                  : launch_t6<2, 128>(ws, count, x, (int)m, ys, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "prefill GEMM: group size %lld", (long long)ws[0]->gs);
}

}  // namespace nimf
