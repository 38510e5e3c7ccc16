// q4g_tc.cu -- int4 group-quantised weights (quant.nim:131-167) times a
// prefill-sized x (M >= 33 rows) on the 5th-generation tensor cores:
// tcgen05.mma kind::i8 with the accumulators in tensor memory (TMEM).
//
// The arithmetic is the decode GEMV's, on 128 x 128 tiles:
//   x[m][k] ~= s[m][g] (d0 + d1 / 256), two signed 8-bit digits per element
//   with one scale per (row of x, quantisation group g), and the weights'
//   nibbles n[c][k] (0..15) exact as unsigned bytes.  Per group
//     sum_k (n - zp) sc x = sc s ((A0 + A1 / 256) - zp D),
//   A0 / A1 the integer dot products of the nibbles with d0 / d1 (exact s32
//   tensor-core sums) and D the group's digit sum.  The weights themselves
//   are never rounded; x carries a relative error below 2^-16 of its group
//   maximum.
//
// One CTA computes y[128 rows of x][128 output channels]:
//   D[channel][j] = sum_k nib[channel][k] * B[j][k],  j < 128: d0 of x row j,
//                                                     j >= 128: d1 of row j-128
// as one M=128, N=256, K=32 MMA per 32 k.  Per quantisation group the
// accumulators go to one of two TMEM buffers (2 x 256 columns) and epilogue
// warps apply the group's scales while the tensor core fills the other one.
//
// Warps: 0 producer (bulk copies of x digits and packed weights, before
// griddepcontrol.wait only what does not depend on the previous kernel),
// 1 TMEM owner and MMA issuer, 2-3 unpack the weights' nibbles into the MMA's
// canonical K-major byte layout, 4-11 epilogue (warp e reads TMEM lanes
// 32 (e % 4) .. + 31 = output channels, for x rows 64 ((e - 4) / 4) .. + 63).
// Every wait is bounded; on expiry the kernel records an error, lets the
// other roles run out and still frees its TMEM.
#include <cuda.h>

#include <algorithm>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr int kTcRows = 128;      // x rows per CTA tile
constexpr int kTcChan = 128;      // output channels per CTA tile (8 row tiles)
constexpr int kTcStages = 4;      // x-digit / packed-weight ring
constexpr int kTcEpi = 4;         // ring of per-group x scales for the epilogue
constexpr int kTcThreads = 12 * 32;
constexpr uint32_t kTmemCols = 512;
#ifndef NIMF_TC_WAIT
#define NIMF_TC_WAIT 0
#endif
// wait style of every role (mbar_wait_t)
constexpr int kTcWait = NIMF_TC_WAIT;

// ------------------------------------------------------------ tcgen05 helpers
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core's reads
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// D (TMEM) (+)= A (smem, u8) x B^T (smem, s8), M=128 N=256 K=32
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// mbarrier arrive once every earlier tcgen05 operation of this thread is done
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// 32 consecutive columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D tensor-map load (no multicast) completing on mbarrier `bar`; x (the
// inner coordinate, in 4-byte elements) is a multiple of 4.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte
// core matrices, lbo = byte distance of the two 16-byte K halves of an MMA's
// 32-byte K step, sbo = byte distance of consecutive 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((smem_addr(p) >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version of this architecture
  return d;
}

// Instruction descriptor: s32 accumulate, A u8, B s8, both K-major,
// N = 256, M = 128.
constexpr uint32_t kIdescI8 = (2u << 4) | (0u << 7) | (1u << 10) | ((256u >> 3) << 17) |
                              ((128u >> 4) << 24);

// Byte offset of (row r, k) in a K-major canonical tile with `kbytes` of K.
__host__ __device__ __forceinline__ uint32_t canon_off(int r, int k, int kbytes) {
  return (uint32_t)((r >> 3) * (kbytes * 8) + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}

// x preparation, one CTA per (128-row tile mt, group g), thread = row:
//   [d0: 128 x gs bytes][d1: 128 x gs bytes] in the canonical layout,
//   then s[128] (digit scale) and dz[128] (d0 sum + d1 sum / 256) as floats.
// Rows past m are zero.
__global__ void q4g_tc_prep_x(const float* __restrict__ x, int64_t ldx, int m, int k, int gs,
                              int groups, unsigned char* __restrict__ out) {
  const int mt = blockIdx.x / groups, g = blockIdx.x - (blockIdx.x / groups) * groups;
  const int r = threadIdx.x;
  const int row = mt * kTcRows + r;
  const size_t plane = (size_t)kTcRows * gs;
  unsigned char* base = out + (size_t)blockIdx.x * (2 * plane + 2 * kTcRows * 4);
  float* sv = reinterpret_cast<float*>(base + 2 * plane);
  float* dz = sv + kTcRows;
  griddep_wait();  // x may be written by the previous kernel in the stream
  const bool rv = row < m;
  const float* xr = x + (size_t)(rv ? row : 0) * ldx + (size_t)g * gs;
  const int kvalid = rv ? max(0, min(gs, k - g * gs)) : 0;
  float mx = 0.f;
  for (int i = 0; i < gs; ++i) {
    const float v = i < kvalid ? __ldg(xr + i) : 0.f;
    mx = fmaxf(mx, fabsf(v));
  }
  const float inv = mx > 0.f ? 127.0f / mx : 0.f;
  int s0 = 0, s1 = 0;
  for (int c = 0; c < gs; c += 16) {
    uint32_t w0[4], w1[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t a = 0, b = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = c + 4 * q + e;
        const float v = i < kvalid ? __ldg(xr + i) : 0.f;
        const float t = v * inv;
        const int d0 = max(-127, min(127, __float2int_rn(t)));
        const int d1 = max(-127, min(127, __float2int_rn((t - (float)d0) * 256.0f)));
        a |= (uint32_t)(d0 & 0xFF) << (8 * e);
        b |= (uint32_t)(d1 & 0xFF) << (8 * e);
        s0 += d0;
        s1 += d1;
      }
      w0[q] = a;
      w1[q] = b;
    }
    *reinterpret_cast<uint4*>(base + canon_off(r, c, gs)) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    *reinterpret_cast<uint4*>(base + plane + canon_off(r, c, gs)) =
        make_uint4(w1[0], w1[1], w1[2], w1[3]);
  }
  sv[r] = mx * (1.0f / 127.0f);
  dz[r] = (float)s0 + (float)s1 * (1.0f / 256.0f);
  griddep_launch_dependents();
}

struct TcArgs {
  const uint4* frag;     // weight fragments, row tile 0
  const float4* sz;      // scale/zero pairs, row tile 0
  const unsigned char* xp;  // prepared x, [mt][g]
  float* y;
  int64_t ldy;
  int m, rows, n_rt, kq_total, groups;
  int* err;
};

// Shared memory (offsets from the 1024-aligned base)
template <int KQG>
struct TcLayout {
  static constexpr int GS = 64 * KQG;
  static constexpr int DBYTES = 2 * kTcRows * GS;                    // digit planes d0, d1
  static constexpr int EBYTES = 2 * kTcRows * 4;                     // s and dz
  static constexpr int XBYTES = DBYTES + EBYTES;                     // one prepared group
  static constexpr int WBYTES = 8 * KQG * 512;                       // packed weights
  static constexpr int ABYTES = kTcChan * GS;                        // unpacked nibbles
  static constexpr int XOFF = 1024;                                  // after the barriers
  static constexpr int WOFF = XOFF + kTcStages * DBYTES;
  static constexpr int EOFF = WOFF + kTcStages * WBYTES;
  static constexpr int AOFF = (EOFF + kTcEpi * EBYTES + 1023) / 1024 * 1024;
  static constexpr int TOTAL = AOFF + 2 * ABYTES;
};

// wmap: the weight fragments as a 2-D tensor of 4-byte elements, one row per
// row tile (kq_total * 128 elements); its box is 8 row tiles x one group.
template <int KQG>
__global__ void __launch_bounds__(kTcThreads, 1)
    q4g_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap wmap) {
  using L = TcLayout<KQG>;
  constexpr int GS = L::GS;
  constexpr int KSTEPS = GS / 32;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw;
  uint64_t* sfull = reinterpret_cast<uint64_t*>(smem);    // producer -> MMA, unpack
  uint64_t* sempty = sfull + kTcStages;                    // MMA + 2 unpack warps -> producer
  uint64_t* efull = sempty + kTcStages;                    // producer -> epilogue
  uint64_t* eempty = efull + kTcEpi;                       // 8 epilogue warps -> producer
  uint64_t* afull = eempty + kTcEpi;                       // [2] unpack -> MMA
  uint64_t* aempty = afull + 2;                            // [2] MMA -> unpack
  uint64_t* tfull = aempty + 2;                            // [2] MMA -> epilogue
  uint64_t* tempty = tfull + 2;                            // [2] epilogue -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int G = a.groups;
  const int rt0 = nt * 8;
  const int nrt = max(0, min(8, a.n_rt - rt0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], 1 + 2);
    }
    for (int s = 0; s < kTcEpi; ++s) {
      mbar_init(&efull[s], 1);
      mbar_init(&eempty[s], 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 2);
      mbar_init(&aempty[b], 1);
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
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
    // ---------------- producer: per group, x digits, x scales and the 8 row
    // tiles' packed nibbles (one tensor-map box; rows past the weight read 0)
    int last = -1;
    for (int g = 0; g < G; ++g) {
      const int s = g % kTcStages, es = g % kTcEpi;
      // lane 0 decides for the warp, so its lanes leave the loop together
      int ok = 1;
      if (lane == 0)
        ok = (!stop() &&
              (g < kTcStages || mbar_wait_t<kTcWait>(&sempty[s], ((g / kTcStages) - 1) & 1)) &&
              (g < kTcEpi || mbar_wait_t<kTcWait>(&eempty[es], ((g / kTcEpi) - 1) & 1)))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0 && !stop()) fail(3);
        break;
      }
      unsigned char* xs = smem + L::XOFF + s * L::DBYTES;
      unsigned char* ws = smem + L::WOFF + s * L::WBYTES;
      unsigned char* ep = smem + L::EOFF + es * L::EBYTES;
      if (lane == 0) {
        mbar_arrive_expect_tx(&sfull[s], L::DBYTES + L::WBYTES);
        mbar_arrive_expect_tx(&efull[es], L::EBYTES);
        if (g == 0) griddep_wait();  // the prepared x comes from the previous kernel
      }
      __syncwarp();
      const unsigned char* src = a.xp + ((size_t)mt * G + g) * L::XBYTES;
      if (lane == 0) bulk_g2s(xs, src, L::DBYTES, &sfull[s]);
      if (lane == 1) bulk_g2s(ep, src + L::DBYTES, L::EBYTES, &efull[es]);
      if (lane == 2) tma_load_2d(ws, &wmap, g * KQG * 128, rt0, &sfull[s]);
      last = g;
    }
    // the last copies land before the CTA may exit
    if (lane == 0 && last >= 0) {
      for (int g = max(0, last - kTcStages + 1); g <= last; ++g)
        if (!mbar_wait_t<kTcWait>(&sfull[g % kTcStages], (g / kTcStages) & 1)) fail(3);
      for (int g = max(0, last - kTcEpi + 1); g <= last; ++g)
        if (!mbar_wait_t<kTcWait>(&efull[g % kTcEpi], (g / kTcEpi) & 1)) fail(3);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      for (int g = 0; g < G; ++g) {
        const int s = g % kTcStages, b = g & 1;
        if (stop() || !mbar_wait_t<kTcWait>(&sfull[s], (g / kTcStages) & 1) ||
            !mbar_wait_t<kTcWait>(&afull[b], (g >> 1) & 1) ||
            (g >= 2 && !mbar_wait_t<kTcWait>(&tempty[b], ((g >> 1) - 1) & 1))) {
          fail(4);
          break;
        }
        tc_fence_after();
        const unsigned char* at = smem + L::AOFF + b * L::ABYTES;
        const unsigned char* bt = smem + L::XOFF + s * L::DBYTES;
        const uint32_t td = tmem + (uint32_t)b * 256u;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk)
          umma_i8(td, smem_desc(at + kk * 256, 128, GS * 8), smem_desc(bt + kk * 256, 128, GS * 8),
                  kIdescI8, kk > 0 ? 1u : 0u);
        umma_commit(&aempty[b]);
        umma_commit(&tfull[b]);
        umma_commit(&sempty[s]);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ---------------- unpack: packed nibbles (fragment order) -> u8 canonical
    const int ut = threadIdx.x - 64;  // 0..63
    for (int g = 0; g < G; ++g) {
      const int s = g % kTcStages, b = g & 1;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kTcWait>(&sfull[s], (g / kTcStages) & 1) &&
              (g < 2 || mbar_wait_t<kTcWait>(&aempty[b], ((g >> 1) - 1) & 1)))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(5);
        break;
      }
      const uint4* wsrc = reinterpret_cast<const uint4*>(smem + L::WOFF + s * L::WBYTES);
      unsigned char* at = smem + L::AOFF + b * L::ABYTES;
      for (int i = ut; i < nrt * KQG * 32; i += 64) {
        const int rl = i / (KQG * 32), qq = (i / 32) % KQG, ln = i & 31;
        const int gq = ln >> 2, t = ln & 3;
        const uint4 w = wsrc[i];
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const int kloc = qq * 64 + 32 * (wi >> 1) + 16 * (wi & 1) + 4 * t;
          const uint32_t lo = words[wi] & 0x0F0F0F0Fu, hi = (words[wi] >> 4) & 0x0F0F0F0Fu;
          *reinterpret_cast<uint32_t*>(at + canon_off(rl * 16 + gq, kloc, GS)) = lo;
          *reinterpret_cast<uint32_t*>(at + canon_off(rl * 16 + 8 + gq, kloc, GS)) = hi;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[b]);
        mbar_arrive(&sempty[s]);
      }
    }
  } else {
    // ---------------- epilogue: thread = output channel (TMEM lane), 64 x rows
    const int e = warp - 4;
    const int quad = e & 3, half = e >> 2;
    const int ch = quad * 32 + lane;              // channel within the tile
    const int rt = rt0 + (ch >> 4), r16 = ch & 15;
    const bool cvalid = rt < a.n_rt && rt * 16 + r16 < a.rows;
    const float4* szp = a.sz + ((size_t)min(rt, a.n_rt - 1) * a.groups) * 8 + (r16 & 7);
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    griddep_wait();
    for (int g = 0; g < G; ++g) {
      const int es = g % kTcEpi, b = g & 1;
      const float4 zz = __ldg(szp + (size_t)g * 8);
      // y += sc s / 256 ((256 A0 + A1) - 256 zp dz): one conversion per element
      const float sc = ((r16 >> 3) ? zz.z : zz.x) * (1.0f / 256.0f);
      const float zp = ((r16 >> 3) ? zz.w : zz.y) * 256.0f;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kTcWait>(&tfull[b], (g >> 1) & 1) &&
              mbar_wait_t<kTcWait>(&efull[es], (g / kTcEpi) & 1))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(6);
        break;
      }
      tc_fence_after();
      const float4* sv4 = reinterpret_cast<const float4*>(smem + L::EOFF + es * L::EBYTES);
      const float4* dz4 = sv4 + kTcRows / 4;
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)b * 256u;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t c0[32], c1[32];
        const int j0 = half * 64 + c * 32;  // first x row of this chunk
        tmem_ld32(tl + (uint32_t)j0, c0);
        tmem_ld32(tl + 128u + (uint32_t)j0, c1);
        tmem_wait_ld();
        if (c == 1) {
          // both chunks are in registers: the buffer may be refilled
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          const float4 s4 = sv4[(j0 >> 2) + i4], d4 = dz4[(j0 >> 2) + i4];
          const float sv[4] = {s4.x, s4.y, s4.z, s4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int i = i4 * 4 + e4;
            const float u = (float)((int)c0[i] * 256 + (int)c1[i]);
            acc[c * 32 + i] = fmaf(sc * sv[e4], fmaf(-zp, dv[e4], u), acc[c * 32 + i]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&eempty[es]);
    }
    if (cvalid && !stop()) {
      const int n = rt * 16 + r16;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int row = mt * kTcRows + half * 64 + i;
        if (row < a.m) a.y[(size_t)row * a.ldy + n] = acc[i];
      }
    }
  }
  // every role is done; outstanding MMAs finished before the last tfull
  // phase, which the epilogue waited for (or the kernel failed, in which case
  // the MMA thread waits here for its own last commit)
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && stop() && G > 0) mbar_wait_t<kTcWait>(&tfull[(G - 1) & 1], ((G - 1) >> 1) & 1);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// x-preparation scratch, one buffer per device, grown outside stream capture
struct PrepBuf {
  int device = -1;
  void* p = nullptr;
  size_t bytes = 0;
};
PrepBuf g_prep[16];

int prep_buffer(size_t bytes, cudaStream_t st, unsigned char** out) {
  Context* c = ctx();
  const int dev = c ? c->device : 0;
  PrepBuf& b = g_prep[dev & 15];
  if (b.device != dev || b.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "int4 prefill GEMM: its x scratch must grow, which cannot happen during "
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependence on the driver library).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int weight_tensor_map(const Q4GWeight& w, int kqg, CUtensorMap* tm) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    NIMF_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess)
      return set_error(NIMF_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    fn = (EncodeTiledFn)p;
  }
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
int launch_tc(const Q4GWeight& w, const float* x, int64_t ldx, int m, float* y, int64_t ldy,
              cudaStream_t st) {
  using L = TcLayout<KQG>;
  Context* c = ctx();
  const int G = (int)w.groups;
  const int mts = (m + kTcRows - 1) / kTcRows;
  const int nts = (int)((w.rows + kTcChan - 1) / kTcChan);
  unsigned char* xp = nullptr;
  NIMF_TRY(prep_buffer((size_t)mts * G * L::XBYTES, st, &xp));
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
    cfg.gridDim = dim3((unsigned)(mts * G), 1, 1);
    cfg.blockDim = dim3(kTcRows, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4g_tc_prep_x, x, ldx, m, (int)w.k, 64 * KQG, G, xp));
  }
  TcArgs a;
  a.frag = (const uint4*)w.frag;
  a.sz = (const float4*)w.sz;
  a.xp = xp;
  a.y = y;
  a.ldy = ldy;
  a.m = m;
  a.rows = (int)w.rows;
  a.n_rt = (int)w.n_rt;
  a.kq_total = (int)w.kq_total;
  a.groups = G;
  a.err = c ? c->dev_err : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nts, (unsigned)mts, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = L::TOTAL;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap wmap;
  NIMF_TRY(weight_tensor_map(w, KQG, &wmap));
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, wmap));
  return NIMF_OK;
}

}  // namespace

// Group sizes 64 and 128 (256 would need more shared memory than a CTA has).
bool q4g_tc_supported(const Q4GWeight& w) {
  return w.fast && (w.gs == 64 || w.gs == 128) && w.rows > 0 && w.k > 0;
}

int q4g_gemm_tc(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (m <= 0 || w.rows <= 0) return NIMF_OK;
  if (m > 0x7fffffff / 2) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: M = %lld", (long long)m);
  switch (w.gs) {
    case 64: return launch_tc<1>(w, x, w.k, (int)m, y, w.rows, st);
    case 128: return launch_tc<2>(w, x, w.k, (int)m, y, w.rows, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "prefill GEMM: group size %lld", (long long)w.gs);
}

}  // namespace nimf
