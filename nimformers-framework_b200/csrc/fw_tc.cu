// fw_tc.cu -- GEMM (x with more than 8 rows) of the byte-coded float
// weights (int8, one-byte CustomFloat E4M3 / E5M2, FP4 E2M1 block-16) on the
// 5th-generation tensor cores: tcgen05.mma kind::f16, fp32 accumulators in
// tensor memory (TMEM).
//
//   y[r][c] = s_c 2^-e_r sum_k w[c][k] xh[r][k],   xh = fp16(x 2^e_r)
//
// Every code of these formats is exact in fp16 (fw.cu), and so is FP4's
// e2m1 x e4m3 block-scale product, so operand A is the weight itself; x is
// rounded once to fp16 after a per-row power-of-two scale that puts the row's
// largest magnitude in [128, 256) (relative 2^-11 per element, the only
// approximation).  s_c is the per-channel / tensor scale, applied once.
//
// One CTA computes y[128 rows of x][128 output channels] over all of K in one
// TMEM accumulator (M=128 channels x N=npad x rows x K=16 per MMA).  Per
// k-block of 128 k: the producer warp copies the prepared x tile (bulk copy)
// and the 8 row tiles' codes of the tensor-core layout (3-D tensor map; FP4
// also its block scales); unpack warps decode the codes into fp16 rows of A
// in TMEM (thread = output channel = TMEM lane) with tcgen05.st; the MMA warp
// issues 8 MMAs from one elected lane of the converged warp.  The epilogue
// warps read the accumulator once at the end.
//
// Warps: 0 producer, 1 TMEM owner and MMA issuer, 2-9 unpack in two sets of 4
// taking alternate k-blocks, 10-13 epilogue.  Every wait is bounded; on expiry
// the kernel records an error in the host-mapped word, the roles run out, and
// TMEM is freed after the MMA warp's last commit.
#include <algorithm>

#include "tc_util.cuh"

namespace nimf {

namespace {

constexpr int kFtRows = 128;                 // x rows per CTA tile
constexpr int kFtChan = 128;                 // channels per CTA tile (8 row tiles)
constexpr int kFtKB = 128;                   // k per stage (k-block)
constexpr int kFtStages = 4;
constexpr int kFtABuf = 4;                   // unpacked A buffers in TMEM
constexpr int kFtUnp0 = 2, kFtEpi0 = 10, kFtWarps = 14;
constexpr int kFtThreads = kFtWarps * 32;
constexpr int kFtRB = 2 * kFtKB;             // bytes per prepared x row of a k-block
constexpr int kFtXB = kFtRows * kFtRB;       // one prepared x tile
constexpr uint32_t kFtACol = kFtRows;        // TMEM: accumulator [0, 128), then A buffers
constexpr uint32_t kFtAW = kFtKB / 2;        // TMEM columns of one A buffer
constexpr int kFtWait = 0;                   // mbar_wait_t style: try_wait, bounded

template <int FMT>
struct FtLayout {
  static constexpr int TK = FMT == FW_FP4 ? 64 : 32;
  static constexpr int TPB = kFtKB / TK;                 // layout tiles per row tile per k-block
  static constexpr int WB = 8 * TPB * 512;               // weight bytes per stage
  static constexpr int SB = FMT == FW_FP4 ? 8 * TPB * 64 : 0;  // FP4 scale bytes per stage
  static constexpr int XOFF = 1024;
  static constexpr int WOFF = XOFF + kFtStages * kFtXB;
  static constexpr int SOFF = WOFF + kFtStages * WB;
  static constexpr int TOTAL = SOFF + kFtStages * SB;
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

// x tile preparation: tile (mt, kb) holds kFtRows rows of kFtKB fp16 values
// fp16(x * scale[row]) in the canonical K-major layout, natural k order; rows
// past m and k past K are zero.  Thread = (row, 8 consecutive k); block = 256
// threads = 16 rows; grid = (tiles x kFtRows / 16, k-blocks).
__global__ void __launch_bounds__(256) fw_tc_prep_x(const float* __restrict__ x, int64_t ldx, int m,
                                                    int k, const float* __restrict__ scale,
                                                    unsigned char* __restrict__ out) {
  const int kb = blockIdx.y, nkb = gridDim.y;
  const int grow = blockIdx.x * 16 + (int)threadIdx.x / 16;
  const int c8 = (int)threadIdx.x % 16;
  const int mt = grow / kFtRows, r = grow % kFtRows;
  unsigned char* base = out + ((size_t)mt * nkb + kb) * kFtXB;
  griddep_wait();  // scale comes from the previous kernel
  const bool rv = grow < m;
  const float sf = rv ? __ldg(scale + grow) : 0.f;
  const int c = kb * kFtKB + c8 * 8;
  const float* xr = x + (size_t)(rv ? grow : 0) * ldx + c;
  const int kvalid = rv ? max(0, min(8, k - c)) : 0;
  float v[8];
  if (kvalid == 8 && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0)) {
    const float4 p = __ldg(reinterpret_cast<const float4*>(xr));
    const float4 q = __ldg(reinterpret_cast<const float4*>(xr + 4));
    v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
    v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = j < kvalid ? __ldg(xr + j) : 0.f;
  }
  uint32_t h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 p = __floats2half2_rn(v[2 * j] * sf, v[2 * j + 1] * sf);
    h[j] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(base + canon_off(r, 16 * c8, kFtRB)) = make_uint4(h[0], h[1], h[2], h[3]);
  griddep_launch_dependents();
}

struct FtArgs {
  const unsigned char* xp;  // prepared x, [mt][kb] tiles
  const float* xinv;        // per-row 2^-e of x's scale
  const float* rscale;      // per-channel scale (nullable: uscale)
  float uscale;
  float* y;                 // [m][ldy]
  int64_t ldy;
  int m, rows, n_rt, nkb;
  int* err;
};
struct FtMaps {
  CUtensorMap w;            // codes: {128 words, ntk tiles, n_rt row tiles}
  CUtensorMap s;            // FP4 scales: {16 words, ntk tiles, n_rt row tiles}
};

// Decodes two codes (16 bits, lower k in the lower byte / nibble) to f16x2.
template <int FMT>
__device__ __forceinline__ uint32_t ft_pair(uint32_t v16) {
  uint32_t r;
  const unsigned short h = (unsigned short)v16;
  if (FMT == FW_E4M3) {
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  } else if (FMT == FW_E5M2) {
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(r) : "h"(h));
  } else {  // int8: 1024 + (q + 128) as fp16, minus 1152
    const uint32_t u = (v16 & 0xFFFFu) ^ 0x8080u;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(r) : "r"(u), "r"(0x64646464u));
    const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&r), __half2half2(__ushort_as_half(0x6480)));
    r = *reinterpret_cast<const uint32_t*>(&d);
  }
  return r;
}
__device__ __forceinline__ uint32_t ft_e2m1x2(uint32_t byte) {
  uint32_t r;
  const unsigned short h = (unsigned short)(byte & 0xFFu);
  asm("{ .reg .b8 lo, hi;\n"
      "  mov.b16 {lo, hi}, %1;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, lo; }"
      : "=r"(r)
      : "h"(h));
  return r;
}

// Exact product of two f16x2 words (e2m1 x e4m3 needs at most 6 bits).
__device__ __forceinline__ uint32_t ft_hmul2(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <int FMT>
__global__ void __launch_bounds__(kFtThreads, 1)
    fw_tc_kernel(const FtArgs a, const __grid_constant__ FtMaps maps) {
  using L = FtLayout<FMT>;
  constexpr int NS = kFtStages, NA = kFtABuf;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* sfull = reinterpret_cast<uint64_t*>(smem);  // producer -> MMA, unpack
  uint64_t* sempty = sfull + NS;                          // MMA + 4 unpack warps -> producer
  uint64_t* afull = sempty + NS;                          // unpack (4 warps) -> MMA
  uint64_t* aempty = afull + NA;                          // MMA -> unpack
  uint64_t* tfull = aempty + NA;                          // MMA -> epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x, nt = blockIdx.y;  // x tile fastest: CTAs of one weight tile run together
  const int rt0 = nt * 8;
  const int nrows = min(kFtRows, a.m - mt * kFtRows);
  const int npad = (nrows + 15) & ~15;
  const int KBN = a.nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], 1 + 4);
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
    // ---------------- producer
    const uint32_t xbytes = (uint32_t)npad * kFtRB;
    int last = -1;
    for (int kb = 0; kb < KBN; ++kb) {
      const int s = kb % NS;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && (kb < NS || mbar_wait_t<kFtWait>(&sempty[s], ((kb / NS) - 1) & 1))) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0 && !stop()) fail(3);
        break;
      }
      if (kb == 0) griddep_wait();  // the prepared x comes from the previous kernel
      if (elect_one()) {
        mbar_arrive_expect_tx(&sfull[s], xbytes + L::WB + L::SB);
        bulk_g2s(smem + L::XOFF + s * kFtXB, a.xp + ((size_t)mt * KBN + kb) * kFtXB, xbytes, &sfull[s]);
        tma_load_3d(smem + L::WOFF + s * L::WB, &maps.w, 0, kb * L::TPB, rt0, &sfull[s]);
        if (FMT == FW_FP4) tma_load_3d(smem + L::SOFF + s * L::SB, &maps.s, 0, kb * L::TPB, rt0, &sfull[s]);
      }
      __syncwarp();
      last = kb;
    }
    if (lane == 0 && last >= 0) {
      for (int kb = max(0, last - NS + 1); kb <= last; ++kb)
        if (!mbar_wait_t<kFtWait>(&sfull[kb % NS], (kb / NS) & 1)) fail(3);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_n(npad);
    const uint64_t bdesc0 = smem_desc(smem + L::XOFF, 128, kFtRB * 8);
    for (int kb = 0; kb < KBN; ++kb) {
      const int s = kb % NS, ab = kb % NA;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kFtWait>(&sfull[s], (kb / NS) & 1) &&
              mbar_wait_t<kFtWait>(&afull[ab], (kb / NA) & 1))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(4);
        break;
      }
      tc_fence_after();
      const uint64_t bd = bdesc0 + (uint64_t)((s * kFtXB) >> 4);
      const uint32_t ta = tmem + kFtACol + (uint32_t)ab * kFtAW;
#pragma unroll
      for (int kk = 0; kk < kFtKB / 16; ++kk)
        if (elect_one())
          umma_f16_ts(tmem, ta + (uint32_t)kk * 8u, bd + (uint64_t)(kk * 16), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
      if (elect_one()) {
        umma_commit(&aempty[ab]);
        umma_commit(&sempty[s]);
      }
      __syncwarp();
    }
    // the accumulator is final (or the kernel failed) once every issued MMA is done
    if (elect_one()) umma_commit(tfull);
    __syncwarp();
  } else if (warp < kFtEpi0) {
    // ---------------- unpack: thread = output channel (TMEM lane).  Row tile
    // rl = r / 16 of the stage, fragment row g8 = r % 8, upper half hi = r & 8.
    // One-byte codes: lane (g8, t) word 2j holds k 16j + 2t, +1 (low 16 bits
    // row g8, high row g8 + 8) and word 2j + 1 the same + 8 -> A columns
    // 8j + t and 8j + t + 4 of the layout tile.  FP4: word j byte (hi, 2 + hi)
    // holds k 16j + 2t, +1 and + 8, +9 -> columns 8j + t and 8j + t + 4 of
    // the tile's 32 columns, times the block scale of subtile j.
    const int r = (warp & 3) * 32 + lane;
    const int uset = (warp - kFtUnp0) >> 2;
    const int rl = r >> 4, g8 = r & 7, rot = g8 >> 1;
    const bool hi = (r & 8) != 0;
    for (int kb = uset; kb < KBN; kb += 2) {
      const int s = kb % NS, ab = kb % NA;
      int ok = 1;
      if (lane == 0)
        ok = (!stop() && mbar_wait_t<kFtWait>(&sfull[s], (kb / NS) & 1) &&
              (kb < NA || mbar_wait_t<kFtWait>(&aempty[ab], ((kb / NA) - 1) & 1)))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(5);
        break;
      }
      tc_fence_after();
      const uint4* wsrc = reinterpret_cast<const uint4*>(smem + L::WOFF + s * L::WB);
      const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + kFtACol + (uint32_t)ab * kFtAW;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t col[32];
#pragma unroll
        for (int tq = 0; tq < (FMT == FW_FP4 ? 1 : 2); ++tq) {
          const int tile = (FMT == FW_FP4 ? half : 2 * half + tq);
          // load j reads fragment lane (g8, (j + rot) & 3): the 8 g8 of a warp
          // hit 8 different 16-byte bank groups; then back to fragment order
          uint4 u[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) u[j] = wsrc[(rl * L::TPB + tile) * 32 + g8 * 4 + ((j + rot) & 3)];
          if (rot & 1) {
            const uint4 t3 = u[3];
            u[3] = u[2];
            u[2] = u[1];
            u[1] = u[0];
            u[0] = t3;
          }
          if (rot & 2) {
            const uint4 t0 = u[0], t1 = u[1];
            u[0] = u[2];
            u[1] = u[3];
            u[2] = t0;
            u[3] = t1;
          }
          if (FMT == FW_FP4) {
            const uint2 sv = reinterpret_cast<const uint2*>(smem + L::SOFF + s * L::SB)[(rl * L::TPB + tile) * 8 + g8];
            const uint32_t sw[2] = {sv.x, sv.y};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // block scale of this channel for subtile j, in both halves
              const uint32_t b = (sw[j >> 1] >> (16 * (j & 1) + 8 * (hi ? 1 : 0))) & 0xFFu;
              uint32_t s2;
              asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s2) : "h"((unsigned short)(b | (b << 8))));
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const uint32_t wv[4] = {u[t].x, u[t].y, u[t].z, u[t].w};
                const uint32_t w = wv[j];
                const uint32_t lo8 = (w >> (hi ? 8 : 0)) & 0xFFu, hi8 = (w >> (hi ? 24 : 16)) & 0xFFu;
                col[8 * j + t] = ft_hmul2(ft_e2m1x2(lo8), s2);
                col[8 * j + t + 4] = ft_hmul2(ft_e2m1x2(hi8), s2);
              }
            }
          } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint32_t wv[4] = {u[t].x, u[t].y, u[t].z, u[t].w};
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const uint32_t w0 = hi ? (wv[2 * j] >> 16) : wv[2 * j];
                const uint32_t w1 = hi ? (wv[2 * j + 1] >> 16) : wv[2 * j + 1];
                col[16 * tq + 8 * j + t] = ft_pair<FMT>(w0);
                col[16 * tq + 8 * j + t + 4] = ft_pair<FMT>(w1);
              }
            }
          }
        }
        tmem_st32(ta + (uint32_t)half * 32u, col);
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
    // ---------------- epilogue: thread = output channel, all npad x rows
    const int quad = warp & 3;
    const int ch = quad * 32 + lane;
    const int n = rt0 * 16 + ch;
    const bool cvalid = n < a.rows;
    const float sc = cvalid ? (a.rscale ? __ldg(a.rscale + n) : a.uscale) : 0.f;
    int ok = 1;
    if (lane == 0) ok = mbar_wait_t<kFtWait>(tfull, 0) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok && lane == 0) fail(6);
    tc_fence_after();
    griddep_wait();  // y may be read by the previous kernel
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
    for (int c0 = 0; c0 < npad; c0 += 16) {
      uint32_t d[16];
      tmem_ld16(tl + (uint32_t)c0, d);
      tmem_wait_ld();
      if (cvalid && ok && !stop()) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int row = mt * kFtRows + c0 + i;
          if (row < a.m) a.y[(size_t)row * a.ldy + n] = __uint_as_float(d[i]) * sc * __ldg(a.xinv + row);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    // every MMA is complete once tfull has its arrival (already seen by the
    // epilogue on the normal path)
    if (lane == 0) mbar_wait_t<kFtWait>(tfull, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int ft_map(void* base, int words, int64_t ntk, int64_t n_rt, int box_tiles, CUtensorMap* tm) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(NIMF_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {(cuuint64_t)words, (cuuint64_t)ntk, (cuuint64_t)n_rt};
  const cuuint64_t strides[2] = {(cuuint64_t)words * 4, (cuuint64_t)ntk * words * 4};
  const cuuint32_t box[3] = {(cuuint32_t)words, (cuuint32_t)box_tiles, 8};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(NIMF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NIMF_OK;
}

template <int FMT>
int ft_launch(const FWLayout& Lw, const float* x, int m, float* y, cudaStream_t st) {
  using L = FtLayout<FMT>;
  Context* c = ctx();
  const int64_t K = Lw.k;
  const int KBN = (int)((Lw.ntk * L::TK + kFtKB - 1) / kFtKB);
  const int mts = (m + kFtRows - 1) / kFtRows;
  const int nts = (int)((Lw.rows + kFtChan - 1) / kFtChan);
  if (KBN > 65535 || nts > 65535) return set_error(NIMF_ERR_SHAPE, "prefill GEMM: shape too large");
  const size_t tiles = ((size_t)mts * KBN * kFtXB + 255) & ~(size_t)255;
  const size_t mpad = (size_t)mts * kFtRows;
  unsigned char* xp = nullptr;
  NIMF_TRY(tc_prep_buffer(tiles + 2 * mpad * sizeof(float), st, &xp));
  float* scale = reinterpret_cast<float*>(xp + tiles);
  float* inv = scale + mpad;
  FtMaps maps;
  NIMF_TRY(ft_map(Lw.frag, 128, Lw.ntk, Lw.n_rt, L::TPB, &maps.w));
  if (FMT == FW_FP4) NIMF_TRY(ft_map(Lw.sfrag, 16, Lw.ntk, Lw.n_rt, L::TPB, &maps.s));
  else maps.s = maps.w;
  static int attr_dev = -1;
  auto kern = fw_tc_kernel<FMT>;
  if (attr_dev != c->device) {
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
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, tc_rowscale, x, (int64_t)K, m, (int)K, scale, inv));
  }
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(mpad / 16), (unsigned)KBN, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, fw_tc_prep_x, x, (int64_t)K, m, (int)K, (const float*)scale, xp));
  }
  FtArgs a = {};
  a.xp = xp;
  a.xinv = inv;
  a.rscale = Lw.rscale;
  a.uscale = Lw.uscale;
  a.y = y;
  a.ldy = Lw.rows;
  a.m = m;
  a.rows = (int)Lw.rows;
  a.n_rt = (int)Lw.n_rt;
  a.nkb = KBN;
  a.err = c->dev_err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)mts, (unsigned)nts, 1);
  cfg.blockDim = dim3(kFtThreads, 1, 1);
  cfg.dynamicSmemBytes = L::TOTAL;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, maps));
  return NIMF_OK;
}

}  // namespace

int fw_gemm_tc(const FWLayout& L, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (m <= 0 || L.rows <= 0) return NIMF_OK;
  if (L.k == 0) {
    NIMF_CUDA_TRY(cudaMemsetAsync(y, 0, (size_t)(m * L.rows) * 4, st));
    return NIMF_OK;
  }
  if (m > 0x7fffffff / 2 || L.rows > 0x7fffffff || L.k > 0x7fffffff)
    return set_error(NIMF_ERR_SHAPE, "prefill GEMM: M = %lld", (long long)m);
  switch (L.fmt) {
    case FW_I8: return ft_launch<FW_I8>(L, x, (int)m, y, st);
    case FW_E4M3: return ft_launch<FW_E4M3>(L, x, (int)m, y, st);
    case FW_E5M2: return ft_launch<FW_E5M2>(L, x, (int)m, y, st);
    case FW_FP4: return ft_launch<FW_FP4>(L, x, (int)m, y, st);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "prefill GEMM: format %d", L.fmt);
}

}  // namespace nimf
