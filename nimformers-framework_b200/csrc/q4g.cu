// q4g.cu -- int4 asymmetric per-group weights (QuantTensor kind 3 with
// groupSize > 0, quant.nim:131-167) on sm_100a: device repack, bit-exact
// dequantisation and the decode GEMV y[M][N] = x[M][K] . W^T (M <= 16; more
// rows go to the tensor-core GEMM in q4g_tc.cu).
//
// GEMV design (memory-bound: 0.5 B of weight per multiply-add):
//   * Weights are repacked once at registration into mma.sync m16n8k32
//     A-fragment order: for row tile rt (16 output rows) and k-quad kq (64 k),
//     lane (g, t) of a warp owns one uint4 whose word 2h + half holds, in
//     byte b, the nibbles of k = 32h + 16half + 4t + b for rows g (low
//     nibble) and g + 8 (high nibble).  A row tile's quads are one
//     contiguous range, streamed by bulk copies.
//   * Persistent kernel, one CTA per SM: a producer warp fills an mbarrier
//     ring with cp.async.bulk copies (before griddepcontrol.wait, so the next
//     launch's weights stream while the previous kernel drains), 16 consumer
//     warps and a merge warp.
//   * x is quantised per CTA into two signed 8-bit digits,
//     x ~= s (d0 + d1 / 256) with s = max|x| / 127; consumers unpack the
//     nibbles with two masks and run mma.sync m16n8k32 s8 against the digits,
//     so the dot products are exact integers.  Per group the fp32 epilogue
//     applies sc s (A - zp D) with D the exact digit sum: the algebra of
//     sum_k (n_k - zp) sc x_k.  The dequantised weights themselves
//     (q4g_dequant below) are bit-identical to the reference.
//   * The merge warp sums chunk partials of a row tile in a fixed order and
//     writes y (deterministic).
//   * Row tiles are cut into k-blocks of about 36 KB (direct mode); when
//     there are too few row tiles for the SMs, CTAs of a thread-block cluster
//     split K and reduce through distributed shared memory in rank order.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <cstring>

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

// Fragment order of the packed weights (one uint4 per lane per 64-k quad):
// word w = 2h + half of lane (g, t) covers k = 32h + 16*half + 4t + b (byte
// b = 0..3); the low nibble of byte b is row g, the high nibble row g + 8.
// Hence (w & 0x0F0F0F0F) and ((w >> 4) & 0x0F0F0F0F) are exactly the s8 A
// fragments {row g, row g+8} x k[4t..4t+3] of mma.m16n8k32.
__device__ __forceinline__ int nib_k(int w, int t, int b) {
  return 32 * (w >> 1) + 16 * (w & 1) + 4 * t + b;
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
  for (int wi = 0; wi < 4; ++wi) {
    uint32_t w = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int64_t col = kq * 64 + nib_k(wi, t, b);
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int64_t row = rt * 16 + g + 8 * hi;
        uint32_t nib = 0;
        if (row < rows && col < k) {
          const uint8_t byte = wq[row * bpr + (col >> 1)];
          nib = (col & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15);
        }
        w |= nib << (8 * b + 4 * hi);
      }
    }
    words[wi] = w;
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

// *bad = 1 if a zero point is not finite or |zp| >= 60000 (the tensor-core
// GEMM carries zp + 64 as two fp16 parts).
// Registration checks of the tensor-core paths, over every (row, group):
// st[0] = 1 if a zero point is not finite or |zp| >= 60000 (the exact-nibble
// GEMM splits 64 + zp into two fp16 parts); st[1] = the largest dequantised
// magnitude sc * max(|zp|, |15 - zp|) and st[2] = the smallest non-zero |sc|,
// as float bits (non-negative floats order like their bits), for the
// fp16-tile GEMM's range check.
__global__ void q4g_zp_range(const float* __restrict__ sc, const float* __restrict__ zp,
                             int64_t ngr, int64_t rows, unsigned* __restrict__ st) {
  const int64_t n = rows * ngr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float z = zp[i], a = fabsf(sc[i]);
    if (!(fabsf(z) < 60000.0f)) st[0] = 1u;
    const float m = a * fmaxf(fabsf(z), fabsf(15.0f - z));
    atomicMax(&st[1], m == m ? __float_as_uint(m) : 0x7F800000u);   // NaN counts as inf
    if (a > 0.0f) atomicMin(&st[2], a == a ? __float_as_uint(a) : 0x7F800000u);
  }
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
  const int g = r & 7, rhi = r >> 3;
  const int kk = (int)(col & 63);                 // k within the quad
  const int h = kk >> 5, half = (kk >> 4) & 1, t = (kk & 15) >> 2, b = kk & 3;
  const int lane = g * 4 + t;
  const uint4 v = frag[((rt * kq_total) + (col >> 6)) * 32 + lane];
  const int wi = 2 * h + half;
  const uint32_t word = wi == 0 ? v.x : (wi == 1 ? v.y : (wi == 2 ? v.z : v.w));
  const uint32_t nib = (word >> (8 * b + 4 * rhi)) & 15u;
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

// One weight of a (grouped) launch: its row tiles occupy global row tiles
// [rt_prefix[p], rt_prefix[p+1]) of the launch.
constexpr int kMaxProblems = 16;
struct GemvProblem {
  const uint4* frag;
  const float4* sz;
  float* y;
  int64_t ldy;
  int rows;
};

struct GemvArgs {
  GemvProblem prob[kMaxProblems];
  int rt_prefix[kMaxProblems + 1];
  int nprob;
  const float* x;
  int* err;            // host-mapped error word (1: a bounded wait expired)
  int64_t ldx;
  int m, k, n_rt;      // n_rt: total row tiles of the launch
  int kq_total, groups;
  int gps;             // quantisation groups per k-split (the last split may have fewer)
  int kbg, nkb;        // groups per ring stage (k-block) and k-blocks per row tile
  int n_clusters;      // clusters in the grid; cluster size = number of k-splits
  int tchunk;          // max row tiles per cluster (sizes the partial-y buffers)
  int ns;              // stages in the weight ring (a multiple of kCons)
  int vec4;            // x rows 16-byte aligned
  // Fused all-gather of N-shard outputs (world > 1): every y value is also
  // stored at the same offset of each rank's output buffer (rank q's copy of
  // a local address p is p + peer_off[q] bytes, through CUDA IPC); the last
  // CTA to finish raises one arrival on every rank and waits (bounded) until
  // every rank's arrival for this launch is in, so the launch completes with
  // the gathered outputs in place on this rank.
  int world;
  long long peer_off[kCommMaxRanks];
  unsigned* gctl;      // local control words: [0] launches, [1] CTAs done, [2] rank arrivals
  unsigned long long wait_ns;
};

__device__ __forceinline__ void gather_store(const GemvArgs& a, float* p, float v) {
  if (a.world <= 1) {
    *p = v;
    return;
  }
  for (int q = 0; q < a.world; ++q)
    *reinterpret_cast<float*>(reinterpret_cast<char*>(p) + a.peer_off[q]) = v;
}

// End of a gathering launch, called by every CTA after a __syncthreads that
// follows its last y stores (each storing thread fenced them at system scope).
__device__ void gather_finish(const GemvArgs& a) {
  if (threadIdx.x != 0) return;
  unsigned* done = a.gctl + 1;
  if (atomicAdd(done, 1u) != gridDim.x - 1) return;
  // the last CTA of this rank's launch: nothing else of the launch touches
  // the control words now, and the next launch on this stream starts after
  // this one completes
  *done = 0u;
  const unsigned epoch = *(volatile unsigned*)a.gctl;
  __threadfence_system();
  for (int q = 0; q < a.world; ++q) {
    unsigned* arr = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(a.gctl + 2) + a.peer_off[q]);
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(arr) : "memory");
  }
  const unsigned target = (epoch + 1u) * (unsigned)a.world;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (unsigned it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.gctl + 2) : "memory");
    if ((int)(v - target) >= 0) break;
    if ((it & 63u) == 63u) {
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > a.wait_ns) {
        if (a.err) atomicExch(a.err, 5);
        break;
      }
    }
    __nanosleep(64);
  }
  *(volatile unsigned*)a.gctl = epoch + 1u;
  __threadfence();
}

// A stage holds one k-block of a row tile's slice of this CTA's k-split
// (packed weights, then the scale/zero pairs of its groups), moved by two bulk
// copies; a row tile spans nkb stages.  A stage is consumed as chunks of
// kChunkQ k-quads (512 k), one chunk per warp-unit.
constexpr int kChunkQ = 8;
#ifndef NIMF_Q4G_ISSUERS
#define NIMF_Q4G_ISSUERS 4
#endif
constexpr int kIssuers = NIMF_Q4G_ISSUERS;  // producer lanes issuing stages round-robin
#ifndef NIMF_Q4G_PWAIT
#define NIMF_Q4G_PWAIT -32
#endif
#ifndef NIMF_Q4G_CWAIT
#define NIMF_Q4G_CWAIT 1000
#endif
// Wait styles (mbar_wait_t) of the producer lanes and of the consumer warps.
// The producer's lanes diverge, so they poll instead of sleeping in try_wait.
constexpr int kProdWait = NIMF_Q4G_PWAIT;
constexpr int kConsWait = NIMF_Q4G_CWAIT;

// Shared-memory layout of one CTA:
//   head: full/empty/merged/pfull[kStages] mbarriers,
//         xmax[8] (|x| maxima as float bits), 16 B spare, problem table
//   ring[ns][stage]   k-blocks of row tiles (packed weights, then the
//                     scale/zero pairs of their groups)
//   xs    B fragments of the two s8 digits of x for the k-split:
//         MODE 1: [k32 tiles][2M columns][4 lanes t] uint2 (d0 of row m in
//                 column m, d1 in column M + m)
//         MODE 2: [k32 tiles][M][4 lanes t] uint4 {d0 b0, d0 b1, d1 b0, d1 b1}
//   sdi   [gps][16] int: per group, sums of the d0 (0..7) and d1 (8..15) digits
//   part  split mode: [tchunk*ncs][16][8] per-unit partial y; direct mode (no
//         k-split): [ns][ncs][16][8] per-stage slots summed into y in-CTA
struct SmemLayout {
  size_t ring, stage, xs, sdi, part, total;
};

// + the launch's problem table copied to shared memory (pointers, y strides,
// rows, row-tile prefix): dynamic indexing into kernel parameters is slow
constexpr size_t kBarBytes = 4 * kStages * sizeof(uint64_t) + 64;
constexpr size_t kTabBytes = 3 * kMaxProblems * 8 + kMaxProblems * 8 + kMaxProblems * 4 + 80;
constexpr size_t kHeadBytes = kBarBytes + kTabBytes;

__host__ __device__ inline SmemLayout q4g_smem_layout(int mode, int kqg, int gps, int kbg, int m,
                                                      int ns, int tchunk, bool direct) {
  SmemLayout L;
  const int cg = kChunkQ / kqg;                       // groups per chunk
  const int nchunk = (kbg + cg - 1) / cg;             // chunks per stage
  L.stage = (size_t)kbg * kqg * 512 + (size_t)kbg * 128;  // one k-block
  L.ring = (kHeadBytes + 127) / 128 * 128;
  L.xs = L.ring + L.stage * ns;
  const size_t k32 = (size_t)gps * kqg * 2;
  L.sdi = L.xs + k32 * (mode == 1 ? 2 * m * 4 * 8 : m * 4 * 16);
  L.part = L.sdi + (size_t)gps * 16 * sizeof(int);
  L.part = (L.part + 15) & ~(size_t)15;
  L.total = L.part + (size_t)(direct ? ns : tchunk) * nchunk * 16 * 8 * sizeof(float);
  return L;
}

// One CTA = k-split `rank` of the row tiles of its cluster.  Warp kCons is the
// producer (lanes 0..kIssuers-1 stream row-tile slices with bulk copies);
// consumer warp w takes the 512-k chunk units (stage q, chunk c) with
// (q * ncs + c) % kCons == w (ncs = nominal chunks per stage, the same on
// every rank); ring slot q % ns therefore always serves the same warps (ns is
// a multiple of kCons / gcd(ncs, kCons)), so no warp ever waits more than one
// phase ahead on a stage barrier.  In direct mode (no k-split) warp kCons + 1
// sums the chunk partials of each row tile's stages and writes y.
//
// Math: the nibbles (0..15, exact s8) multiply two s8 digits of x,
// x ~= s_m (d0 + d1 / 256) with s_m = max|x_m| / 127 over the k-split, on the
// s8 tensor cores (mma.m16n8k32, exact s32 sums); per group the fp32 epilogue
// applies  sum_k (n - zp) sc x = sc s_m (A - zp D)  with A the MMA sum and D
// the digit sum.  The weight values themselves are never rounded.
// MODE 1: M <= 4, one MMA per 32 k (d0 in columns 0..3, d1 in 4..7).
// MODE 2: M <= 8, two MMAs per 32 k (d0 and d1 each in columns 0..7).
// KQG: k-quads (64 k) per quantisation group (group size 64 * KQG).
// M1 (MODE 1 only): exactly one row of x, so the B column stride is a
// constant and only the two result columns of x row 0 are computed.
template <int MODE, int KQG, bool M1>
__global__ void __launch_bounds__((kCons + 2) * 32, kCtasPerSm)
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
  const bool direct = nsplit == 1;  // no k-split: row tiles are finished in-CTA
  const int nkb = a.nkb;
  const int ncs = (a.kbg + CG - 1) / CG;           // nominal chunks per stage (every rank)
  // split mode has one stage per row tile; its last rank may have fewer chunks
  const int nchunk = direct ? ncs : (ng + CG - 1) / CG;
  const int nstg = nrt * nkb;                      // stages of this CTA
  const int nunits = nstg * ncs;
  // groups of k-block kb (the last k-block may have fewer)
  auto kb_groups = [&](int kb) { return max(0, min(a.kbg, ng - kb * a.kbg)); };
  const int NS = a.ns;

  const SmemLayout Ls = q4g_smem_layout(MODE, KQG, a.gps, a.kbg, a.m, NS, a.tchunk, direct);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  uint64_t* merged = empty + kStages;  // direct mode: the stage's partial slots are free again
  uint64_t* pfull = merged + kStages;  // direct mode: all chunk partials of the stage written
  unsigned* xmax = reinterpret_cast<unsigned*>(pfull + kStages);
  const uint4** tfrag = reinterpret_cast<const uint4**>(smem + kBarBytes);
  const float4** tsz = reinterpret_cast<const float4**>(tfrag + kMaxProblems);
  float** ty = reinterpret_cast<float**>(smem + kBarBytes + 2 * kMaxProblems * 8);
  int64_t* tldy = reinterpret_cast<int64_t*>(ty + kMaxProblems);
  int* trows = reinterpret_cast<int*>(tldy + kMaxProblems);
  int* tpref = trows + kMaxProblems;
  // problem of global row tile grt (problems are few; p only grows with grt)
  auto prob_of = [&](int grt, int p) {
    while (p + 1 < a.nprob && grt >= tpref[p + 1]) ++p;
    return p;
  };
  unsigned char* ring = smem + Ls.ring;
  unsigned char* xs = smem + Ls.xs;
  int* sdi = reinterpret_cast<int*>(smem + Ls.sdi);
  float* part = reinterpret_cast<float*>(smem + Ls.part);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nchunk > 0 ? nchunk : 1);
      mbar_init(&merged[s], 1);
      mbar_init(&pfull[s], nchunk > 0 ? nchunk : 1);
    }
    mbar_fence_init();
  }
  if (threadIdx.x < a.nprob) {
    const int i = threadIdx.x;
    tfrag[i] = a.prob[i].frag;
    tsz[i] = a.prob[i].sz;
    ty[i] = a.prob[i].y;
    tldy[i] = a.prob[i].ldy;
    trows[i] = a.prob[i].rows;
  }
  if (threadIdx.x <= a.nprob) tpref[threadIdx.x] = a.rt_prefix[threadIdx.x];
  if (threadIdx.x < 8) xmax[threadIdx.x] = 0u;
  for (int i = threadIdx.x; i < ng * 16; i += blockDim.x) sdi[i] = 0;
  __syncthreads();

  if (warp == kCons) {
    // ---------------- producer.  Weights do not depend on earlier kernels, so
    // this runs without griddepcontrol.wait and overlaps the previous kernel.
    // Lanes 0..kIssuers-1 own the stages s = lane (mod kIssuers).
    griddep_launch_dependents();
    if (lane < kIssuers && ng > 0) {
      bool ok = true;
      int issued_last = -1;
      int pp = 0;
      for (int q = lane; q < nstg; q += kIssuers) {
        const int s = q % NS;
        if (q >= NS && !mbar_wait_t<kProdWait>(&empty[s], ((q / NS) - 1) & 1)) {
          ok = false;
          break;
        }
        const int i = q / nkb, kb = q - i * nkb;
        const int ngk = kb_groups(kb), gk0 = g0 + kb * a.kbg;
        const uint32_t wb = (uint32_t)ngk * KQG * 512u, zb = (uint32_t)ngk * 128u;
        const int grt = rt0 + i;
        pp = prob_of(grt, pp);
        const int p = pp;
        const int rt = grt - tpref[p];
        unsigned char* dst = ring + (size_t)s * Ls.stage;
        mbar_arrive_expect_tx(&full[s], wb + zb);
        bulk_g2s(dst, tfrag[p] + ((size_t)rt * a.kq_total + (size_t)gk0 * KQG) * 32, wb,
                 &full[s]);
        bulk_g2s(dst + (size_t)a.kbg * KQG * 512,
                 tsz[p] + ((size_t)rt * a.groups + gk0) * 8, zb, &full[s]);
        issued_last = q;
      }
      // drain: this lane's last copies land before the CTA may exit
      if (ok) {
        for (int q = issued_last; q >= 0 && q > issued_last - NS; q -= kIssuers)
          if (!mbar_wait_t<kProdWait>(&full[q % NS], (q / NS) & 1)) ok = false;
      }
      if (!ok && a.err) atomicExch(a.err, 1);
    }
    __syncwarp();
  } else if (warp == kCons + 1) {
    // ---------------- merger (direct mode): sums each row tile's chunk
    // partials in chunk order (deterministic), writes y and frees the
    // stage's partial slots for the next round
    if (direct) {
      griddep_wait();  // y may be read or written by the previous kernel
      int pp = 0;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < nstg; ++q) {
        const int s = q % NS;
        const int i = q / nkb, kb = q - i * nkb;
        if (!mbar_wait_t<kConsWait>(&pfull[s], (q / NS) & 1)) {
          if (lane == 0 && a.err) atomicExch(a.err, 1);
          break;
        }
        const float* red = part + ((size_t)s * ncs) * 128;
        // lane sums elements 4 lane .. 4 lane + 3 (row lane / 2, columns
        // 4 (lane & 1) .. 4 (lane & 1) + 3) over the row tile's stages and
        // chunks in order (unused chunks hold zeros)
        if (kb == 0) v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c2 = 0; c2 < ncs; ++c2) {
          const float4 e4 = reinterpret_cast<const float4*>(red + (size_t)c2 * 128)[lane];
          v.x += e4.x;
          v.y += e4.y;
          v.z += e4.z;
          v.w += e4.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&merged[s]);
        if (kb != nkb - 1) continue;
        float4 o = v;
        if (MODE == 1) {
          // columns 4..7 hold the d1 parts of x rows 0..3: add them to 0..3
          o.x += __shfl_xor_sync(0xffffffffu, o.x, 1);
          o.y += __shfl_xor_sync(0xffffffffu, o.y, 1);
          o.z += __shfl_xor_sync(0xffffffffu, o.z, 1);
          o.w += __shfl_xor_sync(0xffffffffu, o.w, 1);
        }
        const int grt = rt0 + i;
        pp = prob_of(grt, pp);
        const int rbase = (grt - tpref[pp]) * 16;
        const int r = lane >> 1, m0 = (lane & 1) * 4;
        if ((MODE == 2 || (lane & 1) == 0) && rbase + r < trows[pp]) {
          float* yp = ty[pp] + rbase + r;
          const int64_t ld = tldy[pp];
          if (m0 < a.m) gather_store(a, yp + (size_t)m0 * ld, o.x);
          if (m0 + 1 < a.m) gather_store(a, yp + (size_t)(m0 + 1) * ld, o.y);
          if (m0 + 2 < a.m) gather_store(a, yp + (size_t)(m0 + 2) * ld, o.z);
          if (m0 + 3 < a.m) gather_store(a, yp + (size_t)(m0 + 3) * ld, o.w);
        }
      }
      if (a.world > 1) __threadfence_system();
    }
  } else {
    // ---------------- consumers: quantise x of the k-split into two s8 digits
    griddep_wait();  // x may be written by the previous kernel in the stream
    const int kb0 = g0 * GS;
    const int f4 = (ng * GS) >> 2;
    constexpr int kUnroll = 4;
    const int nthr = kCons * 32;
    // x item (mrow, j): float4 f = threadIdx.x + nthr j of row mrow; fpt per
    // row, m fpt per thread, stepped as (mrow, j) without divisions.  A warp's
    // 32 lanes share (mrow, j) and cover 32 consecutive f (128 k): the row
    // maxima and the 64-k digit sums reduce per warp.  Float4 past the slice
    // load as zeros and store no digits.
    const int fpt = (f4 + nthr - 1) / nthr;
    const int nit = a.m * fpt;
    auto next_item = [&](int& mrow, int& j) {
      if (++j == fpt) {
        j = 0;
        ++mrow;
      }
    };
    auto load_x = [&](int mrow, int j) -> float4 {
      const int f = threadIdx.x + j * nthr;
      const int k = kb0 + 4 * f;
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
    // pass 1: max |x| per row.  The first kCache items of every thread are
    // loaded at once and kept in registers for pass 2; only a larger x is
    // read a second time.
    constexpr int kCache = MODE == 1 ? 8 : (KQG == 1 ? 0 : 4);
    float4 cache[kCache > 0 ? kCache : 1];
    {
      int mr = 0, jj = 0;
#pragma unroll
      for (int r = 0; r < kCache; ++r) {
        cache[r] = r < nit ? load_x(mr, jj) : make_float4(0.f, 0.f, 0.f, 0.f);
        next_item(mr, jj);
      }
    }
    auto row_max = [&](const float4& v, int mrow) {
      float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) atomicMax(&xmax[mrow], __float_as_uint(mx));
    };
    int mr1 = 0, jj1 = 0;   // the first item past the cached ones
#pragma unroll
    for (int r = 0; r < kCache; ++r) {
      if (r < nit) row_max(cache[r], mr1);
      next_item(mr1, jj1);
    }
    for (int i0 = kCache, mr = mr1, jj = jj1; i0 < nit; i0 += kUnroll) {
      float4 vv[kUnroll];
      int mq = mr, jq = jj;
#pragma unroll
      for (int r = 0; r < kUnroll; ++r) {
        vv[r] = i0 + r < nit ? load_x(mr, jj) : make_float4(0.f, 0.f, 0.f, 0.f);
        next_item(mr, jj);
      }
#pragma unroll
      for (int r = 0; r < kUnroll; ++r) {
        if (i0 + r >= nit) break;   // the same for every thread
        row_max(vv[r], mq);
        next_item(mq, jq);
      }
    }
    named_barrier(1, nthr);
    // pass 2: digits d0 = rint(x / s), d1 = rint((x / s - d0) * 256), packed
    // 4 k per word straight into the B fragment slots, and exact digit sums
    const int cols = MODE == 1 ? 2 * a.m : a.m;
    uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
    int inv_row = -1;
    float inv = 0.f;
    auto digits = [&](const float4& v, int mrow, int jidx) {
      const int f = threadIdx.x + jidx * nthr;
      if (mrow != inv_row) {        // 127 / max|x| once per row, not per item
        const float mxv = __uint_as_float(xmax[mrow]);
        inv = mxv > 0.f ? 127.0f / mxv : 0.f;
        inv_row = mrow;
      }
      const float xv[4] = {v.x, v.y, v.z, v.w};
      uint32_t w0 = 0, w1 = 0;
      int s0 = 0, s1 = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float q = xv[b] * inv;
        const int d0 = max(-127, min(127, __float2int_rn(q)));
        const int d1 = max(-127, min(127, __float2int_rn((q - (float)d0) * 256.0f)));
        w0 |= (uint32_t)(d0 & 0xFF) << (8 * b);
        w1 |= (uint32_t)(d1 & 0xFF) << (8 * b);
        s0 += d0;
        s1 += d1;
      }
      if (f < f4) {
        const int kt32 = f >> 3, j = f & 7;
        const int half = j >> 2, tt = j & 3;
        if (MODE == 1) {
          xw[(((size_t)kt32 * cols + mrow) * 4 + tt) * 2 + half] = w0;
          xw[(((size_t)kt32 * cols + a.m + mrow) * 4 + tt) * 2 + half] = w1;
        } else {
          xw[(((size_t)kt32 * cols + mrow) * 4 + tt) * 4 + half] = w0;
          xw[(((size_t)kt32 * cols + mrow) * 4 + tt) * 4 + 2 + half] = w1;
        }
      }
      // 64-k chunk sums over 16 lanes, then into the group's digit sums
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      }
      if ((lane & 15) == 0 && f < f4) {
        const int grp = (f >> 4) / KQG;
        atomicAdd(&sdi[grp * 16 + mrow], s0);
        atomicAdd(&sdi[grp * 16 + 8 + mrow], s1);
      }
    };
    {
      int mr = 0, jj = 0;
#pragma unroll
      for (int r = 0; r < kCache; ++r) {
        if (r < nit) digits(cache[r], mr, jj);
        next_item(mr, jj);
      }
      for (int i0 = kCache; i0 < nit; i0 += kUnroll) {
        float4 vv[kUnroll];
        int mq = mr, jq = jj;
#pragma unroll
        for (int r = 0; r < kUnroll; ++r) {
          vv[r] = i0 + r < nit ? load_x(mr, jj) : make_float4(0.f, 0.f, 0.f, 0.f);
          next_item(mr, jj);
        }
#pragma unroll
        for (int r = 0; r < kUnroll; ++r) {
          if (i0 + r >= nit) break;
          digits(vv[r], mq, jq);
          next_item(mq, jq);
        }
      }
    }
    named_barrier(1, nthr);
    griddep_launch_dependents();

    // lane (n = g, t) carries B column n
    const int mcol = MODE == 1 ? (g & 3) : g;
    const bool bvalid = mcol < a.m;
    const int ccol = MODE == 1 ? (g < 4 ? mcol : a.m + mcol) : mcol;
    const int sd_off = MODE == 1 ? (t < 2 ? 2 * t : 2 * t + 4) : 2 * t;
    const bool lane_has = MODE == 1 ? (t < 2) : true;
    // digit scale of this lane's result columns 2t, 2t+1
    float dsc[2], dsc2[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int m = MODE == 1 ? (t < 2 ? 2 * t + c : 2 * t - 4 + c) : 2 * t + c;
      const float mxv = m < a.m ? __uint_as_float(xmax[m]) : 0.f;
      const float sm = mxv / 127.0f;
      dsc[c] = (MODE == 1 && t >= 2) ? sm * (1.0f / 256.0f) : sm;
      dsc2[c] = sm * (1.0f / 256.0f);
    }
    // Lanes of columns past M read column 0's digits (d0 / d1 half) of the
    // same k32 tile: the warp's B load then touches the tile's digits only
    // (one shared-memory wavefront at M = 1, not two with a separate zero
    // pad).  Those MMA columns belong to x rows >= M, whose results are never
    // stored.
    const int ccol_rd = bvalid ? ccol : (MODE == 1 ? (g < 4 ? 0 : a.m) : 0);
    const uint2* xs2 = reinterpret_cast<const uint2*>(xs) + ccol_rd * 4 + t;
    const uint4* xs4 = reinterpret_cast<const uint4*>(xs) + ccol_rd * 4 + t;
    const int xstride = M1 ? 8 : cols * 4;

    // unit u = q ncs + c (stage q, chunk c) steps by kCons units without
    // divisions: s = q mod NS (ring slot), ph = (q / NS) & 1 (its phase),
    // kb = q mod nkb (k-block)
    int q = warp / ncs, c = warp - (warp / ncs) * ncs;
    int s = q % NS, ph = (q / NS) & 1, kb = q % nkb;
    auto advance = [&]() {
      c += kCons;
      while (c >= ncs) {
        c -= ncs;
        ++q;
        if (++s == NS) {
          s = 0;
          ph ^= 1;
        }
        if (++kb == nkb) kb = 0;
      }
    };
    for (int u = warp; u < nunits; u += kCons, advance()) {
      if (c >= nchunk) continue;  // the last k-split may have fewer chunks
      // chunks past the end of a short last k-block (direct mode) still take
      // part in the stage's barriers, with no groups (their partial is zero)
      const int cg0 = c * CG, ncg = max(0, min(CG, kb_groups(kb) - cg0));
      const int gb = kb * a.kbg + cg0;  // first group of the chunk in the k-split
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      if (!mbar_wait_t<kConsWait>(&full[s], ph)) {
        if (lane == 0 && a.err) atomicExch(a.err, 1);
      } else {
        // MODE 1 (group size >= 128) loads the chunk (weights and scales) into
        // registers and gives the ring slot back at once, so the producer
        // refills it while this warp computes; MODE 2 (two accumulator sets)
        // has no registers to spare and reads the slot in place.
        constexpr bool kStaged = MODE == 1 && KQG >= 2;
        const unsigned char* st = ring + (size_t)s * Ls.stage;
        const uint4* wq = reinterpret_cast<const uint4*>(st + (size_t)c * kChunkQ * 512) + lane;
        const float4* szp =
            reinterpret_cast<const float4*>(st + (size_t)a.kbg * KQG * 512 + (size_t)cg0 * 128) + g;
        uint4 wr[kStaged ? kChunkQ : 1];
        float4 sr[kStaged ? CG : 1];
        if (kStaged) {
#pragma unroll
          for (int gl = 0; gl < CG; ++gl) {
            if (gl < ncg) {
#pragma unroll
              for (int qq = 0; qq < KQG; ++qq) wr[gl * KQG + qq] = wq[(gl * KQG + qq) * 32];
              sr[gl] = szp[gl * 8];
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
        // one accumulator set per group of the chunk: CG independent MMA chains
        int acc[CG][4], acc2[MODE == 2 ? CG : 1][4];
#pragma unroll
        for (int gl = 0; gl < CG; ++gl)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[gl][q] = 0;
            acc2[MODE == 2 ? gl : 0][q] = 0;
          }
#pragma unroll
        for (int gl = 0; gl < CG; ++gl) {
          if (gl < ncg) {
#pragma unroll
            for (int qq = 0; qq < KQG; ++qq) {
              const int ql = gl * KQG + qq;                // quad within the chunk
              const uint4 w = kStaged ? wr[kStaged ? ql : 0] : wq[ql * 32];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                // low nibbles: rows g (a0, a2); high nibbles masked in
                // place: rows g + 8 (a1, a3) at 16 times their value, taken
                // out of the sums in the group epilogue (exact)
                const uint32_t wa = h == 0 ? w.x : w.z, wb = h == 0 ? w.y : w.w;
                const uint32_t a0 = wa & 0x0F0F0F0Fu, a1 = wa & 0xF0F0F0F0u;
                const uint32_t a2 = wb & 0x0F0F0F0Fu, a3 = wb & 0xF0F0F0F0u;
                const int kt32 = (gb * KQG + ql) * 2 + h;  // k32 tile within the k-split
                if (MODE == 1) {
                  const uint2 b = xs2[(size_t)kt32 * xstride];
                  mma_u8s8_16832(acc[gl], a0, a1, a2, a3, b.x, b.y);
                } else {
                  const uint4 b = xs4[(size_t)kt32 * xstride];
                  mma_u8s8_16832(acc[gl], a0, a1, a2, a3, b.x, b.y);
                  mma_u8s8_16832(acc2[MODE == 2 ? gl : 0], a0, a1, a2, a3, b.z, b.w);
                }
              }
            }
          }
        }
        // per-group epilogue: sum_k (n - zp) sc x = sc s (A - zp D); rows
        // g + 8 (accumulator elements 2, 3) carry 16 A: every term is a
        // multiple of 16, so the shift is exact
#pragma unroll
        for (int gl = 0; gl < CG; ++gl) {
          acc[gl][2] >>= 4;
          acc[gl][3] >>= 4;
          if (MODE == 2) {
            acc2[MODE == 2 ? gl : 0][2] >>= 4;
            acc2[MODE == 2 ? gl : 0][3] >>= 4;
          }
        }
#pragma unroll
        for (int gl = 0; gl < CG; ++gl) {
          if (gl < ncg) {
            const float4 sp = kStaged ? sr[kStaged ? gl : 0] : szp[gl * 8];
            const int* sd = sdi + (gb + gl) * 16;
            const float d0a = (float)sd[sd_off], d0b = (float)sd[sd_off + 1];
            if (MODE == 1 && M1) {
              // column 2t only (x row 0's d0 or d1 part); 2t + 1 stays zero
              tot[0] = fmaf(sp.x * dsc[0], fmaf(-sp.y, d0a, (float)acc[gl][0]), tot[0]);
              tot[2] = fmaf(sp.z * dsc[0], fmaf(-sp.w, d0a, (float)acc[gl][2]), tot[2]);
            } else if (MODE == 1) {
              tot[0] = fmaf(sp.x * dsc[0], fmaf(-sp.y, d0a, (float)acc[gl][0]), tot[0]);
              tot[1] = fmaf(sp.x * dsc[1], fmaf(-sp.y, d0b, (float)acc[gl][1]), tot[1]);
              tot[2] = fmaf(sp.z * dsc[0], fmaf(-sp.w, d0a, (float)acc[gl][2]), tot[2]);
              tot[3] = fmaf(sp.z * dsc[1], fmaf(-sp.w, d0b, (float)acc[gl][3]), tot[3]);
            } else {
              // the two digits' sums joined in integers first: 256 (A0 - zp D0)
              // + (A1 - zp D1) = (256 A0 + A1) - zp (256 D0 + D1), scaled by
              // s / 256 (|256 A0 + A1| < 2^26; the digit sums are exact)
              const int g2 = MODE == 2 ? gl : 0;
              const float da = (float)(sd[sd_off] * 256 + sd[8 + sd_off]);
              const float db = (float)(sd[sd_off + 1] * 256 + sd[8 + sd_off + 1]);
              tot[0] = fmaf(sp.x * dsc2[0], fmaf(-sp.y, da, (float)(acc[gl][0] * 256 + acc2[g2][0])), tot[0]);
              tot[1] = fmaf(sp.x * dsc2[1], fmaf(-sp.y, db, (float)(acc[gl][1] * 256 + acc2[g2][1])), tot[1]);
              tot[2] = fmaf(sp.z * dsc2[0], fmaf(-sp.w, da, (float)(acc[gl][2] * 256 + acc2[g2][2])), tot[2]);
              tot[3] = fmaf(sp.z * dsc2[1], fmaf(-sp.w, db, (float)(acc[gl][3] * 256 + acc2[g2][3])), tot[3]);
            }
          }
        }
        if (!kStaged) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
      }
      if (!direct) {
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
        continue;
      }
      // direct mode: hand the chunk's partial (all 8 MMA columns) to the
      // merger warp.  The stage's partial slots are reused by the next round
      // of the same stage: wait until the merger has read the previous one.
      float* red = part + ((size_t)s * ncs) * 128;
      if (q >= NS && !mbar_wait_t<kConsWait>(&merged[s], ph ^ 1)) {
        if (lane == 0 && a.err) atomicExch(a.err, 1);
        continue;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = g + ((q & 2) ? 8 : 0);
        const int mm = 2 * t + (q & 1);
        red[(size_t)c * 128 + r * 8 + mm] = tot[q];
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[s]);
    }
  }
  if (direct) {
    __syncthreads();  // the producer's drain completes before the CTA exits
    if (a.world > 1) gather_finish(a);
    return;
  }
  // sum the chunks of each row tile locally (chunk order) into the now idle
  // ring, then over the cluster's k-splits (rank order): deterministic.
  __syncthreads();
  float* sums = reinterpret_cast<float*>(ring);
  for (int e = threadIdx.x; e < nrt * 128; e += blockDim.x) {
    const int i = e >> 7, r = e & 127;
    float s = 0.f;
    for (int c = 0; c < nchunk; ++c) s += part[((size_t)(i * ncs + c)) * 128 + r];
    sums[e] = s;
  }
  cluster.sync();
  const int total = nrt * 128;
  for (int e = rank * blockDim.x + threadIdx.x; e < total; e += nsplit * blockDim.x) {
    const int mm = e & 7;
    const int grt = rt0 + (e >> 7);
    const int p = prob_of(grt, 0);
    const int row = (grt - tpref[p]) * 16 + ((e >> 3) & 15);
    if (mm >= a.m || row >= trows[p]) continue;
    float s = 0.0f;
    for (int r = 0; r < nsplit; ++r) s += cluster.map_shared_rank(sums, r)[e];
    gather_store(a, ty[p] + (size_t)mm * tldy[p] + row, s);
  }
  if (a.world > 1) __threadfence_system();
  cluster.sync();
  if (a.world > 1) gather_finish(a);
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
    w.tc_zp_ok = false;
    w.tc16_ok = false;
    if (rows * ngr > 0) {
      unsigned* stats = nullptr;
      NIMF_TRY(device_alloc((void**)&stats, 3 * sizeof(unsigned)));
      unsigned hs[3] = {0u, 0u, 0x7F800000u};
      cudaError_t e = cudaMemcpyAsync(stats, hs, sizeof(hs), cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) {
        const int64_t n = rows * ngr;
        q4g_zp_range<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, st>>>(scs, zps, ngr, rows, stats);
        e = cudaGetLastError();
      }
      if (e == cudaSuccess) e = cudaMemcpyAsync(hs, stats, sizeof(hs), cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      device_free(stats);
      NIMF_CUDA_TRY(e);
      w.tc_zp_ok = hs[0] == 0u;
      // fp16 tiles of (n - zp) * sc * 2^e: e puts the largest magnitude in
      // [2^13, 2^14); the smallest group scale must then stay >= 2^-10 so a
      // unit step of the nibbles keeps fp16's relative precision
      float wmax, smin;
      std::memcpy(&wmax, &hs[1], 4);
      std::memcpy(&smin, &hs[2], 4);
      if (std::isfinite(wmax)) {
        int ex = 0;
        if (wmax > 0.f) std::frexp(wmax, &ex);   // wmax = f 2^ex, f in [0.5, 1)
        const int e2 = wmax > 0.f ? 14 - ex : 0;
        w.tc16_exp = e2;
        w.tc16_ok = e2 > -100 && e2 < 100 &&
                    (!(smin < 3e38f) || std::ldexp((double)smin, e2) >= std::ldexp(1.0, -10));
      }
    }
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

// Stage counts must be multiples of both the stage->warp period and the
// issuer count, so that every ring slot keeps the same consumer warps and the
// same producer lane.
inline int lcm_int(int a, int b) {
  int x = a, y = b;
  while (y) {
    const int t2 = x % y;
    x = y;
    y = t2;
  }
  return a / x * b;
}

// Ring stages for stages of kbg groups and the given fixed shared memory, 0 if
// fewer than one period (and at least 4) fit.
inline int ring_stages(const SmemLayout& L0, int kqg, int kbg, bool direct) {
  if (L0.total >= kSmemBudget) return 0;
  const int ncs = (kbg + kChunkQ / kqg - 1) / (kChunkQ / kqg);
  int gcdv = kCons, bb = ncs;
  while (bb) {
    const int tmp = gcdv % bb;
    gcdv = bb;
    bb = tmp;
  }
  const int period = lcm_int(kCons / gcdv, kIssuers);
  const size_t per_stage = L0.stage + (direct ? (size_t)ncs * 512 : 0);
  int ns = (int)((kSmemBudget - L0.total) / per_stage);
  ns = std::min(ns, kStages) / period * period;
  return ns >= std::max(period, 4) ? ns : 0;
}

// Direct mode (no k-split): x of the whole K in shared memory, row tiles cut
// into k-blocks of about 36 KB of weights (18 or 9 KB when x leaves too little
// room for a ring of the larger ones).  False if it does not fit.
inline bool plan_direct(int mode, int kqg, int groups, int mc, int* kbg, int* nkb, int* ns) {
  const int cg = kChunkQ / kqg;
  for (int target = 36864; target >= 9216; target /= 2) {
    int kmax = (target / (kqg * 512 + 128)) / cg * cg;
    if (kmax < cg) kmax = cg;
    const int nb = (groups + kmax - 1) / kmax;
    const int per = (groups + nb - 1) / nb;
    const int kb = (per + cg - 1) / cg * cg;
    const SmemLayout L0 = q4g_smem_layout(mode, kqg, groups, kb, mc, 0, 1, true);
    const int n = ring_stages(L0, kqg, kb, true);
    if (n == 0) continue;
    *kbg = kb;
    *nkb = (groups + kb - 1) / kb;
    *ns = n;
    return true;
  }
  return false;
}

// A row-tile range of one weight inside a launch.
struct Piece {
  const Q4GWeight* w;
  int64_t rt_begin;
  int n_rt;
  float* y;       // y of the whole weight (row 0)
  int64_t ldy;
};

// Launches the GEMV over the given pieces (same K, group size and x).
template <int MODE, int KQG>
int launch_fast(const Piece* pcs, int npc, const float* x, int64_t ldx, int mc, int num_sms,
                cudaStream_t st, const GatherSpec* gsp) {
  Context* c = ctx();
  const Q4GWeight& w0 = *pcs[0].w;
  const int groups = (int)w0.groups;
  int n_rt = 0;
  for (int i = 0; i < npc; ++i) n_rt += pcs[i].n_rt;
  const int slots = num_sms * kCtasPerSm;
  auto kern = q4g_gemv_kernel<MODE, KQG, false>;
  auto kern1 = q4g_gemv_kernel<MODE, KQG, MODE == 1>;
  static int attr_dev = -1;
  static int max_active[kMaxSplits + 1];
  if (c && attr_dev != c->device) {
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBudget));
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBudget));
    // clusters of each size that fit on the GPU at once (GPC boundaries make
    // this less than SMs / size for sizes that do not divide a GPC)
    for (int cs = 1; cs <= kMaxSplits; ++cs) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3((unsigned)(cs * 64), 1, 1);
      q.blockDim = dim3((kCons + 2) * 32, 1, 1);
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
  // Pick direct mode or a k-split count (= cluster size) by the estimated
  // weight bytes of the busiest CTA (in units of 16 rows x one group).
  int best_s = -1, best_gps = 0, best_nclu = 1, best_ns = 0, best_kbg = 0, best_nkb = 1;
  double best_score = 1e30;
  {
    int kbg, nkb, ns;
    if (plan_direct(MODE, KQG, groups, mc, &kbg, &nkb, &ns)) {
      best_s = 1;
      best_gps = groups;
      best_nclu = std::max(1, std::min(n_rt, slots));
      best_ns = ns;
      best_kbg = kbg;
      best_nkb = nkb;
      best_score = (double)((n_rt + best_nclu - 1) / best_nclu) * groups;
    }
  }
  for (int s = 2; s <= kMaxSplits; ++s) {
#ifdef NIMF_Q4G_FORCE_SPLITS
    if (s != NIMF_Q4G_FORCE_SPLITS) continue;
#endif
    const int gps = (groups + s - 1) / s;
    const int ss = (groups + gps - 1) / gps;
    if (ss != s) continue;
    const int act = (c && attr_dev == c->device) ? max_active[ss] : slots / ss;
    const int nclu = std::max(1, std::min(n_rt, act));
    const int tchunk = (n_rt + nclu - 1) / nclu;
    if (tchunk > kMaxTilesPerCluster) continue;
    const SmemLayout L0 = q4g_smem_layout(MODE, KQG, gps, gps, mc, 0, tchunk, false);
    const int ns = ring_stages(L0, KQG, gps, false);
    if (ns == 0 || (size_t)ns * L0.stage < (size_t)tchunk * 512) continue;
    // split mode pays for its cluster reduction: measured on the 7B decode
    // stack, a 25% penalty picks the faster mode for up to 4 rows of x, none
    // for up to 8 (batch 8: 3,255 vs 2,872 tok/s; batch 1 keeps 735)
    const double score = (MODE == 1 ? 1.25 : 1.0) * tchunk * gps;
    if (score < best_score - 1e-9) {
      best_score = score;
      best_s = ss;
      best_gps = gps;
      best_nclu = nclu;
      best_ns = ns;
      best_kbg = gps;
      best_nkb = 1;
    }
  }
  if (best_s < 0)
    return set_error(NIMF_ERR_UNSUPPORTED, "q4g gemv: K=%lld, M=%d (%d row tiles) does not fit",
                     (long long)w0.k, mc, n_rt);
  const int s = best_s, gps = best_gps, n_clusters = best_nclu, ns = best_ns;
  const int tchunk = (n_rt + n_clusters - 1) / n_clusters;
  const SmemLayout L = q4g_smem_layout(MODE, KQG, gps, best_kbg, mc, ns, tchunk, s == 1);

  GemvArgs a;
  a.nprob = npc;
  a.rt_prefix[0] = 0;
  for (int i = 0; i < npc; ++i) {
    const Q4GWeight& w = *pcs[i].w;
    a.prob[i].frag = (const uint4*)w.frag + (size_t)pcs[i].rt_begin * w.kq_total * 32;
    a.prob[i].sz = (const float4*)w.sz + (size_t)pcs[i].rt_begin * w.groups * 8;
    a.prob[i].y = pcs[i].y + pcs[i].rt_begin * 16;
    a.prob[i].ldy = pcs[i].ldy;
    a.prob[i].rows = (int)std::min<int64_t>((int64_t)pcs[i].n_rt * 16, w.rows - pcs[i].rt_begin * 16);
    a.rt_prefix[i + 1] = a.rt_prefix[i] + pcs[i].n_rt;
  }
  a.x = x;
  a.err = c ? c->dev_err : nullptr;
  a.ldx = ldx;
  a.m = mc;
  a.k = (int)w0.k;
  a.n_rt = n_rt;
  a.kq_total = (int)w0.kq_total;
  a.groups = groups;
  a.gps = gps;
  a.kbg = best_kbg;
  a.nkb = best_nkb;
  a.n_clusters = n_clusters;
  a.tchunk = tchunk;
  a.ns = ns;
  a.vec4 = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 4 == 0);
  a.world = gsp ? gsp->world : 1;
  for (int q = 0; q < kCommMaxRanks; ++q) a.peer_off[q] = gsp ? gsp->peer_off[q] : 0;
  a.gctl = gsp ? gsp->ctl : nullptr;
  a.wait_ns = gsp ? gsp->wait_ns : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_clusters * s), 1, 1);
  cfg.blockDim = dim3((kCons + 2) * 32, 1, 1);
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
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, (MODE == 1 && mc == 1) ? kern1 : kern, a));
  return NIMF_OK;
}

// Splits the concatenated row tiles of the weights into launches of at most
// kMaxProblems pieces and a bounded number of row tiles per cluster.
template <int MODE, int KQG>
int launch_rows(const Q4GWeight* const* ws, float* const* ys, int count, const float* x,
                int64_t ldx, int mc, int64_t m0, int num_sms, cudaStream_t st,
                const GatherSpec* gsp = nullptr, const int64_t* ldys = nullptr) {
  // Direct mode (no k-split) streams any number of row tiles; split mode keeps
  // at most kMaxTilesPerCluster partial row tiles per cluster in shared memory.
  int kbg, nkb, nsd;
  const bool direct_fits = plan_direct(MODE, KQG, (int)ws[0]->groups, mc, &kbg, &nkb, &nsd);
  const int64_t cap = direct_fits ? ((int64_t)1 << 40)
                                  : (int64_t)kMaxTilesPerCluster *
                                        std::max(1, num_sms * kCtasPerSm / kMaxSplits);
  if (gsp && (!direct_fits || count > kMaxProblems))
    return set_error(NIMF_ERR_UNSUPPORTED,
                     "gathering GEMV: %d weights of K=%lld at %d rows of x need more than one launch",
                     count, (long long)ws[0]->k, mc);
  Piece pcs[kMaxProblems];
  int npc = 0;
  int64_t in_launch = 0;
  for (int i = 0; i < count; ++i) {
    const Q4GWeight& w = *ws[i];
    for (int64_t r0 = 0; r0 < w.n_rt;) {
      const int64_t n = std::min<int64_t>(w.n_rt - r0, cap - in_launch);
      pcs[npc].w = &w;
      pcs[npc].rt_begin = r0;
      pcs[npc].n_rt = (int)n;
      pcs[npc].y = ys[i] + m0 * (ldys ? ldys[i] : w.rows);
      pcs[npc].ldy = ldys ? ldys[i] : w.rows;
      ++npc;
      in_launch += n;
      r0 += n;
      if (npc == kMaxProblems || in_launch == cap) {
        NIMF_TRY((launch_fast<MODE, KQG>(pcs, npc, x, ldx, mc, num_sms, st, gsp)));
        npc = 0;
        in_launch = 0;
      }
    }
  }
  if (npc > 0) NIMF_TRY((launch_fast<MODE, KQG>(pcs, npc, x, ldx, mc, num_sms, st, gsp)));
  return NIMF_OK;
}

template <int MODE>
int launch_mode(const Q4GWeight* const* ws, float* const* ys, int count, const float* x,
                int64_t ldx, int mc, int64_t m0, int num_sms, cudaStream_t st,
                const GatherSpec* gsp = nullptr, const int64_t* ldys = nullptr) {
  switch (ws[0]->gs) {
    case 64: return launch_rows<MODE, 1>(ws, ys, count, x, ldx, mc, m0, num_sms, st, gsp, ldys);
    case 128: return launch_rows<MODE, 2>(ws, ys, count, x, ldx, mc, m0, num_sms, st, gsp, ldys);
    case 256: return launch_rows<MODE, 4>(ws, ys, count, x, ldx, mc, m0, num_sms, st, gsp, ldys);
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "q4g fast path: group size %lld", (long long)ws[0]->gs);
}

}  // namespace

// Rows of x above which the tensor-core GEMM replaces the GEMV.
constexpr int64_t kTcMinRows = 16;
int g_q4_prefill_mode = NIMF_Q4_PREFILL_AUTO;

int q4g_gemv_group(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                   float* const* ys, cudaStream_t st) {
  Context* c = ctx();
  const int num_sms = c ? c->num_sms : 148;
  if (m <= 0 || count <= 0) return NIMF_OK;
  const Q4GWeight& w0 = *ws[0];
  for (int i = 1; i < count; ++i)
    if (ws[i]->k != w0.k || ws[i]->gs != w0.gs || ws[i]->fast != w0.fast)
      return set_error(NIMF_ERR_SHAPE, "grouped GEMV: weights must share K and group size");
  if (w0.k == 0) {
    for (int i = 0; i < count; ++i)
      if (ws[i]->rows > 0)
        NIMF_CUDA_TRY(cudaMemsetAsync(ys[i], 0, (size_t)(m * ws[i]->rows) * sizeof(float), st));
    return NIMF_OK;
  }
  // prefill-sized x: one tensor-core GEMM per weight (the weights are read
  // once per 128 rows of x instead of once per 8)
  if (m > kTcMinRows) {
    bool tc = true;
    int64_t gs0 = 0;
    for (int i = 0; i < count; ++i) {
      if (ws[i]->rows == 0) continue;
      if (gs0 == 0) gs0 = ws[i]->gs;
      tc = tc && q4g_tc_supported(*ws[i]) && ws[i]->gs == gs0;
    }
    // the fp16-tile GEMM when every weight fits fp16 tiles (and the mode
    // allows it), else the exact-nibble GEMM
    bool t16 = g_q4_prefill_mode != NIMF_Q4_PREFILL_EXACT;
    for (int i = 0; i < count && t16; ++i)
      if (ws[i]->rows > 0) t16 = q4g_tc16_supported(*ws[i]) && ws[i]->gs == gs0;
    if (t16 || tc) {
      // weights with rows share one x preparation and one launch per 4
      const Q4GWeight* tw[64];
      float* ty[64];
      int n = 0;
      auto run = [&](int cnt) {
        return t16 ? q4g_gemm_tc16_group(tw, cnt, x, m, ty, st) : q4g_gemm_tc_group(tw, cnt, x, m, ty, st);
      };
      for (int i = 0; i < count; ++i) {
        if (ws[i]->rows <= 0) continue;
        tw[n] = ws[i];
        ty[n] = ys[i];
        if (++n == 64) {
          NIMF_TRY(run(n));
          n = 0;
        }
      }
      if (n > 0) NIMF_TRY(run(n));
      return NIMF_OK;
    }
  }
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    const float* xc = x + m0 * w0.k;
    if (w0.fast) {
      if (mc <= 4) NIMF_TRY(launch_mode<1>(ws, ys, count, xc, w0.k, mc, m0, num_sms, st));
      else NIMF_TRY(launch_mode<2>(ws, ys, count, xc, w0.k, mc, m0, num_sms, st));
    } else {
      for (int i = 0; i < count; ++i) {
        const Q4GWeight& w = *ws[i];
        if (w.rows == 0) continue;
        const int block = 256;
        const int64_t want = (w.rows * 32 + block - 1) / block;
        const unsigned grid = (unsigned)std::min<int64_t>(want, (int64_t)num_sms * 16);
        q4g_gemv_generic<<<grid, block, 0, st>>>((const uint8_t*)w.raw, (const float*)w.scales,
                                                 (const float*)w.zeros, w.rows, w.k, w.gs, w.ngr,
                                                 xc, w.k, mc, ys[i] + m0 * w.rows, w.rows);
        NIMF_CUDA_TRY(cudaGetLastError());
      }
    }
  }
  return NIMF_OK;
}

int q4g_gemv_group_gather(const Q4GWeight* const* ws, int count, const float* x, int64_t m,
                          float* const* ys, const int64_t* ldys, const GatherSpec& g,
                          cudaStream_t st) {
  Context* c = ctx();
  const int num_sms = c ? c->num_sms : 148;
  if (m <= 0 || m > 8 || count <= 0)
    return set_error(NIMF_ERR_UNSUPPORTED, "gathering GEMV: %lld rows of x (1 .. 8)", (long long)m);
  const Q4GWeight& w0 = *ws[0];
  for (int i = 0; i < count; ++i)
    if (ws[i]->k != w0.k || ws[i]->gs != w0.gs || !ws[i]->fast || ws[i]->k == 0)
      return set_error(NIMF_ERR_UNSUPPORTED,
                       "gathering GEMV: weights must share K > 0 and a group size of 64, 128 or 256");
  if (m <= 4) return launch_mode<1>(ws, ys, count, x, w0.k, (int)m, 0, num_sms, st, &g, ldys);
  return launch_mode<2>(ws, ys, count, x, w0.k, (int)m, 0, num_sms, st, &g, ldys);
}

int q4g_gemv(const Q4GWeight& w, const float* x, int64_t m, float* y, cudaStream_t st) {
  if (w.rows <= 0) return NIMF_OK;
  const Q4GWeight* ws[1] = {&w};
  float* ys[1] = {y};
  return q4g_gemv_group(ws, 1, x, m, ys, st);
}

}  // namespace nimf
