// decode.cu -- one whole decode step of a Llama-style stack with int4
// group-128 weights (LlamaModelL.forwardStep with isPrefill = false,
// nim_inference.nim:887-921, followed by the temperature <= 0 branch of
// sampleTopP, :1019-1036) as ONE persistent launch.
//
// Why one launch: a decode step at batch 1 is 129 weight-streaming GEMVs
// (3.7 GB at the 7B shape) separated by small glue steps.  Launched one by one,
// every GEMV pays a ramp (an empty weight ring at launch), a drain (the
// slowest CTA) and the launch gap, about 6 us each against 4 us of streaming
// for a 28 MB projection.  Here the producer warp of every CTA streams the
// weights of the whole step back to back: the weights do not depend on the
// activations, so the ring keeps filling with the next projection's weights
// while the grid waits for the previous projection's outputs.
//
// Grid: one CTA per SM (cooperative launch, so every CTA is resident), 18
// warps: a producer (bulk copies of the packed weights into a 4-stage
// mbarrier ring of 36 KB stages), 16 consumer warps and a merge warp, as in
// the standalone GEMV (q4g.cu).  The step is a table of stages:
//   per layer  S1 q/k/v GEMV     x = RMSNorm(h + down_prev) (layer 0: the
//                                embedding row), the sum kept as the residual
//              S2 attention      (head, position split) units: RoPE on q and
//                                the new k, KV append, scores, softmax
//                                partials (max, sum, unnormalised P.V)
//              S3 o GEMV         x = the split partials combined
//              S4 gate/up GEMV   x = RMSNorm(residual + o), sum kept; gate
//                                and up row tiles interleave, so each merge
//                                warp stores SwiGLU(gate, up) of its rows
//              S5 down GEMV      x = that SwiGLU output
//   then       lm_head GEMV      x = RMSNorm(residual + down) with the final
//                                norm; the merge warps keep the repetition-
//                                penalised argmax of their rows, and CTA 0
//                                picks the next token from the CTA results.
// Stage s may start (its consumers compute x) only when every CTA has
// finished stage s-1: a grid barrier on a per-stage arrival counter, waited
// on by one consumer thread with ld.acquire and a %globaltimer bound.  Every
// x is computed redundantly by every CTA from the previous stage's outputs
// (read through L2 with ld.global.cg, since they were written in this launch),
// quantised into two signed 8-bit digits per element with one scale per row
// (max|x| / 127), and multiplied on the s8 tensor cores against the nibbles,
// as in q4g.cu: per group sc s (A - zp D) with A the exact MMA sum, D the exact
// digit sum.  The glue arithmetic follows glue.cu (same roundings).
//
// Every wait is bounded: mbarrier waits as in the GEMV, grid barriers by the
// plan's wait bound; an expired wait sets the context's host-mapped error word
// (nimf_sync then reports NIMF_ERR_TIMEOUT) and a device-side abort flag that
// makes later waits of the plan give up at once.  No TMA multicast, no
// cluster: plain bulk copies into this CTA's shared memory.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr int kCons = 16;                        // consumer warps
constexpr int kConsThreads = kCons * 32;         // 512
constexpr int kThreads = (kCons + 2) * 32;       // + producer + merge warp
constexpr int kKQG = 2;                          // 64-k quads per group of 128
constexpr int kGS = 128;
constexpr int kChunkQ = 8;                       // quads per consumer chunk (512 k)
constexpr int kCG = kChunkQ / kKQG;              // groups per chunk
constexpr int kKbg = 32;                         // groups per ring stage (4096 k)
constexpr int kNcs = kKbg / kCG;                 // chunks per ring stage
constexpr int kStageW = kKbg * kKQG * 512;       // weight bytes of a ring stage
constexpr int kStageBytes = kStageW + kKbg * 128;  // + the scale/zero float4s
constexpr int kNS = 4;                           // ring stages
constexpr int kIssuers = 4;                      // producer lanes (lane l issues stages q = l mod 4)
constexpr int kMaxK = 14336;                     // largest K of a stage
constexpr int kMaxGroups = kMaxK / kGS;
constexpr int kNV = (kMaxK / 4 + kConsThreads - 1) / kConsThreads;  // float4 of x per thread
constexpr int kPB = 4;                           // prologue slots whose loads are issued together
constexpr int kMaxHeads = 64;
constexpr int kMaxSplit = 8;
constexpr int kMaxProb = 3;
constexpr int kMaxRanks = kCommMaxRanks;         // GPUs of a sharded plan
constexpr int kMaxRecent = 256;
constexpr int kMaxPs = 4096;                     // positions of one attention unit
constexpr int kMaxHeadDim = 256;
constexpr int kBarCons = 1;                      // named barrier of the consumer warps
// ring slot q % kNS always serves the same 8 consumer warps and producer lane
static_assert(kNS == kIssuers && (kNS * kNcs) % kCons == 0, "ring period: producer lane l owns slot l");

// ---- shared memory
constexpr int kOffBar = 0;                        // full, empty, merged, pfull [kNS] uint64
constexpr int kOffRed = 128;                      // float[32] reduction scratch
constexpr int kOffMisc = 288;                     // xmax, counters (256 .. 287 unused)
constexpr int kOffComb = 384;                     // combine weights [kMaxHeads][kMaxSplit]
constexpr int kOffCombML = kOffComb + kMaxHeads * kMaxSplit * 4;   // [kMaxHeads][2]
constexpr int kOffRecent = kOffCombML + kMaxHeads * 2 * 4;         // int[kMaxRecent]
constexpr int kOffMark = kOffRecent + kMaxRecent * 4;              // uint32[128]: recent rows of this CTA
constexpr int kOffRing = 4608;
constexpr int kOffXs = kOffRing + kNS * kStageBytes;
constexpr int kXsBytes = kMaxK / 32 * 64;         // [k32][2 digits][4 lanes][2 words]
constexpr int kOffSdi = kOffXs + kXsBytes;
constexpr int kSdiBytes = kMaxGroups * 16 * 4;
constexpr int kOffPart = kOffSdi + kSdiBytes;
constexpr int kPartBytes = kNS * kNcs * 128 * 4;
constexpr int kWbufK = 4096;                     // RMSNorm weights staged in shared memory up to this K
constexpr int kOffWbuf = kOffPart + kPartBytes;
constexpr int kSmemBytes = kOffWbuf + kWbufK * 4;
// attention scratch reuses xs + sdi (the digits are dead during attention)
constexpr int kAttnBytes = (3 * kMaxHeadDim + kMaxPs) * 4 + kCons * kMaxHeadDim * 4;
static_assert(kAttnBytes <= kXsBytes + kSdiBytes, "attention scratch");
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kOffRing >= kOffMark + 128 * 4, "head layout");

enum { ST_GEMV = 0, ST_ATTN = 1 };

// The fields of a GEMV stage the consumers need, read before the stage's
// grid barrier so that their global loads are not on the critical path.
struct ProDesc {
  int k, groups, pro, nkb, n_rt, pair;
  const float* a;
  const float* b;
  const float* w;
  float* res_out;
  bool wstaged;             // w is in shared memory (kOffWbuf)
};
enum { PRO_EMB_RMS = 0, PRO_ADD_RMS = 1, PRO_COMBINE = 2, PRO_PLAIN = 3 };

struct DecStage {
  int kind, pro;
  int k, groups, nkb, n_rt, nprob, greedy;
  // pair = 1: two problems of equal rows (gate, up) whose row tiles
  // interleave (tile 2 t = gate tile t, 2 t + 1 = up tile t) and are split
  // over the CTAs in whole pairs, so that one merge warp holds both halves of
  // its rows and stores SwiGLU(gate, up) into y[0]
  int pair;
  int rt_prefix[kMaxProb + 1];
  int rows[kMaxProb];
  int row0[kMaxProb];       // first output row of this rank's shard (0 unsharded)
  const uint4* frag[kMaxProb];
  const float4* sz[kMaxProb];
  float* y[kMaxProb];       // nullptr: the launch's logits buffer
  const float* a;           // prologue inputs
  const float* b;
  const float* w;           // norm weight
  float* res_out;           // residual written by CTA 0
  float* kc;                // attention: this layer's caches
  float* vc;
};

struct DecArgs {
  const DecStage* stages;
  int nstages;
  int D, H, HKV, HD, max_seq, nsplit, vocab;
  float eps, scale, penalty;
  const float* emb;         // [vocab][D]
  const float* cos_t;       // [max_seq][HD/2]
  const float* sin_t;
  const float* q;           // S1 outputs, read by S2
  const float* k;
  const float* v;
  float* part_o;            // [H][nsplit][HD]
  float* part_ml;           // [H][nsplit][2]
  float* logits;            // [vocab]
  const int* tok_in;
  int* tok_out;             // nullptr: no token choice
  int* pos;
  int advance_pos;
  const int* recent;
  int n_recent;
  int* cand;                // [grid][4] per-CTA argmax (value bits, index, NaN-at-0, valid)
  unsigned* ctl;            // [0] launches, [1] abort, [2 + s] arrivals at stage s
  int* err;                 // host-mapped error word
  unsigned long long wait_ns;
  // sharded plans (world > 1): every stage output, attention partial and
  // argmax candidate is stored into every rank's scratch (rank q's copy of a
  // local scratch address p is p + peer_off[q] bytes, through CUDA IPC), and
  // the last CTA of a rank to finish stage s adds 1 to gctl[s] of every rank.
  int world, rank;
  int h0, hk0, hloc;        // first query / KV head and query heads of this rank
  long long peer_off[kMaxRanks];
  unsigned* gctl;
  int l2_ahead;             // producer items (per lane) prefetched into L2 ahead of the ring
  // optional stage timeline of CTA tl_cta (%globaltimer ns), [stage][3]:
  // consumers past the stage's grid barrier, prologue done, merge warp's
  // arrival (attention stages: units done); nullptr: not recorded
  unsigned long long* timeline;
  int tl_cta;
};

// per stage: barrier, prologue done, arrival, x loaded, sum, max, first item,
// last chunk of consumer warp 0, merge stores done; warp 0's first chunk:
// computed, partial slot free, partial handed over
constexpr int kTlMarks = 12;
__device__ __forceinline__ void tl_mark(const DecArgs& a, int s, int what) {
  if (a.timeline != nullptr && (int)blockIdx.x == a.tl_cta) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.timeline[(size_t)s * kTlMarks + what] = t;
  }
}

template <typename T>
__device__ __forceinline__ T* at_rank(const DecArgs& a, T* p, int q) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + a.peer_off[q]);
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float2 ldcg2(const float* p) {
  return __ldcg(reinterpret_cast<const float2*>(p));
}
__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Waits until *p >= target (wrap-safe); false if the bound ran out or the plan
// was aborted by an earlier expiry.
template <bool SYS = false>
__device__ bool wait_count(const DecArgs& a, const unsigned* p, unsigned target) {
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    if ((int)((SYS ? ld_acquire_sys(p) : ld_acquire(p)) - target) >= 0) {
      __threadfence();
      return true;
    }
    if ((it & 63u) == 63u) {
      if (*(volatile unsigned*)(a.ctl + 1) != 0u) return false;
      if (gtimer() - t0 > a.wait_ns) {
        atomicExch(a.ctl + 1, 1u);
        if (a.err) atomicExch(a.err, 3);
        return false;
      }
    }
    __nanosleep(20);
  }
}

// Bounded mbarrier wait of the ring (HINT as mbar_wait_t): gives up when the
// plan's wait bound runs out or an earlier wait of the launch gave up, so one
// failure cannot chain into many full-length waits.
template <int HINT>
__device__ bool dwait(const DecArgs& a, uint64_t* m, uint32_t parity) {
  unsigned long long t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (HINT > 0) {
      if (mbar_try_wait_sleep(m, parity, (uint32_t)HINT)) return true;
    } else {
      if (mbar_test_wait(m, parity)) return true;
      __nanosleep((unsigned)(-HINT));
    }
    if ((i & 255u) == 255u) {
      if (*(volatile unsigned*)(a.ctl + 1) != 0u) return false;
      const unsigned long long t = gtimer();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > a.wait_ns) {
        atomicExch(a.ctl + 1, 1u);
        return false;
      }
    }
  }
}

// Arrival of this CTA at the end of stage s.  One GPU: a count per CTA on the
// stage counter.  Sharded: the CTA's stores to the ranks' scratch were fenced
// at system scope by the threads that made them; the rank's last CTA at
// stage s (its local count reaches `target`) then adds 1 to gctl[s] of every
// rank.
__device__ __forceinline__ void arrive(const DecArgs& a, int s, unsigned target) {
  __threadfence();
  if (a.world == 1) {
    atomicAdd(a.ctl + 2 + s, 1u);
    return;
  }
  const unsigned old = atomicAdd(a.ctl + 2 + s, 1u);
  if (old == target - 1u) {
    __threadfence_system();
    for (int q = 0; q < a.world; ++q) red_release_sys(at_rank(a, a.gctl + s, q), 1u);
  }
}

// The grid barrier before stage s + 1: every CTA of every rank has finished
// stage s.
__device__ __forceinline__ bool stage_wait(const DecArgs& a, int s, unsigned target,
                                           unsigned gtarget) {
  if (a.world == 1) return wait_count(a, a.ctl + 2 + s, target);
  return wait_count<true>(a, a.gctl + s, gtarget);
}

__device__ __forceinline__ void row_split(int n_rt, int cid, int G, int* rt0, int* nrt) {
  const int base = n_rt / G, rem = n_rt % G;
  *rt0 = cid * base + min(cid, rem);
  *nrt = base + (cid < rem ? 1 : 0);
}
// The row tiles of a GEMV stage for CTA cid (whole gate/up pairs when paired).
__device__ __forceinline__ void stage_rows(int n_rt, int pair, int cid, int G, int* rt0, int* nrt) {
  if (!pair) {
    row_split(n_rt, cid, G, rt0, nrt);
    return;
  }
  row_split(n_rt >> 1, cid, G, rt0, nrt);
  *rt0 *= 2;
  *nrt *= 2;
}

// v[i] for a small register array and a runtime i (selects, no local memory)
template <typename T, int N>
__device__ __forceinline__ T pick(const T (&v)[N], int i) {
  T r = v[0];
#pragma unroll
  for (int j = 1; j < N; ++j)
    if (i == j) r = v[j];
  return r;
}

__device__ __forceinline__ int prob_of(const DecStage& st, int grt) {
  int p = 0;
  while (p + 1 < st.nprob && grt >= st.rt_prefix[p + 1]) ++p;
  return p;
}

// Global sources and sizes of item i (row tile i / nkb, k-block i % nkb) of
// GEMV stage st for the CTA whose row tiles start at rt0.
struct ItemSrc {
  const uint4* w;
  const float4* z;
  uint32_t wb, zb;
};
__device__ __forceinline__ ItemSrc item_src(const DecStage& st, int rt0, int i) {
  const int nkb = __ldg(&st.nkb), groups = __ldg(&st.groups);
  const int rti = i / nkb, kb = i - rti * nkb;
  const int grt = rt0 + rti;
  const bool pair = __ldg(&st.pair) != 0;
  const int p = pair ? (grt & 1) : prob_of(st, grt);
  const int rt = pair ? (grt >> 1) : grt - __ldg(&st.rt_prefix[p]);
  const int ngk = min(kKbg, groups - kb * kKbg);
  const uint4* fr = reinterpret_cast<const uint4*>(__ldg(reinterpret_cast<const unsigned long long*>(&st.frag[p])));
  const float4* sz = reinterpret_cast<const float4*>(__ldg(reinterpret_cast<const unsigned long long*>(&st.sz[p])));
  ItemSrc r;
  r.w = fr + ((size_t)rt * groups * kKQG + (size_t)kb * kKbg * kKQG) * 32;
  r.z = sz + ((size_t)rt * groups + (size_t)kb * kKbg) * 8;
  r.wb = (uint32_t)ngk * kKQG * 512u;
  r.zb = (uint32_t)ngk * 128u;
  return r;
}

// A producer lane's position in its item sequence (global items q = lane
// mod kIssuers over every GEMV stage of the step, in order), used to look
// ahead for L2 prefetches.
struct LaneCursor {
  int s, q0, nstg, rt0, i;
  bool valid;
};
// Moves to GEMV stage s or the next one after it, starting at global item
// q0; the lane's first item there is `want` (a global index >= q0).
__device__ void cursor_seek(const DecArgs& a, LaneCursor& c, int s, int q0, int want, int cid, int G) {
  for (; s < a.nstages; ++s) {
    const DecStage& st = a.stages[s];
    if (__ldg(&st.kind) != ST_GEMV) continue;
    int nrt;
    stage_rows(__ldg(&st.n_rt), __ldg(&st.pair), cid, G, &c.rt0, &nrt);
    const int nstg = nrt * __ldg(&st.nkb);
    if (want < q0 + nstg) {
      c.s = s;
      c.q0 = q0;
      c.nstg = nstg;
      c.i = want - q0;
      c.valid = true;
      return;
    }
    q0 += nstg;
  }
  c.valid = false;
}
__device__ __forceinline__ void cursor_next(const DecArgs& a, LaneCursor& c, int cid, int G) {
  if (!c.valid) return;
  const int want = c.q0 + c.i + kIssuers;
  if (want < c.q0 + c.nstg) {
    c.i = want - c.q0;
    return;
  }
  cursor_seek(a, c, c.s + 1, c.q0 + c.nstg, want, cid, G);
}

// consumer-wide reductions (512 threads, named barrier 1)
__device__ __forceinline__ float cons_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  named_barrier(kBarCons, kConsThreads);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  named_barrier(kBarCons, kConsThreads);
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kCons; ++i) t += red[i];
  return t;
}
__device__ __forceinline__ float cons_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  named_barrier(kBarCons, kConsThreads);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  named_barrier(kBarCons, kConsThreads);
  float t = red[0];
#pragma unroll
  for (int i = 1; i < kCons; ++i) t = fmaxf(t, red[i]);
  return t;
}

// ------------------------------------------------------------ x prologue
// Computes x of a GEMV stage (K values, float4 f = tid + 512 j, j < NV),
// writes the residual (CTA 0), then the digits into xs, the group digit sums
// into sdi and max|x| into *xmax.  NV is the smallest slot count that holds K:
// x lives in registers across the two consumer-wide reductions, and slots
// sized for the largest K would not fit the 96-register budget.
template <int NV>
__device__ void prologue_nv(const DecArgs& a, const ProDesc& st, int cid, int tok, unsigned char* smem,
                            int stage) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* xmaxp = reinterpret_cast<float*>(smem + kOffMisc);
  int* sdi = reinterpret_cast<int*>(smem + kOffSdi);
  uint32_t* xw = reinterpret_cast<uint32_t*>(smem + kOffXs);
  const int K = st.k;
  const int f4 = K >> 2;
  for (int i = tid; i < st.groups * 16; i += kConsThreads) sdi[i] = 0;
  float4 v[NV];
  // Every global load of a slot set is issued before any of its values is
  // used (no fence, shuffle or data-dependent branch in between), so a
  // prologue costs about one L2 round trip per phase rather than one per
  // load.  Slots j with 512 j >= K / 4 are empty for the whole warp.
  const int warp = tid >> 5;
  if (NV <= 2 && st.pro == PRO_COMBINE && a.HD == 128) {
    // Head dimension 128, up to 32 heads: slot j of warp w is all of head
    // w + 16 j (lane l
    // holds d = 4 l .. 4 l + 3), so one warp combines one head per slot with
    // shuffles, and every load of a slot set (lane j's (m_j, l_j), the
    // lane's d of the first four splits) is issued before any is used.
    // Arithmetic as below: M = max_j m_j, L = sum over live j (l_j > 0) of
    // e^(m_j - M) l_j in split order, o = sum over live j of e^(m_j - M) o_j
    // in split order, x = o / L.
    const int ns = a.nsplit;
    float2 ml[NV];
    float4 o[NV][4];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int f = tid + j * kConsThreads;
      const bool in = (f & ~31) < f4;                  // warp-uniform
      const int h = f >> 5;
      ml[j] = (in && lane < ns) ? ldcg2(a.part_ml + ((size_t)h * ns + lane) * 2) : make_float2(-INFINITY, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[j][q] = (in && q < ns) ? ldcg4(a.part_o + ((size_t)h * ns + q) * 128 + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int f = tid + j * kConsThreads;
      if ((f & ~31) >= f4) {
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      const int h = f >> 5;
      float M = ml[j].x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const bool live = lane < ns && ml[j].y > 0.f;
      const float e = live ? expf(__fsub_rn(ml[j].x, M)) : 0.f;
      const float el = live ? __fmul_rn(e, ml[j].y) : 0.f;
      const unsigned mask = __ballot_sync(0xffffffffu, live);
      float L = 0.f;
      for (int sp = 0; sp < ns; ++sp) {
        const float t = __shfl_sync(0xffffffffu, el, sp);
        if ((mask >> sp) & 1u) L = __fadd_rn(L, t);
      }
      float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
      for (int s0 = 0; s0 < ns; s0 += 4) {
        float4 ob[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          ob[q] = s0 == 0 ? o[j][q]
                          : (s0 + q < ns ? ldcg4(a.part_o + ((size_t)h * ns + s0 + q) * 128 + 4 * lane)
                                         : make_float4(0.f, 0.f, 0.f, 0.f));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int sp = s0 + q;
          const float wgt = __shfl_sync(0xffffffffu, e, sp & 31);
          if (sp < ns && ((mask >> sp) & 1u)) {
            o0 = __fadd_rn(o0, __fmul_rn(wgt, ob[q].x));
            o1 = __fadd_rn(o1, __fmul_rn(wgt, ob[q].y));
            o2 = __fadd_rn(o2, __fmul_rn(wgt, ob[q].z));
            o3 = __fadd_rn(o3, __fmul_rn(wgt, ob[q].w));
          }
        }
      }
      v[j] = make_float4(__fdiv_rn(o0, L), __fdiv_rn(o1, L), __fdiv_rn(o2, L), __fdiv_rn(o3, L));
    }
  } else if (st.pro == PRO_COMBINE) {
    // any head dimension: per head, M = max_j m_j, L = sum_j [l_j > 0]
    // e^(m_j - M) l_j in split order, weights e^(m_j - M)
    // (attn_combine_kernel's arithmetic): lane j of the head's warp holds
    // split j
    float* cw = reinterpret_cast<float*>(smem + kOffComb);
    float* cml = reinterpret_cast<float*>(smem + kOffCombML);
    const int ns = a.nsplit;
    for (int h = warp; h < a.H; h += kCons) {
      const float* ml = a.part_ml + (size_t)h * ns * 2;
      float mj = -INFINITY, lj = 0.f;
      if (lane < ns) {
        mj = __ldcg(ml + 2 * lane);
        lj = __ldcg(ml + 2 * lane + 1);
      }
      float M = mj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      const bool live = lane < ns && lj > 0.f;
      const float e = live ? expf(__fsub_rn(mj, M)) : 0.f;
      const float el = live ? __fmul_rn(e, lj) : 0.f;
      float L = 0.f;
      for (int j = 0; j < ns; ++j) {
        const float t = __shfl_sync(0xffffffffu, el, j);
        const int lv = __shfl_sync(0xffffffffu, live ? 1 : 0, j);
        if (lv) L = __fadd_rn(L, t);
      }
      const unsigned mask = __ballot_sync(0xffffffffu, live);
      if (lane < kMaxSplit) cw[h * kMaxSplit + lane] = e;
      if (lane == 0) {
        cml[2 * h] = L;
        cml[2 * h + 1] = __int_as_float((int)mask);
      }
    }
    named_barrier(kBarCons, kConsThreads);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int f = tid + j * kConsThreads;
      float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
      if (f < f4) {
        const int e0 = 4 * f;
        const int h = e0 / a.HD, d = e0 - h * a.HD;
        const int mask = __float_as_int(cml[2 * h + 1]);
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
        for (int s0 = 0; s0 < kMaxSplit; s0 += 4) {
          if (s0 >= ns) break;
          float4 o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int sp = s0 + q;
            o[q] = (sp < ns && ((mask >> sp) & 1)) ? ldcg4(a.part_o + ((size_t)h * ns + sp) * a.HD + d)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int sp = s0 + q;
            if (sp < ns && ((mask >> sp) & 1)) {
              const float wgt = cw[h * kMaxSplit + sp];
              o0 = __fadd_rn(o0, __fmul_rn(wgt, o[q].x));
              o1 = __fadd_rn(o1, __fmul_rn(wgt, o[q].y));
              o2 = __fadd_rn(o2, __fmul_rn(wgt, o[q].z));
              o3 = __fadd_rn(o3, __fmul_rn(wgt, o[q].w));
            }
          }
        }
        const float L = cml[2 * h];
        r = make_float4(__fdiv_rn(o0, L), __fdiv_rn(o1, L), __fdiv_rn(o2, L), __fdiv_rn(o3, L));
      }
      v[j] = r;
    }
  } else if (st.pro == PRO_PLAIN) {
    // x as stored by the previous stage (the gate/up stage's SwiGLU output)
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int f = tid + j * kConsThreads;
      v[j] = f < f4 ? ldcg4(st.a + 4 * f) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    // RMSNorm of (embedding row) or (a + b); the sum is the residual stream
    const bool emb = st.pro == PRO_EMB_RMS;
    const float* erow = a.emb + (size_t)tok * K;
    const bool tok_ok = tok >= 0 && tok < a.vocab;
    if (emb) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int f = tid + j * kConsThreads;
        v[j] = (f < f4 && tok_ok) ? __ldg(reinterpret_cast<const float4*>(erow) + f)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
#pragma unroll
      for (int j0 = 0; j0 < NV; j0 += kPB) {
        float4 xa[kPB], xb[kPB];
#pragma unroll
        for (int jj = 0; jj < kPB; ++jj) {
          const int f = tid + (j0 + jj) * kConsThreads;
          const bool in = j0 + jj < NV && f < f4;
          xa[jj] = in ? ldcg4(st.a + 4 * f) : make_float4(0.f, 0.f, 0.f, 0.f);
          xb[jj] = in ? ldcg4(st.b + 4 * f) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int jj = 0; jj < kPB; ++jj) {
          if (j0 + jj >= NV) break;
          v[j0 + jj] = make_float4(__fadd_rn(xa[jj].x, xb[jj].x), __fadd_rn(xa[jj].y, xb[jj].y),
                                   __fadd_rn(xa[jj].z, xb[jj].z), __fadd_rn(xa[jj].w, xb[jj].w));
        }
      }
    }
    if (cid == 0 && st.res_out) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int f = tid + j * kConsThreads;
        if (f < f4) reinterpret_cast<float4*>(st.res_out)[f] = v[j];
      }
      __threadfence();
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int f = tid + j * kConsThreads;
      if (f < f4) {
        const float4 r = v[j];
        ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(r.x, r.x), __fmul_rn(r.y, r.y)),
                                     __fadd_rn(__fmul_rn(r.z, r.z), __fmul_rn(r.w, r.w))));
      }
    }
    if (tid == 0) tl_mark(a, stage, 3);
    ss = cons_sum(ss, red);
    if (tid == 0) tl_mark(a, stage, 4);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
#pragma unroll
    for (int j0 = 0; j0 < NV; j0 += kPB) {
      float4 w[kPB];
#pragma unroll
      for (int jj = 0; jj < kPB; ++jj) {
        const int f = tid + (j0 + jj) * kConsThreads;
        const bool in = j0 + jj < NV && f < f4;
        w[jj] = !in ? make_float4(0.f, 0.f, 0.f, 0.f)
                    : st.wstaged ? reinterpret_cast<const float4*>(smem + kOffWbuf)[f]
                                 : __ldg(reinterpret_cast<const float4*>(st.w) + f);
      }
#pragma unroll
      for (int jj = 0; jj < kPB; ++jj) {
        if (j0 + jj >= NV) break;
        const float4 x = v[j0 + jj];
        v[j0 + jj] = make_float4(__fmul_rn(__fmul_rn(x.x, inv), w[jj].x), __fmul_rn(__fmul_rn(x.y, inv), w[jj].y),
                                 __fmul_rn(__fmul_rn(x.z, inv), w[jj].z), __fmul_rn(__fmul_rn(x.w, inv), w[jj].w));
      }
    }
  }
  // max |x|, then the digits (as q4g_gemv_kernel, M = 1)
  float mx = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  mx = cons_max(mx, red);
  if (tid == 0) tl_mark(a, stage, 5);
  if (tid == 0) *xmaxp = mx;
  const float inv = mx > 0.f ? 127.0f / mx : 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int f = tid + j * kConsThreads;
    if ((f & ~31) >= f4) break;   // the whole warp is past K (f4 is a multiple of 32)
    const float xv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
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
      const int kt32 = f >> 3, jj = f & 7;
      const int half = jj >> 2, tt = jj & 3;
      xw[(((size_t)kt32 * 2 + 0) * 4 + tt) * 2 + half] = w0;
      xw[(((size_t)kt32 * 2 + 1) * 4 + tt) * 2 + half] = w1;
    }
    // a warp's 32 float4 are one group of 128 k (512 | 32 | f4 boundaries)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (lane == 0 && f < f4) {
      const int grp = f >> 5;
      sdi[grp * 16] += s0;       // one writer per group
      sdi[grp * 16 + 8] += s1;
    }
  }
  named_barrier(kBarCons, kConsThreads);
}

// The prologue instance whose register slots just hold K.
__device__ __forceinline__ void prologue(const DecArgs& a, const ProDesc& st, int cid, int tok,
                                         unsigned char* smem, int stage) {
  const int f4 = st.k >> 2;
  if (f4 <= 2 * kConsThreads) prologue_nv<2>(a, st, cid, tok, smem, stage);
  else if (f4 <= 6 * kConsThreads) prologue_nv<6>(a, st, cid, tok, smem, stage);
  else prologue_nv<kNV>(a, st, cid, tok, smem, stage);
}

// ------------------------------------------------------------ attention unit
// Query head h, positions [s0, s1) of split j (attn_split_kernel's arithmetic,
// with 16 warps): RoPE (rotate-half) on q and the new k, q scaled, KV append
// of row pos, scores, max, exp-sum, unnormalised P.V.
template <int DV>
__device__ void attn_unit(const DecArgs& a, const DecStage& st, int h, int j, int pos,
                          unsigned char* smem) {
  constexpr int HD = 32 * DV;
  constexpr int half = HD / 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* qs = reinterpret_cast<float*>(smem + kOffXs);
  float* kn = qs + kMaxHeadDim;
  float* vn = kn + kMaxHeadDim;
  float* sc = vn + kMaxHeadDim;
  float* ared = sc + kMaxPs;
  const int nrep = a.H / a.HKV, hkv = h / nrep, hkl = hkv - a.hk0;
  const int S = pos + 1;
  const int ps = (S + a.nsplit - 1) / a.nsplit;
  const int s0 = j * ps, s1 = min(S, s0 + ps), ns = max(0, s1 - s0);
  const bool has_new = ns > 0 && s1 == S;
  const float* cs = a.cos_t + (size_t)pos * half;
  const float* sn = a.sin_t + (size_t)pos * half;
  if (tid < half) {
    const float c = __ldg(cs + tid), s = __ldg(sn + tid);
    const float x1 = __ldcg(a.q + (size_t)h * HD + tid), x2 = __ldcg(a.q + (size_t)h * HD + tid + half);
    qs[tid] = __fmul_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s)), a.scale);
    qs[tid + half] = __fmul_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)), a.scale);
  } else if (tid >= 128 && tid < 128 + half && has_new) {
    const int i = tid - 128;
    const float c = __ldg(cs + i), s = __ldg(sn + i);
    const float x1 = __ldcg(a.k + (size_t)hkv * HD + i), x2 = __ldcg(a.k + (size_t)hkv * HD + i + half);
    kn[i] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
    kn[i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  } else if (tid >= 256 && tid < 256 + HD && has_new) {
    vn[tid - 256] = __ldcg(a.v + (size_t)hkv * HD + tid - 256);
  }
  named_barrier(kBarCons, kConsThreads);
  if (has_new && h % nrep == 0) {
    // appendKV: this unit is the only writer of row pos of KV head hkv
    const size_t row = ((size_t)hkl * a.max_seq + pos) * HD;
    if (tid < HD) st.kc[row + tid] = kn[tid];
    else if (tid >= 256 && tid < 256 + HD) st.vc[row + tid - 256] = vn[tid - 256];
  }
  const float* K = st.kc + ((size_t)hkl * a.max_seq + s0) * HD;
  const float* V = st.vc + ((size_t)hkl * a.max_seq + s0) * HD;
  float ql[DV];
#pragma unroll
  for (int i = 0; i < DV; ++i) ql[i] = qs[lane + 32 * i];
  // warp w takes positions [w U, w U + U) of every block of kCons U: at the
  // split lengths of a 4-way split of a few hundred positions, one block
  constexpr int U = 8;
  for (int b = warp * U; b < ns; b += kCons * U) {
    float kv[U][DV];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = b + u;
      const bool isnew = s0 + p == pos;
#pragma unroll
      for (int i = 0; i < DV; ++i)
        kv[u][i] = p < ns ? (isnew ? kn[lane + 32 * i] : __ldg(K + (size_t)p * HD + lane + 32 * i)) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < DV; ++i) acc = __fadd_rn(acc, __fmul_rn(ql[i], kv[u][i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0 && b + u < ns) sc[b + u] = acc;
    }
  }
  named_barrier(kBarCons, kConsThreads);
  float mx = -INFINITY;
  for (int s = tid; s < ns; s += kConsThreads) mx = fmaxf(mx, sc[s]);
  mx = cons_max(mx, red);
  float sum = 0.f;
  for (int s = tid; s < ns; s += kConsThreads) {
    const float e = expf(__fsub_rn(sc[s], mx));
    sc[s] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = cons_sum(sum, red);   // its barriers also publish sc
  float acc[DV];
#pragma unroll
  for (int i = 0; i < DV; ++i) acc[i] = 0.f;
  for (int b = warp * U; b < ns; b += kCons * U) {
    float vv[U][DV];
    {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = b + u;
        const bool isnew = s0 + p == pos;
#pragma unroll
        for (int i = 0; i < DV; ++i)
          vv[u][i] = p < ns ? (isnew ? vn[lane + 32 * i] : __ldg(V + (size_t)p * HD + lane + 32 * i)) : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (b + u < ns) {
        const float e = sc[b + u];
#pragma unroll
        for (int i = 0; i < DV; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(e, vv[u][i]));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < DV; ++i) ared[warp * HD + lane + 32 * i] = acc[i];
  named_barrier(kBarCons, kConsThreads);
  float* po = a.part_o + ((size_t)h * a.nsplit + j) * HD;
  float* pml = a.part_ml + ((size_t)h * a.nsplit + j) * 2;
  for (int d = tid; d < HD; d += kConsThreads) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) t = __fadd_rn(t, ared[w * HD + d]);
    if (a.world == 1) po[d] = t;
    else
      for (int q = 0; q < a.world; ++q) at_rank(a, po, q)[d] = t;
  }
  if (tid == 0) {
    if (a.world == 1) {
      pml[0] = mx;
      pml[1] = sum;
    } else {
      for (int q = 0; q < a.world; ++q) {
        at_rank(a, pml, q)[0] = mx;
        at_rank(a, pml, q)[1] = sum;
      }
    }
  }
  // partials and KV row visible before the arrival
  if (a.world == 1) __threadfence();
  else __threadfence_system();
  named_barrier(kBarCons, kConsThreads);  // scratch reused by the next unit
}

// ------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const DecArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int cid = blockIdx.x, G = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kNS;
  uint64_t* merged = empty + kNS;
  uint64_t* pfull = merged + kNS;
  unsigned char* ring = smem + kOffRing;
  float* part = reinterpret_cast<float*>(smem + kOffPart);
  int* rec = reinterpret_cast<int*>(smem + kOffRecent);
  const unsigned epoch = __ldcg(a.ctl);          // launches completed before this one
  const unsigned target = (epoch + 1u) * (unsigned)G;
  const unsigned gtarget = (epoch + 1u) * (unsigned)a.world;
  const int pos = *(volatile const int*)a.pos;
  const int tok = *(volatile const int*)a.tok_in;
  const int nst = a.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNcs);
      mbar_init(&merged[s], 1);
      mbar_init(&pfull[s], kNcs);
    }
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < a.n_recent; i += blockDim.x) rec[i] = __ldg(a.recent + i);
  __syncthreads();

  if (warp == kCons) {
    // ---------------- producer: the weights of every GEMV stage, in order
    if (lane < kIssuers) {
      bool ok = true;
      int q0 = 0, issued_last = -1;
      // L2 look-ahead: while the ring is full (consumers at a grid barrier),
      // DRAM keeps streaming the weights of this lane's item l2_ahead places
      // further on into L2, so the later bulk copy reads L2
      LaneCursor ahead;
      cursor_seek(a, ahead, 0, 0, lane, cid, G);
      for (int j = 0; j < a.l2_ahead && ahead.valid; ++j) cursor_next(a, ahead, cid, G);
      if (a.l2_ahead <= 0) ahead.valid = false;
      for (int s = 0; s < nst && ok; ++s) {
        const DecStage& st = a.stages[s];
        if (__ldg(&st.kind) != ST_GEMV) {
          // attention: pull this CTA's units' cached K / V rows (known before
          // the stage: they do not depend on q) into L2 while the q/k/v GEMV
          // runs; row pos is appended in the stage itself
          if (lane == 0 && pos >= 0 && pos < a.max_seq) {
            const int S = pos, nsp = a.nsplit, HD = a.HD;
            const int ps = (S + 1 + nsp - 1) / nsp;
            for (int u = cid; u < a.hloc * nsp; u += G) {
              const int h = a.h0 + u / nsp, j = u - (h - a.h0) * nsp;
              const int hkl = h / (a.H / a.HKV) - a.hk0;
              const int s0 = j * ps, s1 = min(S, s0 + ps);
              if (s1 <= s0) continue;
              const size_t off = ((size_t)hkl * a.max_seq + s0) * HD;
              const uint32_t bytes = (uint32_t)((s1 - s0) * HD * 4);
              bulk_prefetch_l2(st.kc + off, bytes);
              bulk_prefetch_l2(st.vc + off, bytes);
            }
          }
          continue;
        }
        int rt0, nrt;
        stage_rows(__ldg(&st.n_rt), __ldg(&st.pair), cid, G, &rt0, &nrt);
        const int nstg = nrt * __ldg(&st.nkb);
        const int first = ((lane - q0) % kIssuers + kIssuers) % kIssuers;
        for (int i = first; i < nstg; i += kIssuers) {
          const int qq = q0 + i;
          const int slot = qq % kNS;
          if (ahead.valid) {
            const ItemSrc pf = item_src(a.stages[ahead.s], ahead.rt0, ahead.i);
            bulk_prefetch_l2(pf.w, pf.wb);
            bulk_prefetch_l2(pf.z, pf.zb);
            cursor_next(a, ahead, cid, G);
          }
          if (qq >= kNS && !dwait<-32>(a, &empty[slot], ((qq / kNS) - 1) & 1)) {
            ok = false;
            break;
          }
          const ItemSrc src = item_src(st, rt0, i);
          unsigned char* dst = ring + (size_t)slot * kStageBytes;
          mbar_arrive_expect_tx(&full[slot], src.wb + src.zb);
          bulk_g2s(dst, src.w, src.wb, &full[slot]);
          bulk_g2s(dst + kStageW, src.z, src.zb, &full[slot]);
          issued_last = qq;
        }
        q0 += nstg;
      }
      // Drain: lane l issues only into slot l (kNS == kIssuers), and it waits
      // for `empty` before reusing it, so at most its last copy can still be in
      // flight.  Wait for it even after an abort (with the launch-independent
      // bound of mbar_wait), so the CTA never exits with a bulk copy landing
      // in its shared memory.
      if (issued_last >= 0 && !mbar_wait(&full[issued_last % kNS], (issued_last / kNS) & 1)) ok = false;
      if (!ok && a.err) atomicExch(a.err, 1);
    }
    __syncwarp();
  } else if (warp == kCons + 1) {
    // ---------------- merge warp: chunk partials -> y, stage arrivals, argmax
    uint32_t* mark = reinterpret_cast<uint32_t*>(smem + kOffMark);
    int q0 = 0;
    for (int s = 0; s < nst; ++s) {
      const DecStage& st = a.stages[s];
      if (st.kind != ST_GEMV) continue;
      int rt0, nrt;
      stage_rows(st.n_rt, st.pair, cid, G, &rt0, &nrt);
      const int nkb = st.nkb;
      const int nstg = nrt * nkb;
      const bool greedy = st.greedy && a.tok_out != nullptr;
      if (greedy) {
        // rows of this CTA that the recent list names get the ordered penalty
        for (int i = lane; i < 128; i += 32) mark[i] = 0u;
        __syncwarp();
        for (int i = lane; i < a.n_recent; i += 32) {
          const int r = rec[i] - (st.row0[0] + rt0 * 16);
          if (r >= 0 && r < nrt * 16 && r < 4096) atomicOr(&mark[r >> 5], 1u << (r & 31));
        }
        __syncwarp();
      }
      float bestv = -INFINITY;
      int besti = -1, nan0 = 0;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      // the stage's problem table in registers: read once per stage, not
      // once per item (each read would be a global load on this serial warp)
      int prt[kMaxProb + 1], prow[kMaxProb], pr0[kMaxProb];
      float* pyp[kMaxProb];
      bool ploc[kMaxProb];
#pragma unroll
      for (int j = 0; j < kMaxProb; ++j) {
        prt[j] = st.rt_prefix[j];
        prow[j] = st.rows[j];
        pr0[j] = st.row0[j];
        float* yj = st.y[j];
        pyp[j] = yj ? yj : a.logits;
        ploc[j] = a.world == 1 || !yj;   // logits: this rank's rows, locally
      }
      prt[kMaxProb] = st.rt_prefix[kMaxProb];
      const int np = st.nprob;
      const bool pair = st.pair != 0;
      int kb = 0, rti = 0, p = 0;       // k-block, row tile, problem of item i
      float gate = 0.f;                 // paired stage: this lane's gate value
      for (int i = 0; i < nstg; ++i) {
        const int qq = q0 + i;
        const int slot = qq % kNS;
        if (!dwait<1000>(a, &pfull[slot], (qq / kNS) & 1)) {
          if (lane == 0 && a.err) atomicExch(a.err, 1);
          break;
        }
        const float* rd = part + (size_t)slot * kNcs * 128;
        if (kb == 0) v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int c2 = 0; c2 < kNcs; ++c2) {
          const float4 e4 = reinterpret_cast<const float4*>(rd + c2 * 128)[lane];
          v.x += e4.x;
          v.y += e4.y;
          v.z += e4.z;
          v.w += e4.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&merged[slot]);
        const bool row_done = kb == nkb - 1;
        if (++kb == nkb) kb = 0;
        if (!row_done) continue;
        // columns 4..7 hold the second digit's part of x row 0
        float yv = v.x + __shfl_xor_sync(0xffffffffu, v.x, 1);
        const int grt = rt0 + rti++;
        int r;
        if (pair) {
          // gate tile (even): keep; up tile (odd): store SwiGLU into y[0],
          // as swiglu_kernel: sigmoid = 1 / (1 + e^-g), (g sigmoid) u
          r = (grt >> 1) * 16 + (lane >> 1);
          if ((grt & 1) == 0) {
            gate = yv;
            continue;
          }
          const float sig = __frcp_rn(__fadd_rn(1.0f, expf(-gate)));
          yv = __fmul_rn(__fmul_rn(gate, sig), yv);
          p = 0;
        } else {
          while (p + 1 < np && grt >= pick(prt, p + 1)) ++p;
          r = (grt - pick(prt, p)) * 16 + (lane >> 1);
        }
        if ((lane & 1) == 0 && r < pick(prow, p)) {
          float* yp = pick(pyp, p);
          const int gr = pick(pr0, p) + r;   // output row of the full weight
          if (pick(ploc, p)) {
            yp[gr] = yv;
          } else {
            for (int q2 = 0; q2 < a.world; ++q2) at_rank(a, yp, q2)[gr] = yv;
          }
          if (greedy) {
            float adj = yv;
            const int lr = r - rt0 * 16;
            if (lr >= 4096 || ((mark[lr >> 5] >> (lr & 31)) & 1u)) {
              for (int t = 0; t < a.n_recent; ++t)
                if (rec[t] == gr) adj = adj > 0.0f ? __fdiv_rn(adj, a.penalty) : __fmul_rn(adj, a.penalty);
            }
            if (gr == 0 && adj != adj) nan0 = 1;
            if (adj == adj && (besti < 0 || adj > bestv)) {
              bestv = adj;
              besti = gr;
            }
          }
        }
      }
      q0 += nstg;
      if (greedy) {
        // warp argmax: larger value, then lower index (rows rise with lanes and tiles)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bestv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
          if (oi >= 0 && (besti < 0 || ov > bestv || (ov == bestv && oi < besti))) {
            bestv = ov;
            besti = oi;
          }
        }
        nan0 = __any_sync(0xffffffffu, nan0);
        if (lane == 0) {
          int* cd = a.cand + ((size_t)a.rank * G + cid) * 4;
          for (int q2 = 0; q2 < a.world; ++q2) {
            int* cq = a.world == 1 ? cd : at_rank(a, cd, q2);
            cq[0] = __float_as_int(bestv);
            cq[1] = besti;
            cq[2] = nan0;
          }
        }
      }
      if (lane == 0) tl_mark(a, s, 8);
      // this lane's y (and argmax) visible before the arrival
      if (a.world == 1) __threadfence();
      else __threadfence_system();
      __syncwarp();
      if (lane == 0) {
        tl_mark(a, s, 2);
        arrive(a, s, target);
      }
    }
  } else {
    // ---------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const float* xmaxp = reinterpret_cast<const float*>(smem + kOffMisc);
    const int* sdi = reinterpret_cast<const int*>(smem + kOffSdi);
    // x row 0 is B columns 0 (d0) and 4 (d1); the lanes of columns 1-3 and
    // 5-7 read the same digits (one wavefront per B load), and those MMA
    // columns are never read back
    const int ccol = g < 4 ? 0 : 1;
    const uint2* xs2 = reinterpret_cast<const uint2*>(smem + kOffXs) + ccol * 4 + t;
    const int xstride = 8;
    const int sd_off = t < 2 ? 2 * t : 2 * t + 4;
    int q0 = 0;
    for (int s = 0; s < nst; ++s) {
      const DecStage& st = a.stages[s];
      if (st.kind == ST_ATTN) {
        // wait for q/k/v of every CTA, then this CTA's (head, split) units
        if (threadIdx.x == 0 && s > 0) stage_wait(a, s - 1, target, gtarget);
        named_barrier(kBarCons, kConsThreads);
        if (threadIdx.x == 0) tl_mark(a, s, 0);
        const int units = a.hloc * a.nsplit;   // this rank's heads
        if (pos >= 0 && pos < a.max_seq) {
          for (int u = cid; u < units; u += G) {
            const int h = a.h0 + u / a.nsplit, j = u - (h - a.h0) * a.nsplit;
            if (a.HD == 128) attn_unit<4>(a, st, h, j, pos, smem);
            else attn_unit<2>(a, st, h, j, pos, smem);
          }
        } else if (cid == 0 && threadIdx.x == 0 && a.err) {
          atomicExch(a.err, 4);   // position outside the KV cache: nothing is read or appended
        }
        named_barrier(kBarCons, kConsThreads);
        if (threadIdx.x == 0) {
          tl_mark(a, s, 2);
          arrive(a, s, target);
        }
        continue;
      }
      ProDesc pd;
      pd.k = st.k;
      pd.groups = st.groups;
      pd.pro = st.pro;
      pd.nkb = st.nkb;
      pd.n_rt = st.n_rt;
      pd.pair = st.pair;
      pd.a = st.a;
      pd.b = st.b;
      pd.w = st.w;
      pd.res_out = st.res_out;
      // the norm weights do not depend on the previous stage: staged in
      // shared memory while the grid barrier is pending
      pd.wstaged = (pd.pro == PRO_ADD_RMS || pd.pro == PRO_EMB_RMS) && pd.k <= kWbufK;
      if (pd.wstaged) {
        float4* wb = reinterpret_cast<float4*>(smem + kOffWbuf);
        for (int f = threadIdx.x; f < (pd.k >> 2); f += kConsThreads)
          wb[f] = __ldg(reinterpret_cast<const float4*>(pd.w) + f);
      }
      int rt0, nrt;
      stage_rows(pd.n_rt, pd.pair, cid, G, &rt0, &nrt);
      const int nkb = pd.nkb;
      const int nstg = nrt * nkb;
      if (threadIdx.x == 0 && s > 0) stage_wait(a, s - 1, target, gtarget);
      named_barrier(kBarCons, kConsThreads);  // also: every warp is done with the last x
      if (threadIdx.x == 0) tl_mark(a, s, 0);
      prologue(a, pd, cid, tok, smem, s);
      if (threadIdx.x == 0) tl_mark(a, s, 1);
      const float sm = *xmaxp / 127.0f;
      const float dsc = t < 2 ? sm : sm * (1.0f / 256.0f);
      const int groups = pd.groups;
      const int ubeg = q0 * kNcs, uend = (q0 + nstg) * kNcs;
      const int u0 = ubeg + ((warp - ubeg) % kCons + kCons) % kCons;
      // k-block of the warp's item, stepped without a division (kCons units
      // are kCons / kNcs items)
      int kb = (u0 / kNcs - q0) % nkb;
      static_assert(kCons % kNcs == 0, "whole items per consumer round");
      auto step_kb = [&]() {
        kb += kCons / kNcs;
        while (kb >= nkb) kb -= nkb;
      };
      for (int u = u0; u < uend; u += kCons, step_kb()) {
        const int qq = u / kNcs, c = u - qq * kNcs;
        const int slot = qq % kNS;
        const int ngk = min(kKbg, groups - kb * kKbg);
        const int cg0 = c * kCG, ncg = max(0, min(kCG, ngk - cg0));
        const int gb = kb * kKbg + cg0;  // first group of the chunk
        float tot[4] = {0.f, 0.f, 0.f, 0.f};
        if (!dwait<1000>(a, &full[slot], (qq / kNS) & 1)) {
          if (lane == 0 && a.err) atomicExch(a.err, 1);
        } else {
          if (threadIdx.x == 0 && u == u0) tl_mark(a, s, 6);
          const unsigned char* stg = ring + (size_t)slot * kStageBytes;
          const uint4* wq = reinterpret_cast<const uint4*>(stg + (size_t)c * kChunkQ * 512) + lane;
          const float4* szp = reinterpret_cast<const float4*>(stg + kStageW + (size_t)cg0 * 128) + g;
#pragma unroll
          for (int gl = 0; gl < kCG; ++gl) {
            if (gl < ncg) {
              int ac[4] = {0, 0, 0, 0};
#pragma unroll
              for (int qq2 = 0; qq2 < kKQG; ++qq2) {
                const int ql = gl * kKQG + qq2;
                const uint4 w = wq[ql * 32];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                  // high nibbles masked in place: rows g + 8 at 16 times
                  // their value (u8 A operand), shifted out below
                  const uint32_t wa = hh == 0 ? w.x : w.z, wb = hh == 0 ? w.y : w.w;
                  const uint32_t a0 = wa & 0x0F0F0F0Fu, a1 = wa & 0xF0F0F0F0u;
                  const uint32_t a2 = wb & 0x0F0F0F0Fu, a3 = wb & 0xF0F0F0F0u;
                  const int kt32 = (gb * kKQG + ql) * 2 + hh;
                  const uint2 bfr = xs2[(size_t)kt32 * xstride];
                  mma_u8s8_16832(ac, a0, a1, a2, a3, bfr.x, bfr.y);
                }
              }
              const float4 sp = szp[gl * 8];
              const float d0 = (float)sdi[(gb + gl) * 16 + sd_off];
              tot[0] = fmaf(sp.x * dsc, fmaf(-sp.y, d0, (float)ac[0]), tot[0]);
              tot[2] = fmaf(sp.z * dsc, fmaf(-sp.w, d0, (float)(ac[2] >> 4)), tot[2]);   // exact: 16 A
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
          if (threadIdx.x == 0 && u == u0) tl_mark(a, s, 9);
        }
        // hand the chunk's partial to the merge warp (slot reused: wait until
        // the merge warp has read the previous round)
        float* rd = part + (size_t)slot * kNcs * 128;
        if (qq >= kNS && !dwait<1000>(a, &merged[slot], ((qq / kNS) - 1) & 1)) {
          if (lane == 0 && a.err) atomicExch(a.err, 1);
          continue;
        }
        if (threadIdx.x == 0 && u == u0) tl_mark(a, s, 10);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = g + ((e & 2) ? 8 : 0);
          const int mm = 2 * t + (e & 1);
          rd[(size_t)c * 128 + r * 8 + mm] = tot[e];
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[slot]);
        if (threadIdx.x == 0 && u == u0) tl_mark(a, s, 11);
        if (threadIdx.x == 0 && u + kCons >= uend) tl_mark(a, s, 7);
      }
      q0 += nstg;
    }
    // CTA 0 picks the next token from the per-CTA argmax results
    if (cid == 0 && a.tok_out != nullptr && threadIdx.x == 0) {
      bool ok = stage_wait(a, nst - 1, target, gtarget);
      float bv = -INFINITY;
      int bi = -1, n0 = 0;
      for (int c2 = 0; c2 < G * a.world && ok; ++c2) {   // every rank's CTAs, in rank order
        const int* cd = a.cand + (size_t)c2 * 4;
        const float cv = __int_as_float(__ldcg(cd));
        const int ci = __ldcg(cd + 1);
        n0 |= __ldcg(cd + 2);
        if (ci >= 0 && (bi < 0 || cv > bv || (cv == bv && ci < bi))) {
          bv = cv;
          bi = ci;
        }
      }
      *a.tok_out = (n0 || bi < 0) ? 0 : bi;
    }
    if (cid == 0 && threadIdx.x == 0 && a.advance_pos) {
      stage_wait(a, nst - 1, target, gtarget);
      *a.pos = pos + 1;
    }
  }
  __syncthreads();
  // the last CTA to finish the step counts the launch
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned old = atomicAdd(a.ctl + 2 + nst, 1u);
    if (old == target - 1u) atomicAdd(a.ctl, 1u);
  }
}

// ------------------------------------------------------------ host side
struct DecodePlan {
  int device = -1;
  int grid = 0;
  int world = 1, rank = 0;
  std::vector<DecStage> stages;
  DecStage* d_stages = nullptr;
  void* scratch = nullptr;
  void* peers[kMaxRanks] = {};   // sharded: every rank's scratch as mapped here
  DecArgs base = {};
  int64_t vocab = 0;
  unsigned long long* timeline = nullptr;   // caller's buffer (not owned)
  int tl_cta = 0;
};

std::vector<DecodePlan*> g_plans;
unsigned long long g_dec_wait_ns = 2000000000ull;

DecodePlan* find_plan(int64_t id) {
  if (id < 1 || id > (int64_t)g_plans.size()) return nullptr;
  return g_plans[(size_t)id - 1];
}

// The int4-g128 weight behind handle h, which must hold rows [r0, r1) of an
// n-row, k-column weight (the whole weight on one GPU, this rank's
// shard_range rows on a sharded plan).
int q4_of(nimf_weight_t h, int64_t k, int64_t n, int world, int rank, const char* what,
          const Q4GWeight** out, int* row0) {
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "decode plan: %s: unknown weight handle", what);
  if (w->kind != NIMF_KIND_INT4_ASYM || !w->q4.fast || w->q4.gs != kGS)
    return set_error(NIMF_ERR_UNSUPPORTED,
                     "decode plan: %s must be an int4 asymmetric weight with group size 128", what);
  if (w->kperm) return set_error(NIMF_ERR_UNSUPPORTED, "decode plan: %s has an act-order permutation", what);
  int64_t r0 = 0, r1 = n;
  if (world > 1) shard_range(n, world, rank, &r0, &r1);
  const int64_t nf = w->n_full > 0 ? w->n_full : w->q4.rows;
  if (w->q4.k != k || w->q4.rows != r1 - r0 || w->row_begin != r0 || nf != n)
    return set_error(NIMF_ERR_SHAPE,
                     "decode plan: %s holds rows [%lld, %lld) of [%lld x %lld], expected rows "
                     "[%lld, %lld) of [%lld x %lld]", what, (long long)w->row_begin,
                     (long long)(w->row_begin + w->q4.rows), (long long)nf, (long long)w->q4.k,
                     (long long)r0, (long long)r1, (long long)n, (long long)k);
  *out = &w->q4;
  *row0 = (int)r0;
  return NIMF_OK;
}

DecStage gemv_stage(int pro, const Q4GWeight* const* ws, const int* row0, float* const* ys, int n,
                    int64_t k, bool pair = false) {
  DecStage s = {};
  s.kind = ST_GEMV;
  s.pro = pro;
  s.k = (int)k;
  s.groups = (int)(k / kGS);
  s.nkb = (s.groups + kKbg - 1) / kKbg;
  s.nprob = n;
  s.rt_prefix[0] = 0;
  for (int i = 0; i < n; ++i) {
    s.frag[i] = (const uint4*)ws[i]->frag;
    s.sz[i] = (const float4*)ws[i]->sz;
    s.y[i] = ys[i];
    s.rows[i] = (int)ws[i]->rows;
    s.row0[i] = row0[i];
    s.rt_prefix[i + 1] = s.rt_prefix[i] + (int)ws[i]->n_rt;
  }
  s.n_rt = s.rt_prefix[n];
  s.pair = pair ? 1 : 0;   // (callers check: two problems with equal rows)
  return s;
}

void free_plan(DecodePlan* P) {
  if (!P) return;
  if (P->world > 1) comm_unshare_buffer(P->peers, P->world, P->rank);
  device_free(P->d_stages);
  device_free(P->scratch);
  delete P;
}

// Validates the descriptor and builds the stage table and scratch.  A sharded
// plan (world > 1) also exchanges the scratch's IPC handle with every rank;
// before that exchange the ranks agree on whether all of them validated, so a
// rank whose arguments are wrong makes every rank fail instead of leaving the
// others waiting in the exchange.
int create_plan(const nimf_decode_desc* d, int world, int rank, int64_t* plan_out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  DecodePlan* P = nullptr;
  int rc = NIMF_OK;
  int64_t L = 0, D = 0, H = 0, HKV = 0, HD = 0, F = 0, V = 0, MS = 0, KVD = 0;
  int grid = 0, nsplit = 1;
  size_t off = 0, o_q = 0, o_k = 0, o_v = 0, o_po = 0, o_pml = 0, o_ao = 0, o_g = 0, o_u = 0,
         o_dn = 0, o_xr = 0, o_hr = 0, o_cand = 0, o_ctl = 0, o_gctl = 0;
  int nst = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) / 256 * 256; return o; };
  // ---- validation (no collective before the agreement below)
  do {
    if (!d || !plan_out || !d->layers) {
      rc = set_error(NIMF_ERR_ARG, "decode_create: NULL argument");
      break;
    }
    L = d->n_layers, D = d->d_model, H = d->n_heads, HKV = d->n_kv_heads, HD = d->head_dim,
    F = d->ffn_dim, V = d->vocab, MS = d->max_seq;
    if (L < 1 || D < kGS || D % kGS || F % kGS || D > kMaxK || F > kMaxK || V < 1 || H < 1 ||
        H > kMaxHeads || HKV < 1 || H % HKV || (HD != 64 && HD != 128) || H * HD != D || MS < 1) {
      rc = set_error(NIMF_ERR_SHAPE,
                     "decode_create: unsupported shape (layers %lld, d_model %lld, heads %lld/%lld, "
                     "head_dim %lld, ffn %lld, vocab %lld, max_seq %lld); needs d_model and ffn "
                     "multiples of 128 up to %d, head_dim 64 or 128, heads x head_dim = d_model",
                     (long long)L, (long long)D, (long long)H, (long long)HKV, (long long)HD,
                     (long long)F, (long long)V, (long long)MS, kMaxK);
      break;
    }
    if (world > 1 && (HKV % world || H % world)) {
      rc = set_error(NIMF_ERR_SHAPE,
                     "decode_create_sharded: %lld query and %lld KV heads do not split over %d GPUs",
                     (long long)H, (long long)HKV, world);
      break;
    }
    if (d->n_recent_max < 0 || d->n_recent_max > kMaxRecent) {
      rc = set_error(NIMF_ERR_SHAPE, "decode_create: n_recent_max %lld not in [0, %d]",
                     (long long)d->n_recent_max, kMaxRecent);
      break;
    }
    if (!d->embedding || !d->final_norm || !d->rope_cos || !d->rope_sin) {
      rc = set_error(NIMF_ERR_ARG, "decode_create: NULL model array");
      break;
    }
    KVD = HKV * HD;
    // One GPU: one CTA per SM, at most the row tiles of the smallest GEMV
    // stage (n_rt of q/k/v, o, gate/up, down and lm_head).  A sharded plan
    // takes every SM (a rank's shards can be a few tiles; CTAs without rows in
    // a stage still take part in its barrier).  The attention split count is
    // the one-GPU plan's, so a sharded step computes the same numbers.
    int64_t min_rt = std::min<int64_t>((D + 15) / 16 + 2 * ((KVD + 15) / 16), (D + 15) / 16);
    min_rt = std::min<int64_t>(min_rt, 2 * ((F + 15) / 16));
    min_rt = std::min<int64_t>(min_rt, (V + 15) / 16);
    const int grid1 = (int)std::max<int64_t>(1, std::min<int64_t>(c->num_sms, min_rt));
    grid = world > 1 ? c->num_sms : grid1;
    nsplit = std::max(1, std::min(kMaxSplit, grid1 / (int)H));
    while (nsplit < kMaxSplit && (MS + nsplit - 1) / nsplit > kMaxPs) ++nsplit;
    if ((MS + nsplit - 1) / nsplit > kMaxPs) {
      rc = set_error(NIMF_ERR_SHAPE, "decode_create: max_seq %lld too long", (long long)MS);
      break;
    }
  } while (0);
  if (rc == NIMF_OK) {
    P = new DecodePlan();
    P->device = c->device;
    P->grid = grid;
    P->vocab = V;
    P->world = world;
    P->rank = rank;
    // scratch: q, k, v, attention partials, o out, gate, up, down out, two
    // residual rows, per-CTA argmax of every rank, control words
    nst = (int)(5 * L + 1);
    o_q = take(D * 4), o_k = take(KVD * 4), o_v = take(KVD * 4);
    o_po = take((size_t)H * nsplit * HD * 4), o_pml = take((size_t)H * nsplit * 2 * 4);
    o_ao = take(D * 4), o_g = take(F * 4), o_u = take(F * 4), o_dn = take(D * 4);
    o_xr = take(D * 4), o_hr = take(D * 4);
    o_cand = take((size_t)world * grid * 4 * 4);
    o_ctl = take((size_t)(nst + 3) * 4);
    o_gctl = take((size_t)(nst + 1) * 4);
    rc = device_alloc(&P->scratch, off);
  }
  if (rc == NIMF_OK) {
    char* sb = (char*)P->scratch;
    float *bq = (float*)(sb + o_q), *bk = (float*)(sb + o_k), *bv = (float*)(sb + o_v);
    float *bao = (float*)(sb + o_ao), *bg = (float*)(sb + o_g), *bu = (float*)(sb + o_u);
    float *bdn = (float*)(sb + o_dn), *bxr = (float*)(sb + o_xr), *bhr = (float*)(sb + o_hr);
    for (int64_t l = 0; l < L && rc == NIMF_OK; ++l) {
      const nimf_decode_layer_desc& ld = d->layers[l];
      const Q4GWeight *wq, *wk, *wv, *wo, *wg, *wu, *wd;
      int r0q, r0k, r0v, r0o, r0g, r0u, r0d;
      if ((rc = q4_of(ld.wq, D, D, world, rank, "wq", &wq, &r0q)) ||
          (rc = q4_of(ld.wk, D, KVD, world, rank, "wk", &wk, &r0k)) ||
          (rc = q4_of(ld.wv, D, KVD, world, rank, "wv", &wv, &r0v)) ||
          (rc = q4_of(ld.wo, D, D, world, rank, "wo", &wo, &r0o)) ||
          (rc = q4_of(ld.wgate, D, F, world, rank, "wgate", &wg, &r0g)) ||
          (rc = q4_of(ld.wup, D, F, world, rank, "wup", &wu, &r0u)) ||
          (rc = q4_of(ld.wdown, F, D, world, rank, "wdown", &wd, &r0d)))
        break;
      if (!ld.attn_norm || !ld.ffn_norm || !ld.k_cache || !ld.v_cache) {
        rc = set_error(NIMF_ERR_ARG, "decode_create: layer %lld has a NULL array", (long long)l);
        break;
      }
      {
        const Q4GWeight* ws[3] = {wq, wk, wv};
        const int r0s[3] = {r0q, r0k, r0v};
        float* ys[3] = {bq, bk, bv};
        DecStage s = gemv_stage(l == 0 ? PRO_EMB_RMS : PRO_ADD_RMS, ws, r0s, ys, 3, D);
        s.a = bhr;
        s.b = bdn;
        s.w = ld.attn_norm;
        s.res_out = bxr;
        P->stages.push_back(s);
      }
      {
        DecStage s = {};
        s.kind = ST_ATTN;
        s.kc = ld.k_cache;
        s.vc = ld.v_cache;
        P->stages.push_back(s);
      }
      {
        const Q4GWeight* ws[1] = {wo};
        const int r0s[1] = {r0o};
        float* ys[1] = {bao};
        P->stages.push_back(gemv_stage(PRO_COMBINE, ws, r0s, ys, 1, D));
      }
      {
        // gate and up rows interleaved per 16-row tile: the merge warps store
        // SwiGLU(gate, up) into bg, which the down stage reads as its x
        const Q4GWeight* ws[2] = {wg, wu};
        const int r0s[2] = {r0g, r0u};
        float* ys[2] = {bg, bu};
        if (wg->rows != wu->rows || r0g != r0u) {
          rc = set_error(NIMF_ERR_SHAPE, "decode plan: layer %lld gate and up shards differ", (long long)l);
          break;
        }
        DecStage s = gemv_stage(PRO_ADD_RMS, ws, r0s, ys, 2, D, true);
        s.a = bxr;
        s.b = bao;
        s.w = ld.ffn_norm;
        s.res_out = bhr;
        P->stages.push_back(s);
      }
      {
        const Q4GWeight* ws[1] = {wd};
        const int r0s[1] = {r0d};
        float* ys[1] = {bdn};
        DecStage s = gemv_stage(PRO_PLAIN, ws, r0s, ys, 1, F);
        s.a = bg;
        P->stages.push_back(s);
      }
    }
    if (rc == NIMF_OK) {
      const Q4GWeight* wh;
      int r0h;
      rc = q4_of(d->lm_head, D, V, world, rank, "lm_head", &wh, &r0h);
      if (rc == NIMF_OK) {
        float* ys[1] = {nullptr};  // the launch's logits buffer
        DecStage s = gemv_stage(PRO_ADD_RMS, &wh, &r0h, ys, 1, D);
        s.a = bhr;
        s.b = bdn;
        s.w = d->final_norm;
        s.res_out = bxr;
        s.greedy = 1;
        P->stages.push_back(s);
      }
    }
    if (rc == NIMF_OK) rc = device_alloc((void**)&P->d_stages, P->stages.size() * sizeof(DecStage));
    if (rc == NIMF_OK) {
      cudaError_t e = cudaMemcpy(P->d_stages, P->stages.data(), P->stages.size() * sizeof(DecStage),
                                 cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = cudaMemset(P->scratch, 0, off);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess) rc = set_error(NIMF_ERR_CUDA, "decode_create: %s", cudaGetErrorString(e));
    }
    if (rc == NIMF_OK) {
      cudaError_t e = cudaFuncSetAttribute(decode_step_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      int per_sm = 0;
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads,
                                                          kSmemBytes);
      if (e != cudaSuccess) rc = set_error(NIMF_ERR_CUDA, "decode_create: %s", cudaGetErrorString(e));
      else if (per_sm < 1)
        rc = set_error(NIMF_ERR_UNSUPPORTED, "decode_create: the step kernel does not fit an SM");
    }
  }
  if (world > 1) {
    // every rank learns whether all of them got this far, then (all did)
    // shares its scratch with the others
    int ok_all = 0;
    const int rc_agree = comm_agree(rc == NIMF_OK, &ok_all);
    if (rc == NIMF_OK && rc_agree != NIMF_OK) rc = rc_agree;
    if (rc == NIMF_OK && !ok_all)
      rc = set_error(NIMF_ERR_STATE, "decode_create_sharded: another rank failed to build its plan");
    if (rc == NIMF_OK) rc = comm_share_buffer(P->scratch, P->peers);
  }
  if (rc != NIMF_OK) {
    if (P) {
      P->world = 1;  // nothing was opened
      free_plan(P);
    }
    return rc;
  }
  char* sb = (char*)P->scratch;
  DecArgs& A = P->base;
  A.stages = P->d_stages;
  A.nstages = (int)P->stages.size();
  A.D = (int)D;
  A.H = (int)H;
  A.HKV = (int)HKV;
  A.HD = (int)HD;
  A.max_seq = (int)MS;
  A.nsplit = nsplit;
  A.vocab = (int)V;
  A.eps = d->norm_eps;
  A.scale = 1.0f / sqrtf((float)HD);
  A.emb = d->embedding;
  A.cos_t = d->rope_cos;
  A.sin_t = d->rope_sin;
  A.q = (float*)(sb + o_q);
  A.k = (float*)(sb + o_k);
  A.v = (float*)(sb + o_v);
  A.part_o = (float*)(sb + o_po);
  A.part_ml = (float*)(sb + o_pml);
  A.cand = (int*)(sb + o_cand);
  A.ctl = (unsigned*)(sb + o_ctl);
  A.gctl = (unsigned*)(sb + o_gctl);
  A.world = world;
  A.rank = rank;
  A.timeline = nullptr;
  // L2 look-ahead of the producer lanes, in items of up to 36 KB per lane
  // (NIMF_DECODE_L2_AHEAD, 0 .. 16; default 0: measured slower at 2)
  A.l2_ahead = 0;
  if (const char* ev = getenv("NIMF_DECODE_L2_AHEAD")) A.l2_ahead = std::max(0, std::min(16, atoi(ev)));
  A.hloc = (int)(H / world);
  A.h0 = (int)(rank * (H / world));
  A.hk0 = (int)(rank * (HKV / world));
  for (int q = 0; q < kMaxRanks; ++q)
    A.peer_off[q] = (q < world && P->peers[q]) ? (long long)((char*)P->peers[q] - sb) : 0;
  g_plans.push_back(P);
  *plan_out = (int64_t)g_plans.size();
  return NIMF_OK;
}

}  // namespace

void release_decode_plans() {
  for (DecodePlan*& p : g_plans) {
    free_plan(p);
    p = nullptr;
  }
  g_plans.clear();
}

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_decode_create(const nimf_decode_desc* d, int64_t* plan_out) {
  return create_plan(d, 1, 0, plan_out);
}

int nimf_decode_create_sharded(const nimf_decode_desc* d, int64_t* plan_out) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  int world = 1, rank = 0;
  NIMF_TRY(comm_world(&world, &rank));
  return create_plan(d, world, rank, plan_out);
}

int nimf_decode_step_dev(int64_t plan, int32_t* token_dev, int32_t* next_token_dev,
                         int32_t* pos_dev, int advance_pos, const int32_t* recent_dev,
                         int64_t n_recent, float penalty, float* logits_dev, void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  DecodePlan* P = find_plan(plan);
  if (!P) return set_error(NIMF_ERR_STATE, "decode_step: unknown plan %lld", (long long)plan);
  if (P->device != c->device)
    return set_error(NIMF_ERR_STATE, "decode_step: plan of device %d used on %d", P->device, c->device);
  if (!token_dev || !pos_dev || !logits_dev)
    return set_error(NIMF_ERR_ARG, "decode_step: NULL token, position or logits buffer");
  if (n_recent < 0 || n_recent > kMaxRecent || (n_recent > 0 && !recent_dev))
    return set_error(NIMF_ERR_SHAPE, "decode_step: %lld recent ids (at most %d)", (long long)n_recent,
                     kMaxRecent);
  DecArgs A = P->base;
  A.logits = logits_dev;
  A.tok_in = token_dev;
  A.tok_out = next_token_dev;
  A.pos = pos_dev;
  A.advance_pos = advance_pos ? 1 : 0;
  A.recent = recent_dev;
  A.n_recent = (int)n_recent;
  A.penalty = penalty;
  A.err = c->dev_err;
  A.wait_ns = g_dec_wait_ns;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)P->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream ? (cudaStream_t)stream : c->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_step_kernel, A));
  return NIMF_OK;
}

int nimf_decode_timeline(int64_t plan, uint64_t* timeline_dev, int64_t n, int cta) {
  DecodePlan* P = find_plan(plan);
  if (!P) return set_error(NIMF_ERR_STATE, "decode_timeline: unknown plan %lld", (long long)plan);
  if (timeline_dev && (n < kTlMarks * (int64_t)P->stages.size() || cta < 0 || cta >= P->grid))
    return set_error(NIMF_ERR_SHAPE, "decode_timeline: %lld entries for %zu stages, CTA %d of %d",
                     (long long)n, P->stages.size(), cta, P->grid);
  P->base.timeline = (unsigned long long*)timeline_dev;
  P->base.tl_cta = cta;
  return NIMF_OK;
}

int nimf_decode_info(int64_t plan, int64_t* grid, int64_t* stages, int64_t* attn_splits) {
  DecodePlan* P = find_plan(plan);
  if (!P) return set_error(NIMF_ERR_STATE, "decode_info: unknown plan %lld", (long long)plan);
  if (grid) *grid = P->grid;
  if (stages) *stages = (int64_t)P->stages.size();
  if (attn_splits) *attn_splits = P->base.nsplit;
  return NIMF_OK;
}

int nimf_decode_set_timeout_ms(int64_t ms) {
  if (ms < 1 || ms > 600000)
    return set_error(NIMF_ERR_ARG, "decode_set_timeout_ms: %lld not in [1, 600000]", (long long)ms);
  g_dec_wait_ns = (unsigned long long)ms * 1000000ull;
  return NIMF_OK;
}

int nimf_decode_destroy(int64_t plan) {
  DecodePlan* P = find_plan(plan);
  if (!P) return set_error(NIMF_ERR_STATE, "decode_destroy: unknown plan %lld", (long long)plan);
  cudaDeviceSynchronize();
  // a sharded plan's scratch receives the peers' stores: no rank releases it
  // before every rank has finished its last step
  const int rc = P->world > 1 ? comm_barrier() : NIMF_OK;
  free_plan(P);
  g_plans[(size_t)plan - 1] = nullptr;
  return rc;
}

}  // extern "C"
