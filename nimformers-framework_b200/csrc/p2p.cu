// p2p.cu -- one-shot all-gather of N-shard outputs over peer memory (CUDA IPC
// over NVLink / NVSwitch), for the sharded decode: rank r holds output columns
// [r*cols, (r+1)*cols) of every projection (an N-shard of the weight rows,
// row = output channel as in quant.nim) and the next projection needs all of
// them as its x [rows][world*cols].  The reference has no multi-GPU path; the
// exchange replaces an NCCL all-gather plus a layout copy with one kernel.
//
// Each rank owns one cudaMalloc'd buffer, shared with its peers by IPC handle:
//   stage[2][world][slot]        float: rank q's slice lands in stage[par][q]
//   flags[kMaxRanks][kChunks]    uint32: flags[q][ch] = the call count of q's
//                                last push of chunk ch
// Call e (1, 2, ...) of the group uses parity par = e & 1.  The kernel has
// world x kChunks blocks; block (b, ch) moves chunk ch of the slice (a fixed
// split of the slice's float4 units into kChunks ranges) for peer b: it
// pushes this rank's chunk into peer b's stage[par][rank] with plain stores,
// then (after __syncthreads and a system-scope fence) stores e into peer b's
// flags[rank][ch] with release semantics; it then waits, acquire, for its own
// flags[b][ch] >= e and copies that chunk of stage[par][b] into columns
// [b*cols, (b+1)*cols) of dst (block (rank, ch) copies src directly).  Every
// call runs every block, so all per-block call counters stay equal.  Two
// parities make the reuse safe: a rank can write stage[par] of call e + 2
// only after every peer has pushed all chunks of call e + 1, which each peer
// does only after its call e kernel, including the reads of stage[par], has
// completed in stream order.
//
// The wait is bounded (2 s of %globaltimer by default, nimf_p2p_set_timeout_ms
// changes it): on expiry the block sets the
// context's error word (reported by nimf_sync as NIMF_ERR_TIMEOUT), leaves its
// dst columns unwritten and returns; while the word stays set, later waits
// give up at once, so a missing peer costs one bound, not one per call.  No TMA and no multicast: plain peer
// stores and local loads only.
#include <cstdint>
#include <cstring>
#include <vector>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr int kMaxRanks = 8;
constexpr int kChunks = 8;      // blocks per peer
constexpr int kThreads = 256;
// bound of a peer wait, process-wide (nimf_p2p_set_timeout_ms); 2 s by default
unsigned long long g_wait_ns = 2000000000ull;
constexpr int64_t kMaxSlot = (int64_t)1 << 28;          // floats per slice

struct P2PArgs {
  float* stage[kMaxRanks];      // each rank's stage base, as mapped in this process
  unsigned* flags[kMaxRanks];   // each rank's flags base
  unsigned* epoch;              // this rank's per-block call counters [kMaxRanks][kChunks]
  int* err;
  unsigned long long wait_ns;   // bound of the wait for a peer's flag
  int world, rank;
  int64_t slot;                 // floats per stage slot (a multiple of 4)
};

struct P2PGroup {
  int device = -1;
  int world = 0, rank = 0;
  int64_t slot = 0;
  void* base = nullptr;         // own IPC buffer
  unsigned* epoch = nullptr;    // own, not shared
  void* peer_base[kMaxRanks] = {};
  bool connected = false;
};

std::vector<P2PGroup*> g_groups;

size_t stage_bytes(int world, int64_t slot) { return (size_t)2 * world * slot * sizeof(float); }
size_t buffer_bytes(int world, int64_t slot) {
  return stage_bytes(world, slot) + (size_t)kMaxRanks * kChunks * sizeof(unsigned) + 256;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copies units [lo, hi) of a rows x cols slice: unit u is 4 floats (VEC, cols
// a multiple of 4) or 1; `flat` is the contiguous stage copy, `mat` the
// strided matrix (row stride ld).  TO_FLAT: mat -> flat, else flat -> mat.
template <bool VEC, bool TO_FLAT, bool CG>
__device__ __forceinline__ void copy_units(float* flat, const float* matc, float* matw, int cols,
                                           int64_t ld, int lo, int hi) {
  constexpr int W = VEC ? 4 : 1;
  for (int u = lo + (int)threadIdx.x; u < hi; u += kThreads) {
    const int i = u * W;
    const int r = i / cols, c = i - r * cols;
    const int64_t m = (int64_t)r * ld + c;
    if (VEC) {
      if (TO_FLAT) {
        reinterpret_cast<float4*>(flat)[u] = *reinterpret_cast<const float4*>(matc + m);
      } else {
        const float4 v = CG ? __ldcg(reinterpret_cast<const float4*>(flat) + u)
                            : reinterpret_cast<const float4*>(flat)[u];
        *reinterpret_cast<float4*>(matw + m) = v;
      }
    } else {
      if (TO_FLAT) flat[i] = matc[m];
      else matw[m] = CG ? __ldcg(flat + i) : flat[i];
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) p2p_allgather_kernel(const P2PArgs a, const float* src,
                                                                 int rows, int cols,
                                                                 int64_t ld_src, float* dst,
                                                                 int64_t ld_dst) {
  __shared__ unsigned s_e;
  __shared__ int s_ok;
  griddep_launch_dependents();
  griddep_wait();  // src is written by the previous kernel
  const int b = blockIdx.x, ch = blockIdx.y;
  unsigned* ep = a.epoch + b * kChunks + ch;
  if (threadIdx.x == 0) {
    s_e = *ep + 1;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned e = s_e;
  const int par = (int)(e & 1u);
  const int units = rows * cols / (VEC ? 4 : 1);
  const int per = (units + kChunks - 1) / kChunks;
  const int lo = min(units, ch * per), hi = min(units, lo + per);
  float* dcol = dst + (int64_t)b * cols;
  if (b != a.rank) {
    float* to = a.stage[b] + ((int64_t)par * a.world + a.rank) * a.slot;
    copy_units<VEC, true, false>(to, src, nullptr, cols, ld_src, lo, hi);
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      store_release_sys(a.flags[b] + a.rank * kChunks + ch, e);
      // wait for peer b's push of this chunk of this call into our stage[par][b]
      const unsigned* mine = a.flags[a.rank] + b * kChunks + ch;
      const unsigned long long t0 = globaltimer();
      while ((int)(load_acquire_sys(mine) - e) < 0) {
        // an earlier expired wait (error word still set) fails this one at once
        if (globaltimer() - t0 > a.wait_ns || *(volatile int*)a.err != 0) {
          s_ok = 0;
          atomicExch(a.err, 1);
          break;
        }
        __nanosleep(32);
      }
      *ep = e;
    }
    __syncthreads();
    if (!s_ok) return;
    float* from = a.stage[a.rank] + ((int64_t)par * a.world + b) * a.slot;
    copy_units<VEC, false, true>(from, nullptr, dcol, cols, ld_dst, lo, hi);
  } else {
    // own columns: src -> dst directly (unit u of the slice, both strided)
    constexpr int W = VEC ? 4 : 1;
    for (int u = lo + (int)threadIdx.x; u < hi; u += kThreads) {
      const int i = u * W;
      const int r = i / cols, c = i - r * cols;
      if (VEC)
        *reinterpret_cast<float4*>(dcol + (int64_t)r * ld_dst + c) =
            *reinterpret_cast<const float4*>(src + (int64_t)r * ld_src + c);
      else
        dcol[(int64_t)r * ld_dst + c] = src[(int64_t)r * ld_src + c];
    }
    if (threadIdx.x == 0) *ep = e;
  }
}

P2PGroup* find_group(int64_t id) {
  if (id < 1 || id > (int64_t)g_groups.size()) return nullptr;
  return g_groups[(size_t)id - 1];
}

}  // namespace

void release_p2p_groups() {
  for (P2PGroup*& g : g_groups) {
    if (!g) continue;
    for (int q = 0; q < g->world; ++q)
      if (q != g->rank && g->peer_base[q]) cudaIpcCloseMemHandle(g->peer_base[q]);
    if (g->base) cudaFree(g->base);
    if (g->epoch) cudaFree(g->epoch);
    delete g;
    g = nullptr;
  }
  g_groups.clear();
}

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_p2p_create(int world, int rank, int64_t slot_floats, void* ipc_handle_out,
                    int64_t* group) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (world < 2 || world > kMaxRanks || rank < 0 || rank >= world || slot_floats < 1 ||
      slot_floats > kMaxSlot)
    return set_error(NIMF_ERR_SHAPE, "p2p_create: world %d rank %d slot %lld", world, rank,
                     (long long)slot_floats);
  if (!ipc_handle_out || !group) return set_error(NIMF_ERR_ARG, "p2p_create: NULL argument");
  P2PGroup* g = new P2PGroup();
  g->device = c->device;
  g->world = world;
  g->rank = rank;
  g->slot = (slot_floats + 3) / 4 * 4;  // 16-byte aligned slots
  cudaError_t e1 = cudaMalloc(&g->base, buffer_bytes(world, g->slot));
  cudaError_t e2 = e1 == cudaSuccess ? cudaMalloc((void**)&g->epoch, kMaxRanks * kChunks * sizeof(unsigned)) : e1;
  if (e2 == cudaSuccess) e2 = cudaMemset(g->base, 0, buffer_bytes(world, g->slot));
  if (e2 == cudaSuccess) e2 = cudaMemset(g->epoch, 0, kMaxRanks * kChunks * sizeof(unsigned));
  cudaIpcMemHandle_t h;
  if (e2 == cudaSuccess) e2 = cudaIpcGetMemHandle(&h, g->base);
  if (e2 == cudaSuccess) e2 = cudaDeviceSynchronize();
  if (e2 != cudaSuccess) {
    if (g->base) cudaFree(g->base);
    if (g->epoch) cudaFree(g->epoch);
    delete g;
    return set_error(NIMF_ERR_CUDA, "p2p_create: %s", cudaGetErrorString(e2));
  }
  memcpy(ipc_handle_out, &h, sizeof(h));
  g_groups.push_back(g);
  *group = (int64_t)g_groups.size();
  return NIMF_OK;
}

int nimf_p2p_connect(int64_t group, const void* ipc_handles) {
  P2PGroup* g = find_group(group);
  if (!g) return set_error(NIMF_ERR_STATE, "p2p_connect: unknown group %lld", (long long)group);
  if (!ipc_handles) return set_error(NIMF_ERR_ARG, "p2p_connect: NULL handles");
  if (g->connected) return set_error(NIMF_ERR_STATE, "p2p_connect: group already connected");
  const cudaIpcMemHandle_t* hs = static_cast<const cudaIpcMemHandle_t*>(ipc_handles);
  for (int q = 0; q < g->world; ++q) {
    if (q == g->rank) {
      g->peer_base[q] = g->base;
      continue;
    }
    cudaError_t e = cudaIpcOpenMemHandle(&g->peer_base[q], hs[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      g->peer_base[q] = nullptr;
      return set_error(NIMF_ERR_CUDA, "p2p_connect: peer %d: %s", q, cudaGetErrorString(e));
    }
  }
  g->connected = true;
  return NIMF_OK;
}

int nimf_p2p_connect_comm(int64_t group) {
  P2PGroup* g = find_group(group);
  if (!g) return set_error(NIMF_ERR_STATE, "p2p_connect_comm: unknown group %lld", (long long)group);
  int world = 1, rank = 0;
  NIMF_TRY(comm_world(&world, &rank));
  if (world != g->world || rank != g->rank)
    return set_error(NIMF_ERR_STATE,
                     "p2p_connect_comm: group is rank %d of %d, the communicator rank %d of %d",
                     g->rank, g->world, rank, world);
  cudaIpcMemHandle_t mine;
  NIMF_CUDA_TRY(cudaIpcGetMemHandle(&mine, g->base));
  std::vector<cudaIpcMemHandle_t> all((size_t)world);
  NIMF_TRY(comm_allgather_bytes(&mine, sizeof(mine), all.data()));
  return nimf_p2p_connect(group, all.data());
}

int nimf_p2p_allgather_dev(int64_t group, const float* src, int64_t rows, int64_t cols,
                           int64_t ld_src, float* dst, int64_t ld_dst, void* stream) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  P2PGroup* g = find_group(group);
  if (!g || !g->connected) return set_error(NIMF_ERR_STATE, "p2p_allgather: group %lld not connected", (long long)group);
  if (g->device != c->device) return set_error(NIMF_ERR_STATE, "p2p_allgather: group of device %d used on %d", g->device, c->device);
  if (rows < 0 || cols < 0 || rows * cols > g->slot || ld_src < cols || ld_dst < (int64_t)g->world * cols)
    return set_error(NIMF_ERR_SHAPE, "p2p_allgather: rows %lld cols %lld ld_src %lld ld_dst %lld (slot %lld floats, world %d)",
                     (long long)rows, (long long)cols, (long long)ld_src, (long long)ld_dst,
                     (long long)g->slot, g->world);
  if ((rows * cols > 0) && (!src || !dst)) return set_error(NIMF_ERR_ARG, "p2p_allgather: NULL buffer");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  P2PArgs a = {};
  for (int q = 0; q < g->world; ++q) {
    a.stage[q] = static_cast<float*>(g->peer_base[q]);
    a.flags[q] = reinterpret_cast<unsigned*>(static_cast<char*>(g->peer_base[q]) + stage_bytes(g->world, g->slot));
  }
  a.epoch = g->epoch;
  a.err = c->dev_err;
  a.wait_ns = g_wait_ns;
  a.world = g->world;
  a.rank = g->rank;
  a.slot = g->slot;
  // every call takes part in the exchange (the peers count calls), even an empty one
  const bool vec = (cols % 4 == 0) && (ld_src % 4 == 0) && (ld_dst % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g->world, kChunks);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec)
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, p2p_allgather_kernel<true>, a, src, (int)rows, (int)cols,
                                     ld_src, dst, ld_dst));
  else
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, p2p_allgather_kernel<false>, a, src, (int)rows,
                                     (int)cols, ld_src, dst, ld_dst));
  return NIMF_OK;
}

int nimf_p2p_set_timeout_ms(int64_t ms) {
  if (ms < 1 || ms > 600000)
    return set_error(NIMF_ERR_ARG, "p2p_set_timeout_ms: %lld not in [1, 600000]", (long long)ms);
  g_wait_ns = (unsigned long long)ms * 1000000ull;
  return NIMF_OK;
}

int nimf_p2p_destroy(int64_t group) {
  P2PGroup* g = find_group(group);
  if (!g) return set_error(NIMF_ERR_STATE, "p2p_destroy: unknown group %lld", (long long)group);
  cudaDeviceSynchronize();
  for (int q = 0; q < g->world; ++q)
    if (q != g->rank && g->peer_base[q]) cudaIpcCloseMemHandle(g->peer_base[q]);
  cudaFree(g->base);
  cudaFree(g->epoch);
  delete g;
  g_groups[(size_t)group - 1] = nullptr;
  return NIMF_OK;
}

}  // extern "C"
