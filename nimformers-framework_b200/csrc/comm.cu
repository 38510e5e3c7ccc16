// comm.cu -- the library's own multi-GPU plumbing: an NCCL communicator (one
// process per GPU), the output all-gather of N-sharded weights, and the
// exchange of CUDA IPC handles that the peer-memory paths (p2p.cu, the
// sharded decode plan in decode.cu) need.
//
// The reference has no multi-GPU path (its CUDA device is fixed at 0,
// vendor/bybylang/backends/cuda/cuda_driver.nim:183).  The sharding follows
// the reference's weight layout, row = output channel (nimformer.nim:90): a
// shard is a contiguous range of whole 16-row tiles (shard_range below, the
// same rule as the host mirror's shard_rows), so every rank can compute every
// other rank's range without asking.
//
// NCCL is opened at run time (dlopen of libnccl.so.2): the library loads and
// runs on one GPU where NCCL is absent, and a process that already loaded
// NCCL (torch does) shares that copy.  Calls follow the library's error
// convention: NIMF_ERR_NCCL with NCCL's message, no fallback.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*get_version)(int*) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

struct Comm {
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0, device = -1;
  // all-gather scratch: this rank's padded slice and the gathered slices
  void* send = nullptr;
  size_t send_bytes = 0;
  void* recv = nullptr;
  size_t recv_bytes = 0;
  void* small = nullptr;  // 64 KB for handle exchanges and the barrier
};

Comm g_comm;
constexpr size_t kSmallBytes = 64 * 1024;

int load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.lib) return NIMF_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return set_error(NIMF_ERR_UNSUPPORTED, "NCCL is not available: %s", dlerror());
  NcclApi a;
  a.lib = h;
  a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
  a.init_rank = (decltype(a.init_rank))dlsym(h, "ncclCommInitRank");
  a.destroy = (decltype(a.destroy))dlsym(h, "ncclCommDestroy");
  a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
  a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
  a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
  a.get_version = (decltype(a.get_version))dlsym(h, "ncclGetVersion");
  if (!a.get_unique_id || !a.init_rank || !a.destroy || !a.all_gather || !a.all_reduce ||
      !a.error_string)
    return set_error(NIMF_ERR_UNSUPPORTED, "libnccl.so.2 lacks a required entry point");
  g_nccl = a;
  return NIMF_OK;
}

#define NIMF_NCCL_TRY(expr)                                                                  \
  do {                                                                                       \
    ncclResult_t r__ = (expr);                                                               \
    if (r__ != ncclSuccess)                                                                  \
      return ::nimf::set_error(NIMF_ERR_NCCL, "%s failed: %s", #expr,                       \
                               g_nccl.error_string ? g_nccl.error_string(r__) : "?");        \
  } while (0)

int require_comm(Context** c) {
  NIMF_TRY(require_ctx(c));
  if (!g_comm.comm) return set_error(NIMF_ERR_STATE, "no communicator: call nimf_comm_init first");
  if (g_comm.device != (*c)->device)
    return set_error(NIMF_ERR_STATE, "communicator of device %d used on %d", g_comm.device,
                     (*c)->device);
  return NIMF_OK;
}

int grow_buf(void** p, size_t* have, size_t bytes, cudaStream_t st) {
  if (*have >= bytes) return NIMF_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone)
    return set_error(NIMF_ERR_STATE,
                     "sharded matmul: the gather buffer must grow (%zu bytes), which cannot happen "
                     "during stream capture; run the call once before capturing",
                     bytes);
  NIMF_CUDA_TRY(cudaStreamSynchronize(st));
  device_free(*p);
  *p = nullptr;
  *have = 0;
  NIMF_TRY(device_alloc(p, bytes));
  *have = bytes;
  return NIMF_OK;
}

struct RowTable {
  int64_t r0[kCommMaxRanks + 1];
};

// y[r][t.r0[q] + c] = g[q][r][c]: rank q's slice of the padded gather buffer
// g [world][m][pad] laid out as rows of the full output.  The row table is a
// kernel argument, so a captured call replays with its own values.
__global__ void gather_layout_kernel(const float* __restrict__ g, int64_t m, int64_t pad,
                                     int64_t n_full, const RowTable t, int world,
                                     float* __restrict__ y) {
  const int64_t total = m * n_full;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n_full, col = i - r * n_full;
    int q = 0;
    while (q + 1 < world && col >= t.r0[q + 1]) ++q;
    y[i] = g[((int64_t)q * m + r) * pad + (col - t.r0[q])];
  }
}

}  // namespace

void shard_range(int64_t n, int world, int rank, int64_t* r0, int64_t* r1) {
  const int64_t tiles = (n + 15) / 16;
  const int64_t t0 = tiles * rank / world, t1 = tiles * (rank + 1) / world;
  *r0 = std::min(n, t0 * 16);
  *r1 = std::min(n, t1 * 16);
}

int comm_world(int* world, int* rank) {
  if (!g_comm.comm) {
    *world = 1;
    *rank = 0;
    return NIMF_OK;
  }
  *world = g_comm.world;
  *rank = g_comm.rank;
  return NIMF_OK;
}

int comm_allgather_bytes(const void* src, size_t bytes, void* dst_host) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  if (bytes * (size_t)g_comm.world > kSmallBytes)
    return set_error(NIMF_ERR_SHAPE, "handle exchange of %zu bytes per rank is too large", bytes);
  char* s = (char*)g_comm.small;
  NIMF_CUDA_TRY(cudaMemcpyAsync(s, src, bytes, cudaMemcpyHostToDevice, c->stream));
  NIMF_NCCL_TRY(g_nccl.all_gather(s, s + bytes, bytes, ncclChar, g_comm.comm, c->stream));
  NIMF_CUDA_TRY(cudaMemcpyAsync(dst_host, s + bytes, bytes * g_comm.world, cudaMemcpyDeviceToHost,
                                c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return NIMF_OK;
}

int comm_share_buffer(void* local, void** peers) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  cudaIpcMemHandle_t mine;
  NIMF_CUDA_TRY(cudaIpcGetMemHandle(&mine, local));
  std::vector<cudaIpcMemHandle_t> all((size_t)g_comm.world);
  NIMF_TRY(comm_allgather_bytes(&mine, sizeof(mine), all.data()));
  for (int q = 0; q < kCommMaxRanks; ++q) peers[q] = nullptr;
  for (int q = 0; q < g_comm.world; ++q) {
    if (q == g_comm.rank) {
      peers[q] = local;
      continue;
    }
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, all[(size_t)q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < q; ++j)
        if (j != g_comm.rank && peers[j]) cudaIpcCloseMemHandle(peers[j]);
      return set_error(NIMF_ERR_CUDA, "cudaIpcOpenMemHandle of rank %d: %s", q,
                       cudaGetErrorString(e));
    }
    peers[q] = p;
  }
  return NIMF_OK;
}

void comm_unshare_buffer(void** peers, int world, int rank) {
  for (int q = 0; q < world; ++q) {
    if (q != rank && peers[q]) cudaIpcCloseMemHandle(peers[q]);
    peers[q] = nullptr;
  }
}

int comm_barrier() {
  Context* c;
  NIMF_TRY(require_comm(&c));
  int* s = (int*)g_comm.small;
  NIMF_NCCL_TRY(g_nccl.all_reduce(s, s, 1, ncclInt32, ncclSum, g_comm.comm, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return NIMF_OK;
}

int comm_agree(int ok, int* all_ok) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  int* s = (int*)g_comm.small;
  const int v = ok ? 1 : 0;
  NIMF_CUDA_TRY(cudaMemcpyAsync(s, &v, sizeof(int), cudaMemcpyHostToDevice, c->stream));
  NIMF_NCCL_TRY(g_nccl.all_reduce(s, s, 1, ncclInt32, ncclMin, g_comm.comm, c->stream));
  int r = 0;
  NIMF_CUDA_TRY(cudaMemcpyAsync(&r, s, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  NIMF_CUDA_TRY(cudaStreamSynchronize(c->stream));
  *all_ok = r;
  return NIMF_OK;
}

void release_gathers();

void release_comm() {
  release_gathers();
  if (g_comm.comm) {
    g_nccl.destroy(g_comm.comm);
    device_free(g_comm.send);
    device_free(g_comm.recv);
    device_free(g_comm.small);
  }
  g_comm = Comm();
}

int weight_shard_check(const Weight* w, int world, int rank, int64_t* n_full) {
  const int64_t n = w->n_full > 0 ? w->n_full : w->rows();
  int64_t r0, r1;
  shard_range(n, world, rank, &r0, &r1);
  if (w->row_begin != r0 || w->rows() != r1 - r0)
    return set_error(NIMF_ERR_SHAPE,
                     "sharded matmul: this rank holds rows [%lld, %lld) of %lld; rank %d of %d "
                     "must hold [%lld, %lld) (whole 16-row tiles, sizes within one tile)",
                     (long long)w->row_begin, (long long)(w->row_begin + w->rows()), (long long)n,
                     rank, world, (long long)r0, (long long)r1);
  *n_full = n;
  return NIMF_OK;
}

// A buffer shared by every rank (same size, same offsets) that gathering
// GEMVs store their N-shard outputs into, plus its control words.
struct GatherGroup {
  int device = -1, world = 1, rank = 0;
  void* base = nullptr;
  size_t bytes = 0;             // usable bytes (the control words follow)
  void* peers[kCommMaxRanks] = {};
};
std::vector<GatherGroup*> g_gathers;
unsigned long long g_gather_wait_ns = 2000000000ull;

GatherGroup* find_gather(int64_t id) {
  if (id < 1 || id > (int64_t)g_gathers.size()) return nullptr;
  return g_gathers[(size_t)id - 1];
}

void free_gather(GatherGroup* g) {
  if (!g) return;
  comm_unshare_buffer(g->peers, g->world, g->rank);
  device_free(g->base);
  delete g;
}

void release_gathers() {
  for (GatherGroup*& g : g_gathers) {
    free_gather(g);
    g = nullptr;
  }
  g_gathers.clear();
}

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_comm_unique_id(void* id_out) {
  if (!id_out) return set_error(NIMF_ERR_ARG, "comm_unique_id: NULL output");
  NIMF_TRY(load_nccl());
  ncclUniqueId id;
  NIMF_NCCL_TRY(g_nccl.get_unique_id(&id));
  std::memcpy(id_out, &id, sizeof(id));
  return NIMF_OK;
}

int nimf_comm_init(int world, int rank, const void* id) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!id) return set_error(NIMF_ERR_ARG, "comm_init: NULL id");
  if (world < 1 || world > kCommMaxRanks || rank < 0 || rank >= world)
    return set_error(NIMF_ERR_ARG, "comm_init: rank %d of world %d (world at most %d)", rank, world,
                     kCommMaxRanks);
  if (g_comm.comm) return set_error(NIMF_ERR_STATE, "comm_init: a communicator already exists");
  NIMF_TRY(load_nccl());
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  Comm cm;
  cm.world = world;
  cm.rank = rank;
  cm.device = c->device;
  NIMF_CUDA_TRY(cudaSetDevice(c->device));
  NIMF_NCCL_TRY(g_nccl.init_rank(&cm.comm, world, uid, rank));
  int rc = device_alloc(&cm.small, kSmallBytes);
  if (rc != NIMF_OK) {
    g_nccl.destroy(cm.comm);
    return rc;
  }
  g_comm = cm;
  return NIMF_OK;
}

int nimf_comm_info(int* world, int* rank) {
  if (!world || !rank) return set_error(NIMF_ERR_ARG, "comm_info: NULL output");
  return comm_world(world, rank);
}

int nimf_comm_allgather_dev(const void* src, int64_t bytes, void* dst, void* stream) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  if (bytes < 0) return set_error(NIMF_ERR_SHAPE, "comm_allgather: bytes < 0");
  if (bytes == 0) return NIMF_OK;
  if (!src || !dst) return set_error(NIMF_ERR_ARG, "comm_allgather: NULL buffer");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  NIMF_NCCL_TRY(g_nccl.all_gather(src, dst, (size_t)bytes, ncclChar, g_comm.comm, st));
  return NIMF_OK;
}

int nimf_comm_barrier(void) { return comm_barrier(); }

int nimf_comm_destroy(void) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  if (!g_comm.comm) return NIMF_OK;
  cudaStreamSynchronize(c->stream);
  cudaDeviceSynchronize();
  release_comm();
  return NIMF_OK;
}

int nimf_matmul_w_allgather_dev(nimf_weight_t h, const float* x_dev, int64_t m, float* y_dev,
                                void* stream) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  Weight* w = lookup(h);
  if (!w) return set_error(NIMF_ERR_STATE, "unknown weight handle %llu", (unsigned long long)h);
  if (m < 0) return set_error(NIMF_ERR_SHAPE, "m < 0");
  const int world = g_comm.world, rank = g_comm.rank;
  int64_t n_full;
  NIMF_TRY(weight_shard_check(w, world, rank, &n_full));
  if (m == 0 || n_full == 0) return NIMF_OK;
  if (!y_dev || (!x_dev && w->k() > 0)) return set_error(NIMF_ERR_ARG, "NULL x or y");
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  RowTable t;
  int64_t pad = 0;
  bool equal = true;
  for (int q = 0; q < world; ++q) {
    int64_t a, b;
    shard_range(n_full, world, q, &a, &b);
    t.r0[q] = a;
    pad = std::max(pad, b - a);
    if (q > 0 && b - a != t.r0[1] - t.r0[0]) equal = false;
  }
  t.r0[world] = n_full;
  if (m == 1 && equal) {
    // slices land in place: rank q's rows are y[q * pad, (q + 1) * pad)
    float* mine = y_dev + (size_t)rank * pad;
    if (w->rows() > 0) NIMF_TRY(weight_matmul_dev(w, x_dev, 1, mine, st));
    NIMF_NCCL_TRY(g_nccl.all_gather(mine, y_dev, (size_t)pad, ncclFloat, g_comm.comm, st));
    return NIMF_OK;
  }
  const size_t slice = (size_t)m * pad * 4;
  NIMF_TRY(grow_buf(&g_comm.send, &g_comm.send_bytes, slice + 256, st));
  NIMF_TRY(grow_buf(&g_comm.recv, &g_comm.recv_bytes, slice * world + 256, st));
  float* send = (float*)g_comm.send;
  if (w->rows() > 0) {
    if (w->rows() == pad) {
      NIMF_TRY(weight_matmul_dev(w, x_dev, m, send, st));
    } else {
      // a shorter slice: rows [rows, pad) of each x row stay unused
      NIMF_TRY(weight_matmul_dev(w, x_dev, m, (float*)g_comm.recv, st));
      NIMF_CUDA_TRY(cudaMemcpy2DAsync(send, (size_t)pad * 4, g_comm.recv, (size_t)w->rows() * 4,
                                      (size_t)w->rows() * 4, (size_t)m, cudaMemcpyDeviceToDevice, st));
    }
  }
  NIMF_NCCL_TRY(g_nccl.all_gather(send, g_comm.recv, (size_t)m * pad, ncclFloat, g_comm.comm, st));
  const int64_t total = m * n_full;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)c->num_sms * 8);
  gather_layout_kernel<<<blocks, 256, 0, st>>>((const float*)g_comm.recv, m, pad, n_full, t, world,
                                               y_dev);
  NIMF_CUDA_TRY(cudaGetLastError());
  return NIMF_OK;
}

int nimf_gather_create(int64_t bytes, int64_t* group, void** buffer_dev) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  int rc = NIMF_OK;
  if (!group || !buffer_dev) rc = set_error(NIMF_ERR_ARG, "gather_create: NULL output");
  else if (bytes < 0 || bytes > ((int64_t)1 << 36))
    rc = set_error(NIMF_ERR_SHAPE, "gather_create: %lld bytes", (long long)bytes);
  GatherGroup* g = nullptr;
  if (rc == NIMF_OK) {
    g = new GatherGroup();
    g->device = c->device;
    g->world = g_comm.world;
    g->rank = g_comm.rank;
    g->bytes = ((size_t)bytes + 255) / 256 * 256;
    rc = device_alloc(&g->base, g->bytes + 256);
    if (rc == NIMF_OK) {
      cudaError_t e = cudaMemset(g->base, 0, g->bytes + 256);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess) rc = set_error(NIMF_ERR_CUDA, "gather_create: %s", cudaGetErrorString(e));
    }
  }
  // every rank learns whether all of them got this far before the exchange
  int ok_all = 0;
  const int rc_agree = comm_agree(rc == NIMF_OK, &ok_all);
  if (rc == NIMF_OK && rc_agree != NIMF_OK) rc = rc_agree;
  if (rc == NIMF_OK && !ok_all) rc = set_error(NIMF_ERR_STATE, "gather_create: another rank failed");
  if (rc == NIMF_OK) rc = comm_share_buffer(g->base, g->peers);
  if (rc != NIMF_OK) {
    if (g) {
      device_free(g->base);
      delete g;
    }
    return rc;
  }
  g_gathers.push_back(g);
  *group = (int64_t)g_gathers.size();
  *buffer_dev = g->base;
  return NIMF_OK;
}

int nimf_matmul_w_group_gather_dev(int64_t group, const nimf_weight_t* handles, int count,
                                   const float* x_dev, int64_t m, float* const* y_devs,
                                   void* stream) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  GatherGroup* g = find_gather(group);
  if (!g) return set_error(NIMF_ERR_STATE, "group_gather: unknown group %lld", (long long)group);
  if (g->device != c->device)
    return set_error(NIMF_ERR_STATE, "group_gather: group of device %d used on %d", g->device,
                     c->device);
  if (count < 1 || count > 16 || m < 1 || m > 8)
    return set_error(NIMF_ERR_SHAPE, "group_gather: %d weights (1 .. 16), %lld rows of x (1 .. 8)",
                     count, (long long)m);
  if (!handles || !y_devs || !x_dev) return set_error(NIMF_ERR_ARG, "group_gather: NULL argument");
  const Q4GWeight* qs[16];
  float* ys[16];
  int64_t lds[16];
  const char* lo = (const char*)g->base;
  for (int i = 0; i < count; ++i) {
    Weight* w = lookup(handles[i]);
    if (!w) return set_error(NIMF_ERR_STATE, "group_gather: unknown weight handle");
    if (w->kind != NIMF_KIND_INT4_ASYM || w->kperm)
      return set_error(NIMF_ERR_UNSUPPORTED, "group_gather: int4 group weights without act order only");
    int64_t n_full;
    NIMF_TRY(weight_shard_check(w, g->world, g->rank, &n_full));
    const char* y = (const char*)y_devs[i];
    if (!y || y < lo || y + (size_t)m * n_full * 4 > lo + g->bytes || ((uintptr_t)y & 3))
      return set_error(NIMF_ERR_ARG,
                       "group_gather: output %d must lie inside the group's buffer (%zu bytes)", i,
                       g->bytes);
    qs[i] = &w->q4;
    ys[i] = y_devs[i] + w->row_begin;
    lds[i] = n_full;
  }
  GatherSpec spec;
  spec.world = g->world;
  for (int q = 0; q < g->world; ++q) spec.peer_off[q] = (long long)((char*)g->peers[q] - (char*)g->base);
  spec.ctl = (unsigned*)((char*)g->base + g->bytes);
  spec.wait_ns = g_gather_wait_ns;
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  return q4g_gemv_group_gather(qs, count, x_dev, m, ys, lds, spec, st);
}

int nimf_gather_set_timeout_ms(int64_t ms) {
  if (ms < 1 || ms > 600000)
    return set_error(NIMF_ERR_ARG, "gather_set_timeout_ms: %lld not in [1, 600000]", (long long)ms);
  g_gather_wait_ns = (unsigned long long)ms * 1000000ull;
  return NIMF_OK;
}

int nimf_gather_destroy(int64_t group) {
  Context* c;
  NIMF_TRY(require_comm(&c));
  GatherGroup* g = find_gather(group);
  if (!g) return set_error(NIMF_ERR_STATE, "gather_destroy: unknown group %lld", (long long)group);
  cudaDeviceSynchronize();
  // peers store into this buffer: no rank releases it before all are done
  const int rc = comm_barrier();
  free_gather(g);
  g_gathers[(size_t)group - 1] = nullptr;
  return rc;
}

int nimf_shard_range(int64_t n, int world, int rank, int64_t* row_begin, int64_t* row_end) {
  if (!row_begin || !row_end) return set_error(NIMF_ERR_ARG, "shard_range: NULL output");
  if (n < 0 || world < 1 || rank < 0 || rank >= world)
    return set_error(NIMF_ERR_ARG, "shard_range: rank %d of world %d, n %lld", rank, world,
                     (long long)n);
  shard_range(n, world, rank, row_begin, row_end);
  return NIMF_OK;
}

}  // extern "C"
