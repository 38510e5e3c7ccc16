// tc_util.cuh -- tcgen05 / TMA helpers shared by the tensor-core GEMMs
// (q4g_tc.cu, fw_tc.cu): TMEM allocation and loads/stores, kind::f16 MMA with
// A in TMEM, shared-memory and instruction descriptors, tensor-map loads, the
// per-row power-of-two x scale, and the driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

constexpr uint32_t kTmemCols = 512;

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
// D (TMEM, f32) (+)= A (TMEM, f16, K-major) x B^T (smem, f16), M=128, K=16
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// 8 consecutive columns of this thread's TMEM lane <- registers
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
// 32 consecutive columns of this thread's TMEM lane <- registers
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// mbarrier arrive once every earlier tcgen05 operation of this thread is done
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// 16 consecutive columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
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

// Instruction descriptor: f32 accumulate, A and B f16, both K-major,
// M = 128 (output channels); N (x rows, a multiple of 16) is or-ed in.
constexpr uint32_t kIdescF16 = (1u << 4) | (0u << 7) | (0u << 10) | ((128u >> 4) << 24);
__host__ __device__ constexpr uint32_t idesc_n(int n) { return kIdescF16 | ((uint32_t)(n >> 3) << 17); }


// Byte offset of (row r, k) in a K-major canonical tile with `kbytes` of K.
__host__ __device__ __forceinline__ uint32_t canon_off(int r, int k, int kbytes) {
  return (uint32_t)((r >> 3) * (kbytes * 8) + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}

// Per-row power-of-two scale of x: scale[r] = 2^e, inv[r] = 2^-e with the
// row's largest finite magnitude times 2^e in [128, 256) (e = 0 for a zero
// row; |e| <= 126 keeps both factors finite).  One 128-thread block per row.
__global__ void tc_rowscale(const float* __restrict__ x, int64_t ldx, int m, int k,
                                float* __restrict__ scale, float* __restrict__ inv) {
  __shared__ float part[4];
  const int row = blockIdx.x;
  griddep_wait();  // x may be written by the previous kernel in the stream
  const float* xr = x + (size_t)row * ldx;
  float mx = 0.f;
  auto take = [&](float v) {
    v = fabsf(v);
    if (v <= 3.402823466e38f) mx = fmaxf(mx, v);  // skips inf and NaN
  };
  if (((ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0)) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const int k4 = k >> 2;
    for (int i = threadIdx.x; i < k4; i += blockDim.x) {
      const float4 v = __ldg(x4 + i);
      take(v.x);
      take(v.y);
      take(v.z);
      take(v.w);
    }
    for (int i = (k4 << 2) + threadIdx.x; i < k; i += blockDim.x) take(__ldg(xr + i));
  } else {
    for (int i = threadIdx.x; i < k; i += blockDim.x) take(__ldg(xr + i));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    mx = fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3]));
    int ex = 0;
    if (mx > 0.f) frexpf(mx, &ex);  // mx = f 2^ex, f in [0.5, 1)
    const int e = mx > 0.f ? max(-126, min(126, 8 - ex)) : 0;
    scale[row] = ldexpf(1.0f, e);
    inv[row] = ldexpf(1.0f, -e);
  }
  griddep_launch_dependents();
}

// 3-D tensor-map load (no multicast) completing on mbarrier `bar`; x (the
// inner coordinate, in 4-byte elements) is a multiple of 4.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependence on the driver library); nullptr if unavailable.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        p && q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

}  // namespace

}  // namespace nimf
