// glue.cu -- the element-wise and attention steps between the linears of a
// Llama-style decode step (nim_inference.nim), kept on the device so that the
// activations never return to the host between the quantised matmuls:
//   RMSNorm          nim_inference.nim:114-200 (rmsNormPrep + forward)
//   LayerNorm        nimformer.nim:188-197, CPU path gpubackend.nim:252-266
//   residual add     beAdd (backend.nim) as used by TransformerBlockLlama
//   SwiGLU gating    nim_inference.nim:336-356, sigmoid as gpubackend.nim:111-114
//   RoPE             nim_inference.nim:261-330 (rotate-half, caller's tables)
//   decode attention nim_inference.nim:624-748 with appendKV :404-426 and
//                    softmax as gpubackend.nim:236-250
//   token embedding  cpuEmbeddingLookup, gpubackend.nim:268-278
//   greedy choice    sampleTopP with temperature <= 0, nim_inference.nim:1019-1036
// Every product and sum that the reference rounds separately is rounded
// separately here (__fmul_rn / __fadd_rn, no contraction); reductions (row
// sums, dot products, softmax sums) run in a tree order instead of the
// reference's sequential order.
#include <algorithm>
#include <climits>
#include <cstdint>

#include "device_util.cuh"
#include "nimf_internal.h"

namespace nimf {

namespace {

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float t = sh[0];
  for (int i = 1; i < nw; ++i) t = fmaxf(t, sh[i]);
  return t;
}

// y = (x * inv) * w with inv = 1 / sqrt(sum x^2 / cols + eps); one block per
// row.  With a residual (r != nullptr) x is first replaced by x + r, written
// to h (the residual stream), and normalised.
__global__ void rmsnorm_kernel(const float* __restrict__ x0, const float* __restrict__ r,
                               float* __restrict__ h, const float* __restrict__ w, int64_t cols,
                               float eps, float* __restrict__ y) {
  __shared__ float sh[32];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t off = (int64_t)blockIdx.x * cols;
  const int64_t step = blockDim.x;
  if (cols <= 4 * step) {
    // the row fits in four values per thread: one read of x (and r), the
    // values stay in registers between the sum and the scaling
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = threadIdx.x + u * step;
      v[u] = 0.f;
      if (c < cols) {
        float a = x0[off + c];
        if (r) {
          a = __fadd_rn(a, r[off + c]);
          h[off + c] = a;
        }
        v[u] = a;
      }
    }
    float s = __fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])),
                        __fadd_rn(__fmul_rn(v[2], v[2]), __fmul_rn(v[3], v[3])));
    s = block_sum(s, sh);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)cols), eps)));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = threadIdx.x + u * step;
      if (c < cols) y[off + c] = __fmul_rn(__fmul_rn(v[u], inv), w[c]);
    }
    return;
  }
  if (r) {
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) h[off + c] = __fadd_rn(x0[off + c], r[off + c]);
    __syncthreads();  // each thread reads back only what it wrote; the fence orders it for the block
  }
  const float* xr = (r ? h : x0) + off;
  float* yr = y + off;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t c = threadIdx.x;
  for (; c + 3 * step < cols; c += 4 * step) {
    const float v0 = xr[c], v1 = xr[c + step], v2 = xr[c + 2 * step], v3 = xr[c + 3 * step];
    s4[0] = __fadd_rn(s4[0], __fmul_rn(v0, v0));
    s4[1] = __fadd_rn(s4[1], __fmul_rn(v1, v1));
    s4[2] = __fadd_rn(s4[2], __fmul_rn(v2, v2));
    s4[3] = __fadd_rn(s4[3], __fmul_rn(v3, v3));
  }
  for (; c < cols; c += step) s4[0] = __fadd_rn(s4[0], __fmul_rn(xr[c], xr[c]));
  float s = __fadd_rn(__fadd_rn(s4[0], s4[1]), __fadd_rn(s4[2], s4[3]));
  s = block_sum(s, sh);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)cols), eps)));
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = __fmul_rn(__fmul_rn(xr[c], inv), w[c]);
}

// LayerNorm, one block per row, two passes over the row as the reference's CPU
// path: mean = sum x / cols, then var = sum (x - mean)^2 / cols (not
// E[x^2] - mean^2), y = ((x - mean) * invStd) * gamma + beta.  A row of up to
// 4 * blockDim values is read once and kept in registers for both passes.
__global__ void layernorm_kernel(const float* x, const float* __restrict__ gm,
                                 const float* __restrict__ bt, int64_t cols, float eps,
                                 float* y) {  // x and y may alias (each thread reads its values before writing them)
  __shared__ float sh[32];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t off = (int64_t)blockIdx.x * cols;
  const float* xr = x + off;
  float* yr = y + off;
  const int64_t step = blockDim.x;
  const float fc = (float)cols;
  if (cols <= 4 * step) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = threadIdx.x + u * step;
      v[u] = c < cols ? xr[c] : 0.f;
    }
    float s = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
    const float mean = __fdiv_rn(block_sum(s, sh), fc);
    float d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) d[u] = threadIdx.x + u * step < cols ? __fsub_rn(v[u], mean) : 0.f;
    float q = __fadd_rn(__fadd_rn(__fmul_rn(d[0], d[0]), __fmul_rn(d[1], d[1])),
                        __fadd_rn(__fmul_rn(d[2], d[2]), __fmul_rn(d[3], d[3])));
    const float var = __fdiv_rn(block_sum(q, sh), fc);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = threadIdx.x + u * step;
      if (c < cols) yr[c] = __fadd_rn(__fmul_rn(__fmul_rn(d[u], inv), gm[c]), bt[c]);
    }
    return;
  }
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += step) s = __fadd_rn(s, xr[c]);
  const float mean = __fdiv_rn(block_sum(s, sh), fc);
  float q = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += step) {
    const float dv = __fsub_rn(xr[c], mean);
    q = __fadd_rn(q, __fmul_rn(dv, dv));
  }
  const float var = __fdiv_rn(block_sum(q, sh), fc);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t c = threadIdx.x; c < cols; c += step)
    yr[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[c], mean), inv), gm[c]), bt[c]);
}

// Token embedding rows: out[i][:] = table[ids[i]][:], zeros for an id outside
// [0, vocab).  One block per id; float4 copies when dim allows.
__global__ void __launch_bounds__(1024) embedding_kernel(const float* __restrict__ table, int64_t vocab, int64_t dim,
                                 const int32_t* __restrict__ ids, float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t id = ids[blockIdx.x];
  float* o = out + (int64_t)blockIdx.x * dim;
  const bool ok = id >= 0 && id < vocab;
  const float* src = table + (ok ? id : 0) * dim;
  if ((dim & 3) == 0 && ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t j = threadIdx.x; j < dim / 4; j += blockDim.x)
      reinterpret_cast<float4*>(o)[j] = ok ? reinterpret_cast<const float4*>(src)[j] : z;
  } else {
    for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) o[j] = ok ? src[j] : 0.f;
  }
}

constexpr int kGreedyMaxRecent = 2048;  // with a 32 KB bitmap: 40 KB of static + dynamic shared memory

// Greedy token choice of one row of logits with the repetition penalty: every
// occurrence of an id in the row's recent list divides its logit by `penalty`
// if it is positive at that moment, else multiplies it (so an id listed twice
// is adjusted twice, in sequence); then the first index of the largest
// adjusted value wins.  As in a sequential scan with a strict `>` that starts
// at index 0, NaNs never win, and a NaN at index 0 gives 0.  One block per
// row; recent ids are marked in a shared bitmap so the scan skips their raw
// values.
__global__ void __launch_bounds__(1024) greedy_kernel(const float* __restrict__ logits, int64_t vocab,
                              const int32_t* __restrict__ recent, int nrec, float penalty,
                              int32_t* __restrict__ out_ids) {
  extern __shared__ unsigned gbits[];                 // [ceil(vocab / 32)] bitmap
  __shared__ int srec[kGreedyMaxRecent];
  __shared__ float sv[32];
  __shared__ int si[32];
  griddep_launch_dependents();
  griddep_wait();
  const float* lr = logits + (int64_t)blockIdx.x * vocab;
  const int32_t* rr = recent + (int64_t)blockIdx.x * nrec;
  const bool pen = penalty != 1.0f && nrec > 0;
  const int nwords = (int)((vocab + 31) / 32);
  if (pen) {
    for (int i = threadIdx.x; i < nwords; i += blockDim.x) gbits[i] = 0u;
    for (int r = threadIdx.x; r < nrec; r += blockDim.x) srec[r] = rr[r];
  }
  __syncthreads();
  if (pen)
    for (int r = threadIdx.x; r < nrec; r += blockDim.x) {
      const int id = srec[r];
      if (id >= 0 && id < vocab) atomicOr(&gbits[id >> 5], 1u << (id & 31));
    }
  __syncthreads();
  // the adjusted value of id, applying the penalty once per occurrence
  auto adjusted = [&](int id) {
    float v = lr[id];
    if (!pen) return v;
    for (int q = 0; q < nrec; ++q)
      if (srec[q] == id) v = v > 0.f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
    return v;
  };
  const int kNone = INT_MAX;
  float bv = 0.f;
  int bi = kNone;
  auto consider = [&](float v, int i) {
    if (v != v) return;  // NaN
    if (bi == kNone || v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  };
  if (pen)
    for (int r = threadIdx.x; r < nrec; r += blockDim.x) {
      const int id = srec[r];
      if (id < 0 || id >= vocab) continue;
      bool first = true;
      for (int q = 0; q < r && first; ++q) first = srec[q] != id;
      if (first) consider(adjusted(id), id);
    }
  // the scan issues kBatch independent loads per thread before comparing them
  constexpr int kBatch = 16;
  const int nv = (int)vocab;
  for (int i0 = threadIdx.x; i0 < nv; i0 += blockDim.x * kBatch) {
    float v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      v[u] = i < nv ? lr[i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      if (i < nv && !(pen && ((gbits[i >> 5] >> (i & 31)) & 1u))) consider(v[u], i);
    }
  }
  auto better = [](float v1, int i1, float v2, int i2) {
    if (i1 == INT_MAX) return false;
    if (i2 == INT_MAX) return true;
    return v1 > v2 || (v1 == v2 && i1 < i2);
  };
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; ++i)
      if (better(sv[i], si[i], bv, bi)) {
        bv = sv[i];
        bi = si[i];
      }
    const float v0 = adjusted(0);
    out_ids[blockIdx.x] = (v0 != v0 || bi == kNone) ? 0 : bi;
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                           float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(a[i], b[i]);
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t n,
                              float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float sig = __frcp_rn(__fadd_rn(1.0f, expf(-g[i])));   // = 1 / (1 + e^-g), rounded once
    out[i] = __fmul_rn(__fmul_rn(g[i], sig), u[i]);
  }
}

// one thread per (b, t, h, i < D/2) pair of elements
__global__ void rope_kernel(float* __restrict__ d, int64_t T, int64_t H, int64_t D, int64_t npairs,
                            int64_t pos_offset, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t half = D / 2;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < npairs; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = p % half, bth = p / half;
    const int64_t t = (bth / H) % T;
    const int64_t base = bth * D;
    const int64_t pos = pos_offset + t;
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    const float x1 = d[base + i], x2 = d[base + i + half];
    d[base + i] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
    d[base + i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
}

// RoPE of one token per sequence at the sequence's device position:
// data [B][H][D] in place (rotate-half, as rope_kernel)
__global__ void rope_batch_kernel(float* __restrict__ d, int64_t B, int64_t H, int64_t D,
                                  const int32_t* __restrict__ pos, int64_t max_seq,
                                  const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t half = D / 2, npairs = B * H * half;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < npairs;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = p % half, bh = p / half, b = bh / H;
    const int64_t ps = pos[b];
    if (ps < 0 || ps >= max_seq) continue;
    const int64_t base = bh * D;
    const float c = cos_t[ps * half + i], s = sin_t[ps * half + i];
    const float x1 = d[base + i], x2 = d[base + i + half];
    d[base + i] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
    d[base + i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
}

// pos[b] += 1 for every sequence (after the step's last reader)
__global__ void advance_pos_kernel(int32_t* pos, int64_t B) {
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) pos[b] += 1;
}

// appendKV: row pos of every KV head; one thread per element
__global__ void kv_append_kernel(const float* __restrict__ k_new, const float* __restrict__ v_new,
                                 float* __restrict__ kc, float* __restrict__ vc, int64_t HKV,
                                 int64_t D, int64_t max_seq, int64_t pos) {
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < HKV * D; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t h = i / D, dd = i - h * D;
    kc[(h * max_seq + pos) * D + dd] = k_new[i];
    vc[(h * max_seq + pos) * D + dd] = v_new[i];
  }
}

// appendKV of T prompt rows: k_new / v_new [T][HKV][D] -> rows pos0 + t
__global__ void kv_append_rows_kernel(const float* __restrict__ k_new, const float* __restrict__ v_new,
                                      float* __restrict__ kc, float* __restrict__ vc, int64_t T,
                                      int64_t HKV, int64_t D, int64_t max_seq, int64_t pos0) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t total = T * HKV * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / (HKV * D), r = i - t * HKV * D;
    const int64_t h = r / D, dd = r - h * D;
    kc[(h * max_seq + pos0 + t) * D + dd] = k_new[i];
    vc[(h * max_seq + pos0 + t) * D + dd] = v_new[i];
  }
}

// Causal prompt attention (forwardPrefill, nim_inference.nim:574-620, through
// cpuAttentionFused, vendor/bybylang/gpubackend.nim:171-201): one warp per
// (query token t, query head h), over cache rows 0 .. pos0 + t of KV head
// h / nrep.  score = (q . k) * scale; the softmax runs online over batches of
// kPrefUnroll rows (running max, rescaled exp-sum and P.V), normalised at the
// end -- the reference's two passes up to rounding.  Lane l holds features
// l + 32 i.  The 8 warps of a block take 8 consecutive tokens of one head, so
// they read the same K / V rows through L1.
constexpr int kPrefWarps = 8;
constexpr int kPrefUnroll = 4;   // cache rows per online-softmax batch
template <int DV>
__global__ void __launch_bounds__(kPrefWarps * 32)
attn_prefill_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                    const float* __restrict__ vc, int64_t T, int64_t H, int64_t nrep,
                    int64_t max_seq, int64_t pos0, float scale, float* __restrict__ out) {
  constexpr int D = 32 * DV;
  griddep_launch_dependents();
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kPrefWarps + warp;
  const int64_t h = blockIdx.y;
  if (t >= T) return;
  const float* K = kc + (h / nrep) * max_seq * D;
  const float* V = vc + (h / nrep) * max_seq * D;
  float qv[DV], acc[DV];
#pragma unroll
  for (int i = 0; i < DV; ++i) {
    qv[i] = q[(t * H + h) * D + lane + 32 * i];
    acc[i] = 0.f;
  }
  const int64_t S = pos0 + t + 1;
  float m = -INFINITY, l = 0.f;
  for (int64_t j0 = 0; j0 < S; j0 += kPrefUnroll) {
    float kv[kPrefUnroll][DV];
#pragma unroll
    for (int u = 0; u < kPrefUnroll; ++u)
#pragma unroll
      for (int i = 0; i < DV; ++i)
        kv[u][i] = j0 + u < S ? __ldg(K + (j0 + u) * D + lane + 32 * i) : 0.f;
    float sc[kPrefUnroll];
#pragma unroll
    for (int u = 0; u < kPrefUnroll; ++u) {
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < DV; ++i) dot = fmaf(qv[i], kv[u][i], dot);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      sc[u] = j0 + u < S ? dot * scale : -INFINITY;
    }
    float mn = m;
#pragma unroll
    for (int u = 0; u < kPrefUnroll; ++u) mn = fmaxf(mn, sc[u]);
    const float corr = expf(m - mn);   // m = -inf at the start: 0
    l *= corr;
#pragma unroll
    for (int i = 0; i < DV; ++i) acc[i] *= corr;
#pragma unroll
    for (int u = 0; u < kPrefUnroll; ++u) {
      if (j0 + u < S) {
        const float e = expf(sc[u] - mn);
        l += e;
#pragma unroll
        for (int i = 0; i < DV; ++i) acc[i] = fmaf(e, __ldg(V + (j0 + u) * D + lane + 32 * i), acc[i]);
      }
    }
    m = mn;
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int i = 0; i < DV; ++i) out[(t * H + h) * D + lane + 32 * i] = acc[i] * inv;
}

// Decode attention in position splits (the same softmax, normalised at the
// end): block (h, j) takes positions [j*ps, min(S, (j+1)*ps)) of query head h
// (KV head h / nrep), with q pre-scaled and rounded as the reference does,
// and writes m = max score, l = sum exp(score - m), o[d] = sum exp(score - m)
// v[s][d] to part[h][j][D + 2].  Each warp keeps kAttnUnroll positions'
// loads in flight.  Dynamic shared memory: ps scores + 4 warps x D partials.
constexpr int kAttnWarps = 4;
constexpr int kAttnUnroll = 4;
constexpr int kAttnMaxSplit = 8;
// The split's work for query head q_h (D values) over cache rows [s0, s1)
// of K / V (the KV head's rows from 0); writes D partials, m and l to pp.
template <int DV>  // features per lane: D = 32 DV
__device__ __forceinline__ void attn_split_body(const float* __restrict__ q_h,
                                                const float* __restrict__ Kh,
                                                const float* __restrict__ Vh, int64_t D,
                                                int64_t s0, int64_t s1, float scale, float* pp,
                                                float* sc, float* sh, float* qs, int64_t ps) {
  const int64_t ns = max((int64_t)0, s1 - s0);
  const float* K = Kh + s0 * D;
  const float* V = Vh + s0 * D;
  for (int64_t dd = threadIdx.x; dd < D; dd += blockDim.x) qs[dd] = __fmul_rn(q_h[dd], scale);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // scores: positions warp, warp + 4, ... in batches of kAttnUnroll per warp
  float ql[DV];
#pragma unroll
  for (int i = 0; i < DV; ++i) ql[i] = qs[lane + 32 * i];
  for (int64_t b = (int64_t)warp * kAttnUnroll; b < ns; b += kAttnWarps * kAttnUnroll) {
    // every load of the batch is issued before the products
    float kv[kAttnUnroll][DV];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u)
#pragma unroll
      for (int i = 0; i < DV; ++i) kv[u][i] = b + u < ns ? K[(b + u) * D + lane + 32 * i] : 0.f;
    float a[kAttnUnroll];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      a[u] = 0.f;
#pragma unroll
      for (int i = 0; i < DV; ++i) a[u] = __fadd_rn(a[u], __fmul_rn(ql[i], kv[u][i]));
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a[u] += __shfl_xor_sync(0xffffffffu, a[u], o);
      if (lane == 0 && b + u < ns) sc[b + u] = a[u];
    }
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int64_t s = threadIdx.x; s < ns; s += blockDim.x) mx = fmaxf(mx, sc[s]);
  mx = block_max(mx, sh);
  float sum = 0.f;
  for (int64_t s = threadIdx.x; s < ns; s += blockDim.x) {
    const float e = expf(__fsub_rn(sc[s], mx));
    sc[s] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = block_sum(sum, sh);
  __syncthreads();
  // P . V with unnormalised weights: warp w takes positions w (mod 4) in
  // batches, lane the features lane + 32 i; partials summed in warp order
  float acc[DV];
#pragma unroll
  for (int i = 0; i < DV; ++i) acc[i] = 0.f;
  for (int64_t b = (int64_t)warp * kAttnUnroll; b < ns; b += kAttnWarps * kAttnUnroll) {
    float vv[kAttnUnroll][DV];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u)
#pragma unroll
      for (int i = 0; i < DV; ++i) vv[u][i] = b + u < ns ? V[(b + u) * D + lane + 32 * i] : 0.f;
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      if (b + u < ns) {
        const float e = sc[b + u];
#pragma unroll
        for (int i = 0; i < DV; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(e, vv[u][i]));
      }
    }
  }
  float* red = sc + ps;
#pragma unroll
  for (int i = 0; i < DV; ++i) red[warp * D + lane + 32 * i] = acc[i];
  __syncthreads();
  for (int64_t dd = threadIdx.x; dd < D; dd += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) a = __fadd_rn(a, red[w * D + dd]);
    pp[dd] = a;
  }
  if (threadIdx.x == 0) {
    pp[D] = mx;
    pp[D + 1] = sum;
  }
}

template <int DV>  // features per lane: D = 32 DV
__global__ void attn_split_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                  const float* __restrict__ vc, int64_t nrep, int64_t D,
                                  int64_t max_seq, int64_t S, int64_t ps, float scale,
                                  float* __restrict__ part) {
  extern __shared__ float sc[];
  __shared__ float sh[32];
  __shared__ float qs[256];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t h = blockIdx.x, j = blockIdx.y, nsplit = gridDim.y, hkv = h / nrep;
  const int64_t s0 = j * ps, s1 = min(S, s0 + ps);
  attn_split_body<DV>(q + h * D, kc + hkv * max_seq * D, vc + hkv * max_seq * D, D, s0, s1, scale,
                      part + (h * nsplit + j) * (D + 2), sc, sh, qs, ps);
}

// The same for B sequences at once, each at its own position read on the
// device (so a captured step can be replayed token after token): block
// (h, j, b) works on sequence b (q [B][H][D], caches [B][HKV][max_seq][D]);
// the split length is ceil(S_b / nsplit) for S_b = pos[b] + 1, with shared
// memory sized for S = max_seq.  A position outside [0, max_seq) leaves the
// split empty (its partial has l = 0) and sets the error word.
template <int DV>
__global__ void attn_split_batch_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                        const float* __restrict__ vc, const int32_t* __restrict__ pos,
                                        int64_t H, int64_t nrep, int64_t D, int64_t max_seq,
                                        int64_t ps_max, float scale, float* __restrict__ part,
                                        int* err) {
  extern __shared__ float sc[];
  __shared__ float sh[32];
  __shared__ float qs[256];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t h = blockIdx.x, j = blockIdx.y, nsplit = gridDim.y, b = blockIdx.z;
  const int64_t p = pos[b];
  const bool ok = p >= 0 && p < max_seq;
  if (!ok && h == 0 && j == 0 && threadIdx.x == 0 && err) atomicExch(err, 4);
  const int64_t S = ok ? p + 1 : 0;
  const int64_t ps = (S + nsplit - 1) / nsplit;
  const int64_t s0 = min(S, j * ps), s1 = min(S, s0 + ps);
  const int64_t HKV = H / nrep, hkv = h / nrep;
  const float* Kh = kc + ((b * HKV + hkv) * max_seq) * D;
  const float* Vh = vc + ((b * HKV + hkv) * max_seq) * D;
  attn_split_body<DV>(q + (b * H + h) * D, Kh, Vh, D, s0, s1, scale,
                      part + ((b * H + h) * nsplit + j) * (D + 2), sc, sh, qs, ps_max);
}

// appendKV for B sequences at their device positions: row pos[b] of
// sequence b's caches; one thread per element
__global__ void kv_append_batch_kernel(const float* __restrict__ k_new, const float* __restrict__ v_new,
                                       float* __restrict__ kc, float* __restrict__ vc,
                                       const int32_t* __restrict__ pos, int64_t B, int64_t HKV,
                                       int64_t D, int64_t max_seq) {
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < B * HKV * D;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / (HKV * D), r = i - b * HKV * D, h = r / D, dd = r - h * D;
    const int64_t p = pos[b];
    if (p < 0 || p >= max_seq) continue;
    kc[((b * HKV + h) * max_seq + p) * D + dd] = k_new[i];
    vc[((b * HKV + h) * max_seq + p) * D + dd] = v_new[i];
  }
}

// out[h][d] = sum_j w_j o_j[d] / sum_j w_j l_j, w_j = exp(m_j - max_j m_j),
// splits taken in order; one block per head.
__global__ void attn_combine_kernel(const float* __restrict__ part, int64_t nsplit, int64_t D,
                                    float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t h = blockIdx.x;
  const float* pp = part + h * nsplit * (D + 2);
  float M = -INFINITY;
  for (int64_t j = 0; j < nsplit; ++j) M = fmaxf(M, pp[j * (D + 2) + D]);
  float L = 0.f;
  for (int64_t j = 0; j < nsplit; ++j) {
    const float l = pp[j * (D + 2) + D + 1];
    if (l > 0.f) L = __fadd_rn(L, __fmul_rn(expf(__fsub_rn(pp[j * (D + 2) + D], M)), l));
  }
  for (int64_t dd = threadIdx.x; dd < D; dd += blockDim.x) {
    float a = 0.f;
    for (int64_t j = 0; j < nsplit; ++j) {
      const float l = pp[j * (D + 2) + D + 1];
      if (l > 0.f) a = __fadd_rn(a, __fmul_rn(expf(__fsub_rn(pp[j * (D + 2) + D], M)), pp[j * (D + 2) + dd]));
    }
    out[h * D + dd] = __fdiv_rn(a, L);
  }
}

// split partials, per device (grown outside stream capture; calls using it
// are ordered on one stream)
struct AttnBuf {
  int device = -1;
  void* p = nullptr;
  size_t bytes = 0;
};
AttnBuf g_abuf;

int attn_buffer(size_t bytes, cudaStream_t st, float** out) {
  Context* c = ctx();
  if (g_abuf.device != c->device || g_abuf.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NIMF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(NIMF_ERR_STATE,
                       "decode attention: its partial buffer must grow, which cannot happen during "
                       "stream capture; run the same call once before capturing");
    NIMF_CUDA_TRY(cudaDeviceSynchronize());
    if (g_abuf.device == c->device) device_free(g_abuf.p);
    g_abuf = AttnBuf();
    NIMF_TRY(device_alloc(&g_abuf.p, bytes));
    g_abuf.device = c->device;
    g_abuf.bytes = bytes;
  }
  *out = (float*)g_abuf.p;
  return NIMF_OK;
}

// Launch with programmatic dependent launch allowed, so that a following
// GEMV can become resident and prefetch its weights while this kernel runs.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ((KArgs)args)...));
  return NIMF_OK;
}

unsigned grid_n(int64_t n) {
  Context* c = ctx();
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((int64_t)(c ? c->num_sms : 148) * 8, (n + 255) / 256));
}

int stream_of(void* stream, cudaStream_t* st) {
  Context* c;
  NIMF_TRY(require_ctx(&c));
  *st = stream ? (cudaStream_t)stream : c->stream;
  return NIMF_OK;
}

}  // namespace

void release_attn_buffer() {
  device_free(g_abuf.p);
  g_abuf = AttnBuf();
}

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_rmsnorm_dev(const float* x, const float* w, int64_t rows, int64_t cols, float eps,
                     float* y, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (rows < 0 || cols < 0 || rows > INT32_MAX) return set_error(NIMF_ERR_SHAPE, "rmsnorm: rows %lld cols %lld", (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return NIMF_OK;
  if (!x || !w || !y) return set_error(NIMF_ERR_ARG, "rmsnorm: NULL buffer");
  NIMF_TRY(launch_pdl(rmsnorm_kernel, (unsigned)rows, 1024, 0, st, x, (const float*)nullptr,
                      (float*)nullptr, w, cols, eps, y));
  return NIMF_OK;
}

int nimf_layernorm_dev(const float* x, const float* gamma, const float* beta, int64_t rows,
                       int64_t cols, float eps, float* y, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (rows < 0 || cols < 0 || rows > INT32_MAX) return set_error(NIMF_ERR_SHAPE, "layernorm: rows %lld cols %lld", (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return NIMF_OK;
  if (!x || !gamma || !beta || !y) return set_error(NIMF_ERR_ARG, "layernorm: NULL buffer");
  NIMF_TRY(launch_pdl(layernorm_kernel, (unsigned)rows, 1024, 0, st, x, gamma, beta, cols, eps, y));
  return NIMF_OK;
}

int nimf_add_rmsnorm_dev(const float* a, const float* b, const float* w, int64_t rows,
                         int64_t cols, float eps, float* h, float* y, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (rows < 0 || cols < 0 || rows > INT32_MAX) return set_error(NIMF_ERR_SHAPE, "add_rmsnorm: rows %lld cols %lld", (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return NIMF_OK;
  if (!a || !b || !w || !h || !y) return set_error(NIMF_ERR_ARG, "add_rmsnorm: NULL buffer");
  NIMF_TRY(launch_pdl(rmsnorm_kernel, (unsigned)rows, 1024, 0, st, a, b, h, w, cols, eps, y));
  return NIMF_OK;
}

int nimf_add_dev(const float* a, const float* b, int64_t n, float* out, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (n < 0) return set_error(NIMF_ERR_SHAPE, "add: n < 0");
  if (n == 0) return NIMF_OK;
  if (!a || !b || !out) return set_error(NIMF_ERR_ARG, "add: NULL buffer");
  NIMF_TRY(launch_pdl(add_kernel, grid_n(n), 256, 0, st, a, b, n, out));
  return NIMF_OK;
}

int nimf_swiglu_dev(const float* gate, const float* up, int64_t n, float* out, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (n < 0) return set_error(NIMF_ERR_SHAPE, "swiglu: n < 0");
  if (n == 0) return NIMF_OK;
  if (!gate || !up || !out) return set_error(NIMF_ERR_ARG, "swiglu: NULL buffer");
  NIMF_TRY(launch_pdl(swiglu_kernel, grid_n(n), 256, 0, st, gate, up, n, out));
  return NIMF_OK;
}

int nimf_rope_dev(float* data, int64_t B, int64_t T, int64_t H, int64_t D, int64_t pos_offset,
                  const float* cos_t, const float* sin_t, int64_t max_seq, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (B < 0 || T < 0 || H < 0 || D < 0 || (D & 1) || pos_offset < 0)
    return set_error(NIMF_ERR_SHAPE, "rope: bad shape (D must be even)");
  if (pos_offset + T > max_seq)
    return set_error(NIMF_ERR_SHAPE, "rope: positions up to %lld exceed max_seq %lld",
                     (long long)(pos_offset + T), (long long)max_seq);
  const int64_t npairs = B * T * H * (D / 2);
  if (npairs == 0) return NIMF_OK;
  if (!data || !cos_t || !sin_t) return set_error(NIMF_ERR_ARG, "rope: NULL buffer");
  NIMF_TRY(launch_pdl(rope_kernel, grid_n(npairs), 256, 0, st, data, T, H, D, npairs, pos_offset,
                      cos_t, sin_t));
  return NIMF_OK;
}

int nimf_attention_decode_dev(const float* q, const float* k_new, const float* v_new,
                              float* k_cache, float* v_cache, int64_t H, int64_t HKV, int64_t D,
                              int64_t max_seq, int64_t pos, float scale, float* out, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (H <= 0 || HKV <= 0 || H % HKV || D <= 0 || D > 256 || D % 32 || pos < 0 || pos >= max_seq)
    return set_error(NIMF_ERR_SHAPE, "attention: H %lld HKV %lld D %lld (a multiple of 32, <= 256) pos %lld max_seq %lld",
                     (long long)H, (long long)HKV, (long long)D, (long long)pos, (long long)max_seq);
  const int64_t S = pos + 1;
  if (S > 8 * 40000) return set_error(NIMF_ERR_UNSUPPORTED, "attention: %lld positions exceed the score buffers", (long long)S);
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !out) return set_error(NIMF_ERR_ARG, "attention: NULL buffer");
  NIMF_TRY(launch_pdl(kv_append_kernel, grid_n(HKV * D), 256, 0, st, k_new, v_new, k_cache,
                      v_cache, HKV, D, max_seq, pos));
  // position splits: about 64 positions per block, at most 8 per head
  const int64_t nsplit = std::min<int64_t>(kAttnMaxSplit, (S + 63) / 64);
  const int64_t ps = (S + nsplit - 1) / nsplit;
  const size_t smem = (size_t)(ps + kAttnWarps * D) * 4;
  void (*kern)(const float*, const float*, const float*, int64_t, int64_t, int64_t, int64_t,
               int64_t, float, float*);
  switch (D / 32) {
    case 1: kern = attn_split_kernel<1>; break;
    case 2: kern = attn_split_kernel<2>; break;
    case 3: kern = attn_split_kernel<3>; break;
    case 4: kern = attn_split_kernel<4>; break;
    case 5: kern = attn_split_kernel<5>; break;
    case 6: kern = attn_split_kernel<6>; break;
    case 7: kern = attn_split_kernel<7>; break;
    default: kern = attn_split_kernel<8>; break;
  }
  if (smem > 48 * 1024)
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  float* part = nullptr;
  NIMF_TRY(attn_buffer((size_t)(H * nsplit * (D + 2)) * 4, st, &part));
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)H, (unsigned)nsplit);
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, (const float*)k_cache,
                                     (const float*)v_cache, H / HKV, D, max_seq, S, ps, scale, part));
  }
  NIMF_TRY(launch_pdl(attn_combine_kernel, (unsigned)H, 128, 0, st, (const float*)part, nsplit, D, out));
  return NIMF_OK;
}

int nimf_attention_prefill_dev(const float* q, const float* k_new, const float* v_new,
                               float* k_cache, float* v_cache, int64_t T, int64_t H, int64_t HKV,
                               int64_t D, int64_t max_seq, int64_t pos0, float scale, float* out,
                               void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (T < 0 || H <= 0 || HKV <= 0 || H % HKV || D <= 0 || D > 256 || D % 32 || pos0 < 0 ||
      pos0 + T > max_seq || H > 65535)
    return set_error(NIMF_ERR_SHAPE,
                     "prefill attention: T %lld H %lld HKV %lld D %lld (a multiple of 32, <= 256) "
                     "pos0 %lld max_seq %lld",
                     (long long)T, (long long)H, (long long)HKV, (long long)D, (long long)pos0,
                     (long long)max_seq);
  if (T == 0) return NIMF_OK;
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !out)
    return set_error(NIMF_ERR_ARG, "prefill attention: NULL buffer");
  NIMF_TRY(launch_pdl(kv_append_rows_kernel, grid_n(T * HKV * D), 256, 0, st, k_new, v_new,
                      k_cache, v_cache, T, HKV, D, max_seq, pos0));
  void (*kern)(const float*, const float*, const float*, int64_t, int64_t, int64_t, int64_t,
               int64_t, float, float*);
  switch (D / 32) {
    case 1: kern = attn_prefill_kernel<1>; break;
    case 2: kern = attn_prefill_kernel<2>; break;
    case 3: kern = attn_prefill_kernel<3>; break;
    case 4: kern = attn_prefill_kernel<4>; break;
    case 5: kern = attn_prefill_kernel<5>; break;
    case 6: kern = attn_prefill_kernel<6>; break;
    case 7: kern = attn_prefill_kernel<7>; break;
    default: kern = attn_prefill_kernel<8>; break;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((T + kPrefWarps - 1) / kPrefWarps), (unsigned)H);
  cfg.blockDim = dim3(kPrefWarps * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, (const float*)k_cache, (const float*)v_cache, T,
                                   H, H / HKV, max_seq, pos0, scale, out));
  return NIMF_OK;
}

int nimf_attention_decode_batch_dev(float* q, float* k_new, const float* v_new, float* k_cache,
                                    float* v_cache, int64_t B, int64_t H, int64_t HKV, int64_t D,
                                    int64_t max_seq, int32_t* pos_dev, const float* cos_t,
                                    const float* sin_t, float scale, int advance_pos, float* out,
                                    void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  Context* c = ctx();
  if (B < 0 || H <= 0 || HKV <= 0 || H % HKV || D <= 0 || D > 256 || D % 32 || max_seq < 1 ||
      max_seq > 8 * 40000 || B * H > 65535 * 8)
    return set_error(NIMF_ERR_SHAPE,
                     "batch attention: B %lld H %lld HKV %lld D %lld (a multiple of 32, <= 256) "
                     "max_seq %lld",
                     (long long)B, (long long)H, (long long)HKV, (long long)D, (long long)max_seq);
  if (B == 0) return NIMF_OK;
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !out || !pos_dev || (!cos_t != !sin_t))
    return set_error(NIMF_ERR_ARG, "batch attention: NULL buffer");
  if (cos_t) {
    NIMF_TRY(launch_pdl(rope_batch_kernel, grid_n(B * H * D / 2), 256, 0, st, q, B, H, D,
                        (const int32_t*)pos_dev, max_seq, cos_t, sin_t));
    NIMF_TRY(launch_pdl(rope_batch_kernel, grid_n(B * HKV * D / 2), 256, 0, st, k_new, B, HKV, D,
                        (const int32_t*)pos_dev, max_seq, cos_t, sin_t));
  }
  NIMF_TRY(launch_pdl(kv_append_batch_kernel, grid_n(B * HKV * D), 256, 0, st,
                      (const float*)k_new, v_new, k_cache, v_cache, (const int32_t*)pos_dev, B,
                      HKV, D, max_seq));
  // splits fixed by max_seq (the positions are only known on the device)
  const int64_t nsplit = std::min<int64_t>(kAttnMaxSplit, (max_seq + 63) / 64);
  const int64_t ps_max = (max_seq + nsplit - 1) / nsplit;
  const size_t smem = (size_t)(ps_max + kAttnWarps * D) * 4;
  void (*kern)(const float*, const float*, const float*, const int32_t*, int64_t, int64_t, int64_t,
               int64_t, int64_t, float, float*, int*);
  switch (D / 32) {
    case 1: kern = attn_split_batch_kernel<1>; break;
    case 2: kern = attn_split_batch_kernel<2>; break;
    case 3: kern = attn_split_batch_kernel<3>; break;
    case 4: kern = attn_split_batch_kernel<4>; break;
    case 5: kern = attn_split_batch_kernel<5>; break;
    case 6: kern = attn_split_batch_kernel<6>; break;
    case 7: kern = attn_split_batch_kernel<7>; break;
    default: kern = attn_split_batch_kernel<8>; break;
  }
  if (smem > 48 * 1024)
    NIMF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  float* part = nullptr;
  NIMF_TRY(attn_buffer((size_t)(B * H * nsplit * (D + 2)) * 4, st, &part));
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)H, (unsigned)nsplit, (unsigned)B);
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, (const float*)q, (const float*)k_cache,
                                     (const float*)v_cache, (const int32_t*)pos_dev, H, H / HKV, D,
                                     max_seq, ps_max, scale, part, c ? c->dev_err : nullptr));
  }
  NIMF_TRY(launch_pdl(attn_combine_kernel, (unsigned)(B * H), 128, 0, st, (const float*)part,
                      nsplit, D, out));
  if (advance_pos) NIMF_TRY(launch_pdl(advance_pos_kernel, 1, 32, 0, st, pos_dev, B));
  return NIMF_OK;
}

int nimf_embedding_lookup_dev(const float* table, int64_t vocab, int64_t dim,
                              const int32_t* ids, int64_t n, float* out, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  if (vocab < 0 || dim < 0 || n < 0 || n > INT32_MAX)
    return set_error(NIMF_ERR_SHAPE, "embedding_lookup: vocab %lld dim %lld n %lld", (long long)vocab, (long long)dim, (long long)n);
  if (n == 0 || dim == 0) return NIMF_OK;
  if (!table || !ids || !out) return set_error(NIMF_ERR_ARG, "embedding_lookup: NULL buffer");
  const unsigned threads = (unsigned)std::min<int64_t>(1024, ((dim + 3) / 4 + 31) / 32 * 32);
  NIMF_TRY(launch_pdl(embedding_kernel, (unsigned)n, threads, 0, st, table, vocab, dim, ids, out));
  return NIMF_OK;
}

int nimf_greedy_sample_dev(const float* logits, int64_t rows, int64_t vocab, const int32_t* recent,
                           int64_t n_recent, float repeat_penalty, int32_t* out_ids, void* stream) {
  cudaStream_t st;
  NIMF_TRY(stream_of(stream, &st));
  const int64_t max_vocab = (int64_t)32 * 1024 * 8;  // bitmap within 32 KB of shared memory
  if (rows < 0 || rows > INT32_MAX || vocab < 1 || vocab > max_vocab || n_recent < 0 ||
      n_recent > kGreedyMaxRecent)
    return set_error(NIMF_ERR_SHAPE, "greedy_sample: rows %lld vocab %lld (1..%lld) recent %lld (<= %d)",
                     (long long)rows, (long long)vocab, (long long)max_vocab, (long long)n_recent,
                     kGreedyMaxRecent);
  if (rows == 0) return NIMF_OK;
  if (!logits || !out_ids || (n_recent > 0 && !recent))
    return set_error(NIMF_ERR_ARG, "greedy_sample: NULL buffer");
  const size_t smem = (size_t)((vocab + 31) / 32) * 4;
  NIMF_TRY(launch_pdl(greedy_kernel, (unsigned)rows, 1024, smem, st, logits, vocab, recent,
                      (int)n_recent, repeat_penalty, out_ids));
  return NIMF_OK;
}

}  // extern "C"
