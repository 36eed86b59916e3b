// reg.cu — the sparsity regularisers of SPLADE training on the head's output
// reps [B, V] (one vocabulary shard of it when the head is sharded), fused into
// one pass over reps each way.
//
// Upstream (hhkbble/sparton training/train.py) computes them with separate
// torch reductions:
//   l1_regularization (:80-82)    = mean_b sum_v |reps[b, v]|
//   flops_regularization (:85-87) = mean_v (sum_b reps[b, v])^2
// Here reg_fwd_kernel reads reps once and produces the column sums
// colsum[v] = sum_b reps[b, v] (kept for the backward) and, per block, the
// partial sums of |reps| and of colsum^2; reg_total_kernel adds the block
// partials in a fixed order (deterministic) and scales them, giving
// out = {scale_l1 * sum |reps|, scale_flops * sum_v colsum^2} (1/B and 1/V for
// the losses; shards' outputs then simply add up). reg_bwd_kernel writes
//   grad[b, v] = g_l1 * scale_l1 * sign(reps[b, v]) + g_flops * scale_flops * colsum[v]
// with the upstream gradients g_l1, g_flops read from device memory (1/B and
// 2/V as scales), so neither direction needs a host round trip or any
// arithmetic outside the kernels.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dtype.cuh"
#include "internal.h"

namespace sparton {
namespace {

constexpr int kRegWarps = 8;  // rows are strided over the warps of a block
constexpr int kTotalThreads = 1024;

// One block per 32 vocabulary columns (one per lane); warp w sums rows
// b = w, w + 8, ... of its lane's column.
template <typename T>
__global__ void __launch_bounds__(kRegWarps * 32)
    reg_fwd_kernel(const T* __restrict__ reps, int B, int V, float* __restrict__ colsum,
                   float* __restrict__ partials) {
  __shared__ float s_col[kRegWarps][32];
  __shared__ float s_abs[kRegWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  const int v = blockIdx.x * 32 + lane;
  float col = 0.f, ab = 0.f;
  if (v < V) {
#pragma unroll 8
    for (int b = warp; b < B; b += kRegWarps) {
      const float x = ldg_f32<T>(reps + static_cast<size_t>(b) * V + v);
      col += x;
      ab += fabsf(x);
    }
  }
  s_col[warp][lane] = col;
  s_abs[warp][lane] = ab;
  __syncthreads();
  if (warp == 0) {
    float c = 0.f, a = 0.f;
#pragma unroll
    for (int w = 0; w < kRegWarps; ++w) {
      c += s_col[w][lane];
      a += s_abs[w][lane];
    }
    if (v < V) colsum[v] = c;
    float sq = v < V ? c * c : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    }
    if (lane == 0) {
      partials[2 * blockIdx.x] = a;
      partials[2 * blockIdx.x + 1] = sq;
    }
  }
}

// One block: out[k] = scale_k * sum over blocks of partials[2*blk + k], in a
// fixed order.
__global__ void __launch_bounds__(kTotalThreads)
    reg_total_kernel(const float* __restrict__ partials, int nblocks, float scale_l1,
                     float scale_flops, float* __restrict__ totals) {
  __shared__ float s[2][kTotalThreads / 32];
  pdl_wait();  // the block partials
  float a = 0.f, q = 0.f;
  for (int i = threadIdx.x; i < nblocks; i += kTotalThreads) {
    a += partials[2 * i];
    q += partials[2 * i + 1];
  }
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s[0][warp] = a;
    s[1][warp] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ta = 0.f, tq = 0.f;
    for (int w = 0; w < kTotalThreads / 32; ++w) {
      ta += s[0][w];
      tq += s[1][w];
    }
    totals[0] = ta * scale_l1;
    totals[1] = tq * scale_flops;
  }
}

// Thread per column v (coalesced along a row); rows b = blockIdx.y, + gridDim.y, ...
template <typename T>
__global__ void __launch_bounds__(256)
    reg_bwd_kernel(const T* __restrict__ reps, const float* __restrict__ colsum,
                   const float* __restrict__ g_l1, const float* __restrict__ g_flops,
                   float scale_l1, float scale_flops, int B, int V, T* __restrict__ grad) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  const float c0 = g_l1 != nullptr ? __ldg(g_l1) * scale_l1 : 0.f;
  const float c1 = g_flops != nullptr ? __ldg(g_flops) * scale_flops : 0.f;
  const float cv = c1 * __ldg(colsum + v);
  for (int b = blockIdx.y; b < B; b += gridDim.y) {
    const size_t i = static_cast<size_t>(b) * V + v;
    const float x = ldg_f32<T>(reps + i);
    const float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
    grad[i] = from_f32<T>(fmaf(c0, s, cv));
  }
}

template <typename T>
int launch_fwd_typed(const void* reps, int B, int V, float scale_l1, float scale_flops,
                     float* colsum, float* totals, float* partials, cudaStream_t stream) {
  const int nblocks = (V + 31) / 32;
  reg_fwd_kernel<T><<<nblocks, kRegWarps * 32, 0, stream>>>(static_cast<const T*>(reps), B, V,
                                                            colsum, partials);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reg_fwd_kernel launch");
  e = launch_pdl(reg_total_kernel, dim3(1), dim3(kTotalThreads), 0, stream,
                 static_cast<const float*>(partials), nblocks, scale_l1, scale_flops, totals);
  if (e != cudaSuccess) return cuda_fail(e, "reg_total_kernel launch");
  return SPARTON_OK;
}

template <typename T>
int launch_bwd_typed(const void* reps, const float* colsum, const float* g_l1,
                     const float* g_flops, float scale_l1, float scale_flops, int B, int V,
                     void* grad, cudaStream_t stream) {
  const unsigned cols = static_cast<unsigned>((V + 255) / 256);
  // Enough blocks for ~8 per SM, each covering a strided subset of the rows.
  unsigned rows = static_cast<unsigned>((8ll * device_sm_count() + cols - 1) / cols);
  if (rows > static_cast<unsigned>(B)) rows = static_cast<unsigned>(B);
  if (rows < 1) rows = 1;
  reg_bwd_kernel<T><<<dim3(cols, rows), 256, 0, stream>>>(
      static_cast<const T*>(reps), colsum, g_l1, g_flops, scale_l1, scale_flops, B, V,
      static_cast<T*>(grad));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reg_bwd_kernel launch");
  return SPARTON_OK;
}

}  // namespace

size_t reg_workspace_bytes(int64_t V) { return align256(static_cast<size_t>((V + 31) / 32) * 8); }

int launch_reg_fwd(int dtype, const void* reps, int B, int V, float scale_l1, float scale_flops,
                   float* colsum, float* totals, void* workspace, cudaStream_t stream) {
  float* partials = static_cast<float*>(workspace);
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_fwd_typed<__nv_bfloat16>(reps, B, V, scale_l1, scale_flops, colsum, totals,
                                             partials, stream);
    case SPARTON_DTYPE_F16:
      return launch_fwd_typed<__half>(reps, B, V, scale_l1, scale_flops, colsum, totals, partials,
                                      stream);
    case SPARTON_DTYPE_F32:
      return launch_fwd_typed<float>(reps, B, V, scale_l1, scale_flops, colsum, totals, partials,
                                     stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

int launch_reg_bwd(int dtype, const void* reps, const float* colsum, const float* g_l1,
                   const float* g_flops, float scale_l1, float scale_flops, int B, int V,
                   void* grad, cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_bwd_typed<__nv_bfloat16>(reps, colsum, g_l1, g_flops, scale_l1, scale_flops, B,
                                             V, grad, stream);
    case SPARTON_DTYPE_F16:
      return launch_bwd_typed<__half>(reps, colsum, g_l1, g_flops, scale_l1, scale_flops, B, V,
                                      grad, stream);
    case SPARTON_DTYPE_F32:
      return launch_bwd_typed<float>(reps, colsum, g_l1, g_flops, scale_l1, scale_flops, B, V,
                                     grad, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

}  // namespace sparton
