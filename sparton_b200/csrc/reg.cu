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
// partial sums of |reps| and of colsum^2; the last block to finish (a ticket
// counter in the workspace, zero between calls: the last block clears it) adds
// the block partials
// in a fixed order (deterministic) and scales them, giving
// out = {scale_l1 * sum |reps|, scale_flops * sum_v colsum^2} (1/B and 1/V for
// the losses; shards' outputs then simply add up). reg_bwd_kernel writes
//   grad[b, v] = g_l1 * scale_l1 * sign(reps[b, v]) + g_flops * scale_flops * colsum[v]
// elementwise over the flattened [B * V] (16-byte loads and stores), with the
// upstream gradients g_l1, g_flops read from device memory (1/B and 2/V as
// scales), so neither direction needs a host round trip or any arithmetic
// outside the kernels.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "dtype.cuh"
#include "internal.h"

namespace sparton {
namespace {

constexpr int kRegWarps = 8;  // rows are strided over the warps of a block
constexpr int kRowUnroll = 16;  // row loads of a lane in flight

// kC consecutive columns of a row as fp32 (one 2 * sizeof(T)-byte load for kC = 2).
template <typename T, int kC>
__device__ __forceinline__ void load_cols(const T* p, float (&x)[kC]) {
  if constexpr (kC == 1) {
    x[0] = ldg_f32<T>(p);
  } else if constexpr (sizeof(T) == 2) {
    const unsigned int w = __ldg(reinterpret_cast<const unsigned int*>(p));
    const T* e = reinterpret_cast<const T*>(&w);
    x[0] = to_f32<T>(e[0]);
    x[1] = to_f32<T>(e[1]);
  } else {
    const float2 w = __ldg(reinterpret_cast<const float2*>(p));
    x[0] = w.x;
    x[1] = w.y;
  }
}

// One block per 32 * kC vocabulary columns (kC per lane: kC = 2 when V is
// even and reps is aligned for the pair loads); warp w sums rows b = w, w + 8,
// ... of its lane's columns, kRowUnroll loads in flight. The block's partials
// of |reps| and colsum^2 go to partials[2 * block]; the last block adds them
// over the blocks in order and writes the scaled totals, then re-arms the
// ticket counter.
template <typename T, int kC>
__global__ void __launch_bounds__(kRegWarps * 32)
    reg_fwd_kernel(const T* __restrict__ reps, int B, int V, float* __restrict__ colsum,
                   float* __restrict__ partials, unsigned int* __restrict__ counter,
                   float scale_l1, float scale_flops, float* __restrict__ totals) {
  __shared__ float s_col[kRegWarps][32 * kC];
  __shared__ float s_abs[kRegWarps][32];
  __shared__ bool s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v0 = (blockIdx.x * 32 + lane) * kC;
  float col[kC], ab = 0.f;
#pragma unroll
  for (int j = 0; j < kC; ++j) col[j] = 0.f;
  if (v0 < V) {
    const T* p = reps + v0;
    int b = warp;
    for (; b + (kRowUnroll - 1) * kRegWarps < B; b += kRowUnroll * kRegWarps) {
      float x[kRowUnroll][kC];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
        load_cols<T, kC>(p + static_cast<size_t>(b + u * kRegWarps) * V, x[u]);
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
#pragma unroll
        for (int j = 0; j < kC; ++j) {
          col[j] += x[u][j];
          ab += fabsf(x[u][j]);
        }
    }
    for (; b < B; b += kRegWarps) {
      float x[kC];
      load_cols<T, kC>(p + static_cast<size_t>(b) * V, x);
#pragma unroll
      for (int j = 0; j < kC; ++j) {
        col[j] += x[j];
        ab += fabsf(x[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kC; ++j) s_col[warp][lane * kC + j] = col[j];
  s_abs[warp][lane] = ab;
  __syncthreads();
  if (warp == 0) {
    float a = 0.f, sq = 0.f;
#pragma unroll
    for (int w = 0; w < kRegWarps; ++w) a += s_abs[w][lane];
#pragma unroll
    for (int j = 0; j < kC; ++j) {
      float c = 0.f;
#pragma unroll
      for (int w = 0; w < kRegWarps; ++w) c += s_col[w][lane * kC + j];
      if (v0 + j < V) {
        colsum[v0 + j] = c;
        sq += c * c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    }
    if (lane == 0) {
      partials[2 * blockIdx.x] = a;
      partials[2 * blockIdx.x + 1] = sq;
      __threadfence();  // the partials before the ticket
      s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // every block's partials are visible
  const int nblocks = static_cast<int>(gridDim.x);
  float a = 0.f, q = 0.f;
  for (int i = threadIdx.x; i < nblocks; i += kRegWarps * 32) {
    a += __ldcg(partials + 2 * i);
    q += __ldcg(partials + 2 * i + 1);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  }
  __syncthreads();  // s_abs / s_col reads are done
  if (lane == 0) {
    s_abs[0][warp] = a;
    s_abs[1][warp] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ta = 0.f, tq = 0.f;
    for (int w = 0; w < kRegWarps; ++w) {
      ta += s_abs[0][w];
      tq += s_abs[1][w];
    }
    totals[0] = ta * scale_l1;
    totals[1] = tq * scale_flops;
    *counter = 0u;
  }
}

// grad over the flattened [B * V]: thread t takes kU vectors of kPer
// consecutive elements (vector t + i * stride, i < kU; 16-byte loads and stores
// when reps and grad are 16-byte aligned, else kPer = 1), all kU loads issued
// before any is used; the column index advances with the element and wraps
// at V. The last n % kPer elements go to block 0's first threads.
constexpr int kBwdU = 4;
template <typename T, int kPer>
__global__ void __launch_bounds__(256)
    reg_bwd_kernel(const T* __restrict__ reps, const float* __restrict__ colsum,
                   const float* __restrict__ g_l1, const float* __restrict__ g_flops,
                   float scale_l1, float scale_flops, long long n, int V, T* __restrict__ grad) {
  const long long nvec = n / kPer;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long v0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  using Vec = typename std::conditional<kPer == 1, T, uint4>::type;
  Vec w[kBwdU];
#pragma unroll
  for (int i = 0; i < kBwdU; ++i) {
    const long long vi = v0 + i * stride;
    if (vi < nvec) {
      if constexpr (kPer == 1)
        w[i] = reps[vi];
      else
        w[i] = __ldg(reinterpret_cast<const uint4*>(reps) + vi);
    }
  }
  const float c0 = g_l1 != nullptr ? __ldg(g_l1) * scale_l1 : 0.f;
  const float c1 = g_flops != nullptr ? __ldg(g_flops) * scale_flops : 0.f;
  // the column of the thread's first element, and how far it moves per vector
  // (32-bit divisions when the offsets fit)
  int vcol, vstep;
  if (n <= 0xFFFFFFFFll) {
    vcol = static_cast<int>(static_cast<unsigned>(v0 * kPer) % static_cast<unsigned>(V));
    vstep = static_cast<int>(static_cast<unsigned>(stride * kPer) % static_cast<unsigned>(V));
  } else {
    vcol = static_cast<int>((v0 * kPer) % V);
    vstep = static_cast<int>((stride * kPer) % V);
  }
#pragma unroll
  for (int i = 0; i < kBwdU; ++i) {
    const long long vi = v0 + i * stride;
    if (vi < nvec) {
      int v = vcol;
      if constexpr (kPer == 1) {
        const float x = to_f32<T>(w[i]);
        const float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
        grad[vi] = from_f32<T>(fmaf(c0, s, c1 * __ldg(colsum + v)));
      } else {
        const T* e = reinterpret_cast<const T*>(&w[i]);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const float x = to_f32<T>(e[k]);
          const float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
          oe[k] = from_f32<T>(fmaf(c0, s, c1 * __ldg(colsum + v)));
          if (++v == V) v = 0;
        }
        *reinterpret_cast<uint4*>(grad + vi * kPer) = o;
      }
    }
    vcol += vstep;
    if (vcol >= V) vcol -= V;
  }
  // the last n % kPer elements
  const long long t = nvec * kPer + v0;
  if (kPer > 1 && t < n && blockIdx.x == 0) {
    const float x = ldg_f32<T>(reps + t);
    const float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
    grad[t] = from_f32<T>(fmaf(c0, s, c1 * __ldg(colsum + static_cast<int>(t % V))));
  }
}

int fwd_blocks(int V, int kc) { return (V + 32 * kc - 1) / (32 * kc); }

template <typename T>
int launch_fwd_typed(const void* reps, int B, int V, float scale_l1, float scale_flops,
                     float* colsum, float* totals, void* workspace, cudaStream_t stream) {
  unsigned int* counter = static_cast<unsigned int*>(workspace);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  const bool pairs =
      V % 2 == 0 && reinterpret_cast<uintptr_t>(reps) % (2 * sizeof(T)) == 0;
  if (pairs)
    reg_fwd_kernel<T, 2><<<fwd_blocks(V, 2), kRegWarps * 32, 0, stream>>>(
        static_cast<const T*>(reps), B, V, colsum, partials, counter, scale_l1, scale_flops,
        totals);
  else
    reg_fwd_kernel<T, 1><<<fwd_blocks(V, 1), kRegWarps * 32, 0, stream>>>(
        static_cast<const T*>(reps), B, V, colsum, partials, counter, scale_l1, scale_flops,
        totals);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "reg_fwd_kernel launch");
}

template <typename T>
int launch_bwd_typed(const void* reps, const float* colsum, const float* g_l1,
                     const float* g_flops, float scale_l1, float scale_flops, int B, int V,
                     void* grad, cudaStream_t stream) {
  const long long n = static_cast<long long>(B) * V;
  if (n == 0) return SPARTON_OK;
  constexpr int kPer = 16 / sizeof(T);
  const bool vec = reinterpret_cast<uintptr_t>(reps) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(grad) % 16 == 0;
  const long long units = vec ? n / kPer : n;
  // every thread takes kBwdU vectors (the grid covers all of them in one pass)
  const long long blocks = std::max(1ll, (units + 256ll * kBwdU - 1) / (256ll * kBwdU));
  if (vec)
    reg_bwd_kernel<T, kPer><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(reps), colsum, g_l1, g_flops, scale_l1, scale_flops, n, V,
        static_cast<T*>(grad));
  else
    reg_bwd_kernel<T, 1><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(reps), colsum, g_l1, g_flops, scale_l1, scale_flops, n, V,
        static_cast<T*>(grad));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reg_bwd_kernel launch");
  return SPARTON_OK;
}

}  // namespace

// [0, 256): the ticket counter; then the blocks' partials (2 floats each).
size_t reg_workspace_bytes(int64_t V) {
  return 256 + align256(static_cast<size_t>((V + 31) / 32) * 8);
}

int launch_reg_fwd(int dtype, const void* reps, int B, int V, float scale_l1, float scale_flops,
                   float* colsum, float* totals, void* workspace, cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_fwd_typed<__nv_bfloat16>(reps, B, V, scale_l1, scale_flops, colsum, totals,
                                             workspace, stream);
    case SPARTON_DTYPE_F16:
      return launch_fwd_typed<__half>(reps, B, V, scale_l1, scale_flops, colsum, totals, workspace,
                                      stream);
    case SPARTON_DTYPE_F32:
      return launch_fwd_typed<float>(reps, B, V, scale_l1, scale_flops, colsum, totals, workspace,
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
