// transform.cu — the MLM transform in front of the head, GELU + LayerNorm part:
//   h = LayerNorm(gelu(y)) * gamma + beta,   y = x @ Wd^T + bd (the dense layer,
//   the tcgen05 GEMM of gemm_tc.cu)
// as in hhkbble/sparton training/model.py:25-35 (RoBERTa: dense, gelu,
// layer_norm) and BERT's predictions.transform (model.py:14-19), whose output
// is the head's input (model.py:82-85). gelu is the exact erf form
// (transformers.activations.gelu); the GELU output is rounded to the input
// dtype before the normalisation, as the reference's separate modules do.
//
//   transform_fwd_kernel     one warp per row: g = round(gelu(y)), mean and
//                            rstd = 1/sqrt(var + eps) (biased variance, as
//                            torch's LayerNorm), h = (g - mean) * rstd * gamma
//                            + beta in the input dtype; mean / rstd saved
//   transform_bwd_fused_kernel (D % 8 == 0, D <= 1024) one warp per row, from
//                            dh (the head's d_hidden):
//                            xh = (g - mean) * rstd, dxh = dh * gamma,
//                            dg = rstd * (dxh - mean(dxh) - xh * mean(dxh * xh)),
//                            dy = dg * gelu'(y); and per CTA the column sums
//                            of dh * xh (d_gamma), dh (d_beta), dy (d_bd)
//   transform_bwd_row_kernel, transform_bwd_col_kernel  the same in two
//                            kernels for other D (rows of any length)
//   transform_col_reduce     the partials in a fixed order -> d_gamma, d_beta,
//                            d_bd (deterministic, no atomics)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

#include <type_traits>

#include "dtype.cuh"
#include "internal.h"

namespace sparton {
namespace {

constexpr int kRowWarps = 8;
constexpr int kColRows = 256;  // rows per CTA of the column kernel
constexpr int kMaxPerLane = 32;  // D <= 1024 keeps a row in registers
constexpr int kVecPerLane = 4;   // 8-column chunks per lane: D <= 1024, D % 8 == 0

// gelu(y) = y * Phi(y), rounded to T as a separate activation module would.
template <typename T>
__device__ __forceinline__ float gelu_t(float y) {
  return to_f32<T>(from_f32<T>(0.5f * y * (1.f + erff(y * 0.70710678118654752f))));
}
// d gelu / dy = Phi(y) + y * phi(y).
__device__ __forceinline__ float gelu_grad(float y) {
  return 0.5f * (1.f + erff(y * 0.70710678118654752f)) +
         y * 0.39894228040143268f * expf(-0.5f * y * y);
}

// Eight consecutive elements as fp32 (one 16-byte load for 16-bit types) and
// back (one 16-byte store).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
  return x;
}

// kPath: 0 = 8-column chunks in registers (D % 8 == 0, D <= 1024), 1 = single
// columns in registers (D <= 1024), 2 = long rows, gelu recomputed per pass.
template <typename T, int kPath>
__global__ void __launch_bounds__(kRowWarps * 32)
    transform_fwd_kernel(const T* __restrict__ y, const T* __restrict__ gamma,
                         const T* __restrict__ beta, float eps, int rows, int D,
                         T* __restrict__ h, float* __restrict__ mean_out,
                         float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const T* yr = y + static_cast<size_t>(r) * D;
  T* hr = h + static_cast<size_t>(r) * D;
  const float inv_d = 1.f / static_cast<float>(D);
  float mean, rstd;
  if constexpr (kPath == 0) {
    // lane l owns the 8-column chunks l, l + 32, ...: 16-byte loads and stores
    float g[kVecPerLane][8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        load8<T>(yr + d, g[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          g[j][i] = gelu_t<T>(g[j][i]);
          s += g[j][i];
        }
      }
    }
    mean = warp_sum(s) * inv_d;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j)
      if (8 * (lane + 32 * j) < D)
#pragma unroll
        for (int i = 0; i < 8; ++i) q += (g[j][i] - mean) * (g[j][i] - mean);
    rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        float ga[8], be[8];
        load8<T>(gamma + d, ga);
        load8<T>(beta + d, be);
#pragma unroll
        for (int i = 0; i < 8; ++i) g[j][i] = (g[j][i] - mean) * rstd * ga[i] + be[i];
        store8<T>(hr + d, g[j]);
      }
    }
  } else if constexpr (kPath == 1) {
    float g[kMaxPerLane];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int d = lane + 32 * i;
      g[i] = d < D ? gelu_t<T>(to_f32<T>(yr[d])) : 0.f;
      s += g[i];
    }
    mean = warp_sum(s) * inv_d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int d = lane + 32 * i;
      const float c = d < D ? g[i] - mean : 0.f;
      q += c * c;
    }
    rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < D)
        hr[d] = from_f32<T>((g[i] - mean) * rstd * to_f32<T>(gamma[d]) + to_f32<T>(beta[d]));
    }
  } else {  // long rows: recompute gelu in each pass
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s += gelu_t<T>(to_f32<T>(yr[d]));
    mean = warp_sum(s) * inv_d;
    float q = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float c = gelu_t<T>(to_f32<T>(yr[d])) - mean;
      q += c * c;
    }
    rstd = rsqrtf(warp_sum(q) * inv_d + eps);
    for (int d = lane; d < D; d += 32)
      hr[d] = from_f32<T>((gelu_t<T>(to_f32<T>(yr[d])) - mean) * rstd * to_f32<T>(gamma[d]) +
                        to_f32<T>(beta[d]));
  }
  if (lane == 0) {
    mean_out[r] = mean;
    rstd_out[r] = rstd;
  }
}

// kPath 0: 8-column chunks in registers (D % 8 == 0, D <= 1024); else two
// passes over the row.
template <typename T, int kPath>
__global__ void __launch_bounds__(kRowWarps * 32)
    transform_bwd_row_kernel(const T* __restrict__ dh, const T* __restrict__ y,
                             const T* __restrict__ gamma, const float* __restrict__ mean,
                             const float* __restrict__ rstd, int rows, int D,
                             T* __restrict__ dy) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const size_t o = static_cast<size_t>(r) * D;
  const float mu = mean[r], rs = rstd[r];
  const float inv_d = 1.f / static_cast<float>(D);
  if constexpr (kPath == 0) {
    // y stays in registers; dh and gamma are read again (from L1) in the
    // second pass.
    float yv[kVecPerLane][8];
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        float gv[8], ga[8];
        load8<T>(y + o + d, yv[j]);
        load8<T>(dh + o + d, gv);
        load8<T>(gamma + d, ga);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float dxh = gv[i] * ga[i];
          a += dxh;
          b += dxh * (gelu_t<T>(yv[j][i]) - mu) * rs;
        }
      }
    }
    a = warp_sum(a) * inv_d;
    b = warp_sum(b) * inv_d;
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        float gv[8], ga[8], out[8];
        load8<T>(dh + o + d, gv);
        load8<T>(gamma + d, ga);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = (gelu_t<T>(yv[j][i]) - mu) * rs;
          out[i] = rs * (gv[i] * ga[i] - a - xh * b) * gelu_grad(yv[j][i]);
        }
        store8<T>(dy + o + d, out);
      }
    }
    return;
  } else {
  // mean(dxh) and mean(dxh * xh) over the row
  float a = 0.f, b = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float yv = to_f32<T>(y[o + d]);
    const float xh = (gelu_t<T>(yv) - mu) * rs;
    const float dxh = to_f32<T>(dh[o + d]) * to_f32<T>(gamma[d]);
    a += dxh;
    b += dxh * xh;
  }
  a = warp_sum(a) * inv_d;
  b = warp_sum(b) * inv_d;
  for (int d = lane; d < D; d += 32) {
    const float yv = to_f32<T>(y[o + d]);
    const float xh = (gelu_t<T>(yv) - mu) * rs;
    const float dxh = to_f32<T>(dh[o + d]) * to_f32<T>(gamma[d]);
    const float dg = rs * (dxh - a - xh * b);
    dy[o + d] = from_f32<T>(dg * gelu_grad(yv));
  }
  }
}

// D % 8 == 0, D <= 256 * kNv: the row pass and the column partial sums in one
// kernel. CTA c takes the rows [c * rows / grid, (c + 1) * rows / grid), warp
// w every eighth of them from the w-th; lane l owns the 8-column chunks l,
// l + 32, ... One erff and one expf per element: the first pass keeps (dh,
// xh, gelu'(y)) of each element in registers, the second writes dy and adds
// dh * xh, dh and the rounded dy into the warp's column sums in shared memory
// (each lane its own columns: no atomics). Shared arrays indexed by a lane's
// column are stored lane-minor, element (j, i) of lane l at (j * 8 + i) * 32
// + l, so a warp's accesses fall in 32 distinct banks. The CTA then adds its
// warps' sums in warp order into partials[c][k][col] (k = gamma, beta, bias)
// when partials is not NULL. The grid depends on rows only, so the column
// sums are deterministic.
template <typename T, int kNv>
__global__ void __launch_bounds__(kRowWarps * 32, 2)
    transform_bwd_fused_kernel(const T* __restrict__ dh, const T* __restrict__ y,
                               const T* __restrict__ gamma, const float* __restrict__ mean,
                               const float* __restrict__ rstd, int rows, int D,
                               T* __restrict__ dy, float* __restrict__ partials) {
  constexpr int kSlots = kNv * 8 * 32;  // lane-minor slots of one [D] array
  extern __shared__ float sh[];
  float* sgamma = sh;                   // [kSlots]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* acc = sh + kSlots + static_cast<size_t>(warp) * 3 * kSlots;  // this warp's [3][kSlots]
  const bool want = partials != nullptr;
  auto slot = [](int d) {  // column d -> its lane-minor slot
    const int j = d >> 8, l = (d >> 3) & 31, i = d & 7;
    return (j * 8 + i) * 32 + l;
  };
  for (int d = threadIdx.x; d < kNv * 256; d += kRowWarps * 32)
    sgamma[slot(d)] = d < D ? to_f32<T>(gamma[d]) : 0.f;
  if (want)
    for (int i = lane; i < 3 * kSlots; i += 32) acc[i] = 0.f;
  __syncthreads();
  const long long r_lo = static_cast<long long>(blockIdx.x) * rows / gridDim.x;
  const long long r_hi = static_cast<long long>(blockIdx.x + 1) * rows / gridDim.x;
  const float inv_d = 1.f / static_cast<float>(D);
  for (long long r = r_lo + warp; r < r_hi; r += kRowWarps) {
    const size_t o = static_cast<size_t>(r) * D;
    const float mu = mean[r], rs = rstd[r];
    float gv[kNv][8], xh[kNv][8], gp[kNv][8];
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int j = 0; j < kNv; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        float yv[8];
        load8<T>(y + o + d, yv);
        load8<T>(dh + o + d, gv[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float e = erff(yv[i] * 0.70710678118654752f);
          // gelu rounded to T, and d gelu / dy = Phi(y) + y * phi(y)
          const float g = to_f32<T>(from_f32<T>(0.5f * yv[i] * (1.f + e)));
          gp[j][i] = 0.5f * (1.f + e) + yv[i] * 0.39894228040143268f * expf(-0.5f * yv[i] * yv[i]);
          xh[j][i] = (g - mu) * rs;
          const float dxh = gv[j][i] * sgamma[(j * 8 + i) * 32 + lane];
          a += dxh;
          b += dxh * xh[j][i];
        }
      }
    }
    a = warp_sum(a) * inv_d;
    b = warp_sum(b) * inv_d;
#pragma unroll
    for (int j = 0; j < kNv; ++j) {
      const int d = 8 * (lane + 32 * j);
      if (d < D) {
        float out[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          out[i] = rs * (gv[j][i] * sgamma[(j * 8 + i) * 32 + lane] - a - xh[j][i] * b) * gp[j][i];
        store8<T>(dy + o + d, out);
        if (want) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int q = (j * 8 + i) * 32 + lane;
            acc[q] += gv[j][i] * xh[j][i];
            acc[kSlots + q] += gv[j][i];
            acc[2 * kSlots + q] += to_f32<T>(from_f32<T>(out[i]));
          }
        }
      }
    }
  }
  if (!want) return;
  __syncthreads();
  const float* all = sh + kSlots;
  for (int c = threadIdx.x; c < 3 * D; c += kRowWarps * 32) {
    const int k = c / D, d = c - k * D;
    const int q = k * kSlots + slot(d);
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) t += all[static_cast<size_t>(w) * 3 * kSlots + q];
    partials[static_cast<size_t>(blockIdx.x) * 3 * D + c] = t;
  }
}

// CTA (column block cx of 32, row block ry of kColRows): lane = column, the 8
// warps stride the rows; partials[ry][k][col] for k = gamma, beta, bias.
template <typename T>
__global__ void __launch_bounds__(256)
    transform_bwd_col_kernel(const T* __restrict__ dh, const T* __restrict__ y,
                             const T* __restrict__ dy, const float* __restrict__ mean,
                             const float* __restrict__ rstd, int rows, int D,
                             float* __restrict__ partials) {
  __shared__ float s[3][8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  const int r0 = blockIdx.y * kColRows, r1 = min(rows, r0 + kColRows);
  float pg = 0.f, pb = 0.f, pd = 0.f;
  if (col < D) {
    for (int r = r0 + warp; r < r1; r += 8) {
      const size_t o = static_cast<size_t>(r) * D + col;
      const float g = to_f32<T>(dh[o]);
      const float xh = (gelu_t<T>(to_f32<T>(y[o])) - mean[r]) * rstd[r];
      pg += g * xh;
      pb += g;
      pd += to_f32<T>(dy[o]);
    }
  }
  s[0][warp][lane] = pg;
  s[1][warp][lane] = pb;
  s[2][warp][lane] = pd;
  __syncthreads();
  if (warp < 3 && col < D) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += s[warp][w][lane];
    partials[(static_cast<size_t>(blockIdx.y) * 3 + warp) * D + col] = t;
  }
}

// D % 8 == 0: CTA (column block cx of 256, row block ry of kColRows); lane l
// owns columns cx*256 + 8l .. +7 (16-byte loads), the 8 warps stride the rows
// and are added in warp order through shared memory.
template <typename T>
__global__ void __launch_bounds__(256)
    transform_bwd_col8_kernel(const T* __restrict__ dh, const T* __restrict__ y,
                              const T* __restrict__ dy, const float* __restrict__ mean,
                              const float* __restrict__ rstd, int rows, int D,
                              float* __restrict__ partials) {
  __shared__ float s[8][3][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * kColRows, r1 = min(rows, r0 + kColRows);
  float pg[8], pb[8], pd[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) pg[i] = pb[i] = pd[i] = 0.f;
  if (c0 < D) {
    for (int r = r0 + warp; r < r1; r += 8) {
      const size_t o = static_cast<size_t>(r) * D + c0;
      const float mu = mean[r], rs = rstd[r];
      float gv[8], yv[8], dv[8];
      load8<T>(dh + o, gv);
      load8<T>(y + o, yv);
      load8<T>(dy + o, dv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pg[i] += gv[i] * (gelu_t<T>(yv[i]) - mu) * rs;
        pb[i] += gv[i];
        pd[i] += dv[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s[warp][0][lane * 8 + i] = pg[i];
    s[warp][1][lane * 8 + i] = pb[i];
    s[warp][2][lane * 8 + i] = pd[i];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < 3 * 256; t += 256) {
    const int k = t / 256, cc = t % 256;
    const int col = blockIdx.x * 256 + cc;
    if (col < D) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) acc += s[w][k][cc];
      partials[(static_cast<size_t>(blockIdx.y) * 3 + k) * D + col] = acc;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
    transform_col_reduce(const float* __restrict__ partials, int nblocks, int D,
                         T* __restrict__ d_gamma, T* __restrict__ d_beta, T* __restrict__ d_bias) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= D) return;
  float g = 0.f, b = 0.f, c = 0.f;
  for (int i = 0; i < nblocks; ++i) {
    g += partials[(static_cast<size_t>(i) * 3 + 0) * D + col];
    b += partials[(static_cast<size_t>(i) * 3 + 1) * D + col];
    c += partials[(static_cast<size_t>(i) * 3 + 2) * D + col];
  }
  if (d_gamma != nullptr) d_gamma[col] = from_f32<T>(g);
  if (d_beta != nullptr) d_beta[col] = from_f32<T>(b);
  if (d_bias != nullptr) d_bias[col] = from_f32<T>(c);
}

bool vec_path(int D) { return D % 8 == 0 && D <= 8 * 32 * kVecPerLane; }

template <typename T>
int fwd_typed(const void* y, const void* gamma, const void* beta, float eps, int rows, int D,
              void* h, float* mean, float* rstd, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((rows + kRowWarps - 1) / kRowWarps);
  auto go = [&](auto kernel) {
    kernel<<<grid, kRowWarps * 32, 0, stream>>>(
        static_cast<const T*>(y), static_cast<const T*>(gamma), static_cast<const T*>(beta), eps,
        rows, D, static_cast<T*>(h), mean, rstd);
  };
  if (vec_path(D))
    go(transform_fwd_kernel<T, 0>);
  else if (D <= 32 * kMaxPerLane)
    go(transform_fwd_kernel<T, 1>);
  else
    go(transform_fwd_kernel<T, 2>);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "transform_fwd_kernel launch");
}

// CTAs of transform_bwd_fused_kernel: two per SM of a B200 (a constant, so the
// column sums' order depends on the shape only), at least 8 rows each.
constexpr int kFusedCtas = 2 * 148;
int fused_grid(int rows) { return std::max(1, std::min(kFusedCtas, (rows + 7) / 8)); }
size_t fused_smem(int D) {
  const size_t slots = static_cast<size_t>((D + 255) / 256) * 256;  // kNv * 8 * 32
  return (slots + kRowWarps * 3 * slots) * sizeof(float);
}

template <typename T, int kNv>
int bwd_fused(const void* dh, const void* y, const void* gamma, const float* mean,
              const float* rstd, int rows, int D, void* dy, void* d_gamma, void* d_beta,
              void* d_bias, float* partials, cudaStream_t stream) {
  const bool params = d_gamma != nullptr || d_beta != nullptr || d_bias != nullptr;
  const int grid = fused_grid(rows);
  const size_t smem = fused_smem(D);
  auto kernel = transform_bwd_fused_kernel<T, kNv>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "transform_bwd_fused_kernel smem");
  kernel<<<grid, kRowWarps * 32, smem, stream>>>(
      static_cast<const T*>(dh), static_cast<const T*>(y), static_cast<const T*>(gamma), mean, rstd,
      rows, D, static_cast<T*>(dy), params ? partials : nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "transform_bwd_fused_kernel launch");
  if (!params) return SPARTON_OK;
  transform_col_reduce<T><<<(D + 255) / 256, 256, 0, stream>>>(
      partials, grid, D, static_cast<T*>(d_gamma), static_cast<T*>(d_beta), static_cast<T*>(d_bias));
  e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "transform_col_reduce launch");
}

template <typename T>
int bwd_typed(const void* dh, const void* y, const void* gamma, const float* mean,
              const float* rstd, int rows, int D, void* dy, void* d_gamma, void* d_beta,
              void* d_bias, float* partials, cudaStream_t stream) {
  if (vec_path(D)) {
    const int nv = (D + 255) / 256;
    auto f = nv == 1 ? bwd_fused<T, 1> : nv == 2 ? bwd_fused<T, 2> : nv == 3 ? bwd_fused<T, 3>
                                                                             : bwd_fused<T, 4>;
    return f(dh, y, gamma, mean, rstd, rows, D, dy, d_gamma, d_beta, d_bias, partials, stream);
  }
  const unsigned grid = static_cast<unsigned>((rows + kRowWarps - 1) / kRowWarps);
  auto go = [&](auto kernel) {
    kernel<<<grid, kRowWarps * 32, 0, stream>>>(static_cast<const T*>(dh), static_cast<const T*>(y),
                                                static_cast<const T*>(gamma), mean, rstd, rows, D,
                                                static_cast<T*>(dy));
  };
  if (vec_path(D))
    go(transform_bwd_row_kernel<T, 0>);
  else
    go(transform_bwd_row_kernel<T, 1>);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "transform_bwd_row_kernel launch");
  if (d_gamma == nullptr && d_beta == nullptr && d_bias == nullptr) return SPARTON_OK;
  const int nb = (rows + kColRows - 1) / kColRows;
  if (D % 8 == 0) {
    const dim3 cgrid(static_cast<unsigned>((D + 255) / 256), static_cast<unsigned>(nb));
    transform_bwd_col8_kernel<T><<<cgrid, 256, 0, stream>>>(
        static_cast<const T*>(dh), static_cast<const T*>(y), static_cast<const T*>(dy), mean,
        rstd, rows, D, partials);
  } else {
    const dim3 cgrid(static_cast<unsigned>((D + 31) / 32), static_cast<unsigned>(nb));
    transform_bwd_col_kernel<T><<<cgrid, 256, 0, stream>>>(
        static_cast<const T*>(dh), static_cast<const T*>(y), static_cast<const T*>(dy), mean,
        rstd, rows, D, partials);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "transform_bwd_col_kernel launch");
  transform_col_reduce<T><<<(D + 255) / 256, 256, 0, stream>>>(
      partials, nb, D, static_cast<T*>(d_gamma), static_cast<T*>(d_beta), static_cast<T*>(d_bias));
  e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "transform_col_reduce launch");
}

}  // namespace

size_t transform_workspace_bytes(int64_t rows, int64_t D) {
  int64_t nb = (rows + kColRows - 1) / kColRows;  // column kernels' row blocks
  if (vec_path(static_cast<int>(D)))
    nb = fused_grid(static_cast<int>(std::min<int64_t>(rows, 1 << 30)));
  return align256(static_cast<size_t>(nb > 0 ? nb : 1) * 3 * static_cast<size_t>(D) * sizeof(float));
}

int launch_transform_fwd(int dtype, const void* y, const void* gamma, const void* beta, float eps,
                         int rows, int D, void* h, float* mean, float* rstd, cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return fwd_typed<__nv_bfloat16>(y, gamma, beta, eps, rows, D, h, mean, rstd, stream);
    case SPARTON_DTYPE_F16:
      return fwd_typed<__half>(y, gamma, beta, eps, rows, D, h, mean, rstd, stream);
    case SPARTON_DTYPE_F32:
      return fwd_typed<float>(y, gamma, beta, eps, rows, D, h, mean, rstd, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

int launch_transform_bwd(int dtype, const void* dh, const void* y, const void* gamma,
                         const float* mean, const float* rstd, int rows, int D, void* dy,
                         void* d_gamma, void* d_beta, void* d_bias, void* workspace,
                         cudaStream_t stream) {
  float* partials = static_cast<float*>(workspace);
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return bwd_typed<__nv_bfloat16>(dh, y, gamma, mean, rstd, rows, D, dy, d_gamma, d_beta,
                                      d_bias, partials, stream);
    case SPARTON_DTYPE_F16:
      return bwd_typed<__half>(dh, y, gamma, mean, rstd, rows, D, dy, d_gamma, d_beta, d_bias,
                               partials, stream);
    case SPARTON_DTYPE_F32:
      return bwd_typed<float>(dh, y, gamma, mean, rstd, rows, D, dy, d_gamma, d_beta, d_bias,
                              partials, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

}  // namespace sparton
