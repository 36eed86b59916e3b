// bwd.cu — K2..K4: backward of the SPLADE head without atomics.
//
// Upstream (hhkbble/sparton src/sparton/sparton_kernel.py:472-565) runs one
// Triton kernel over (vocab block, batch block) tiles that computes
//   g' = where(score > 0, g * exp(-score), 0)                         (:531)
// and scatters it with fp32 atomics: db[v] += sum_b g' (:536),
// dW[v,:] += sum_b g' * H[b, idx[b,v], :] (:554-557) and, the dominant cost,
// dH[b, idx[b,v], :] += g' * W[v,:] element by element (:559-561).
//
// Here the same sums are computed gather-side, each output element by exactly
// one thread in a fixed order, so the result is deterministic:
//   K2 bwd_sort_kernel   per batch row, a stable counting sort of the vocab ids
//                        with score > 0 by their argmax position -> CSR
//                        (offs[b][s] .. offs[b][s+1]) of (v, g') pairs.
//   K3 dh_kernel         one warp per (b, s): dH[b,s,:] = sum over its bucket of
//                        g' * W[v,:] (rows gathered, fp32 accumulation).
//   K4 dw_kernel         one warp per v: dW[v,:] = sum_b g' * H[b, idx[b,v], :].
//      db_kernel         one thread per v: db[v] = sum_b g'.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "internal.h"

namespace sparton {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) {
  return __half2float(__ldg(p));
}
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(__ldg(p));
}

// g' of one (b, v) entry; 0 when the head's output is 0 (max logit <= 0).
template <typename T>
__device__ __forceinline__ float scaled_grad(const T* g, const T* reps, size_t o) {
  const float sc = ld_f<T>(reps + o);
  return sc > 0.f ? ld_f<T>(g + o) * expf(-sc) : 0.f;
}

// Eight consecutive elements of a row -> fp32 (16-bit types: one 16-byte load).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&x)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&x)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename O>
__device__ __forceinline__ void store8(O* p, const float (&x)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&x)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&x)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&x)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <typename O>
__device__ __forceinline__ O cvt_out(float x);
template <>
__device__ __forceinline__ float cvt_out<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half cvt_out<__half>(float x) {
  return __float2half_rn(x);
}

// ------------------------------------------------------------------ K2: sort
// One block per batch row, `nw` warps. Warp w owns the contiguous vocab range
// [w*chunk, (w+1)*chunk) and a row `cnt[w][0..S)` of the shared table.
//   pass 1: cnt[w][s] = number of entries of warp w with argmax s
//   scan:   offs[b][s] = exclusive prefix over s of the column sums; then each
//           cnt[w][s] becomes the first output slot of warp w in bucket s
//   pass 2: each warp replays its range in order and writes (v, g') at
//           cnt[w][s] + (rank among lower lanes with the same s) -> stable.
template <typename T>
__global__ void __launch_bounds__(1024)
    bwd_sort_kernel(const T* __restrict__ g, const T* __restrict__ reps,
                    const int32_t* __restrict__ idx, int S, int V, int* __restrict__ offs,
                    int* __restrict__ perm, float* __restrict__ gperm) {
  extern __shared__ int cnt[];  // [nw][S]
  __shared__ int scan_tmp[33];
  const int b = blockIdx.x;
  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < nw * S; i += blockDim.x) cnt[i] = 0;
  __syncthreads();

  const int chunk = (((V + nw - 1) / nw) + 31) & ~31;
  const int v_begin = warp * chunk;
  const int v_end = min(V, v_begin + chunk);
  const size_t row = static_cast<size_t>(b) * V;
  int* my = cnt + warp * S;

  for (int base = v_begin; base < v_end; base += 32) {
    const int v = base + lane;
    int key = -1;
    if (v < v_end) {
      const float sc = ld_f<T>(reps + row + v);
      const int s = __ldg(idx + row + v);
      if (sc > 0.f && s >= 0 && s < S) key = s;
    }
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
    if (key >= 0 && lane == __ffs(peers) - 1) my[key] += __popc(peers);
  }
  __syncthreads();

  // Exclusive scan over positions of the per-position totals.
  const int per = (S + blockDim.x - 1) / blockDim.x;
  const int k_begin = min(S, threadIdx.x * per), k_end = min(S, k_begin + per);
  int local = 0;
  for (int k = k_begin; k < k_end; ++k)
    for (int w = 0; w < nw; ++w) local += cnt[w * S + k];
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) scan_tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nw ? scan_tmp[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) scan_tmp[lane] = t;  // inclusive per-warp totals
    if (lane == 31) scan_tmp[32] = t;
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? scan_tmp[warp - 1] : 0);
  int* orow = offs + static_cast<size_t>(b) * (S + 1);
  for (int k = k_begin; k < k_end; ++k) {
    orow[k] = run;
    for (int w = 0; w < nw; ++w) {
      const int c = cnt[w * S + k];
      cnt[w * S + k] = run;
      run += c;
    }
  }
  if (threadIdx.x == 0) orow[S] = scan_tmp[32];
  __syncthreads();

  int* prow = perm + row;
  float* grow = gperm + row;
  const unsigned lt = (1u << lane) - 1u;
  for (int base = v_begin; base < v_end; base += 32) {
    const int v = base + lane;
    int key = -1;
    float gp = 0.f;
    if (v < v_end) {
      const float sc = ld_f<T>(reps + row + v);
      const int s = __ldg(idx + row + v);
      if (sc > 0.f && s >= 0 && s < S) {
        key = s;
        gp = ld_f<T>(g + row + v) * expf(-sc);
      }
    }
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
    int slot = 0;
    if (key >= 0) slot = my[key] + __popc(peers & lt);
    __syncwarp();
    if (key >= 0) {
      prow[slot] = v;
      grow[slot] = gp;
      if (lane == __ffs(peers) - 1) my[key] += __popc(peers);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ K3: dH
// One warp per (b, s) row. A pass covers up to 1024 columns: lane l handles
// columns d0 + c*256 + 8l .. +7 for c = 0..3. Bucket entries are processed
// four at a time so four W rows are in flight per lane.
template <typename T, typename O>
__global__ void __launch_bounds__(256)
    dh_kernel(const T* __restrict__ W, const int* __restrict__ offs, const int* __restrict__ perm,
              const float* __restrict__ gperm, int B, int S, int D, int V, O* __restrict__ dH) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long rowid = static_cast<long long>(blockIdx.x) * 8 + warp;
  if (rowid >= static_cast<long long>(B) * S) return;
  const int b = static_cast<int>(rowid / S);
  const int s = static_cast<int>(rowid % S);
  const int* orow = offs + static_cast<size_t>(b) * (S + 1);
  const int o0 = __ldg(orow + s), o1 = __ldg(orow + s + 1);
  const int* pv = perm + static_cast<size_t>(b) * V;
  const float* pg = gperm + static_cast<size_t>(b) * V;
  O* out = dH + static_cast<size_t>(rowid) * D;
  for (int d0 = 0; d0 < D; d0 += 1024) {
    float acc[4][8];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
    int e = o0;
    for (; e + 4 <= o1; e += 4) {
      int vv[4];
      float gg[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        vv[u] = __ldg(pv + e + u);
        gg[u] = __ldg(pg + e + u);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int d = d0 + c * 256 + lane * 8;
        if (d < D) {
          float x[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u) load8<T>(W + static_cast<size_t>(vv[u]) * D + d, x[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[c][i] = fmaf(gg[u], x[u][i], acc[c][i]);
        }
      }
    }
    for (; e < o1; ++e) {
      const int v = __ldg(pv + e);
      const float gv = __ldg(pg + e);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int d = d0 + c * 256 + lane * 8;
        if (d < D) {
          float x[8];
          load8<T>(W + static_cast<size_t>(v) * D + d, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[c][i] = fmaf(gv, x[i], acc[c][i]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = d0 + c * 256 + lane * 8;
      if (d < D) store8<O>(out + d, acc[c]);
    }
  }
}

// ------------------------------------------------------------------ K4: dW
// One warp per vocab id, batch rows in order, four at a time.
template <typename T, typename O>
__global__ void __launch_bounds__(256)
    dw_kernel(const T* __restrict__ g, const T* __restrict__ reps, const int32_t* __restrict__ idx,
              const T* __restrict__ H, int B, int S, int D, int V, O* __restrict__ dW) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v = blockIdx.x * 8 + warp;
  if (v >= V) return;
  O* out = dW + static_cast<size_t>(v) * D;
  for (int d0 = 0; d0 < D; d0 += 1024) {
    float acc[4][8];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
    for (int b0 = 0; b0 < B; b0 += 4) {
      float gg[4];
      const T* rows[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        gg[u] = 0.f;
        rows[u] = H;
        const int b = b0 + u;
        if (b < B) {
          const size_t o = static_cast<size_t>(b) * V + v;
          const float gp = scaled_grad<T>(g, reps, o);
          const int s = __ldg(idx + o);
          if (gp != 0.f && s >= 0 && s < S) {
            gg[u] = gp;
            rows[u] = H + (static_cast<size_t>(b) * S + s) * D;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int d = d0 + c * 256 + lane * 8;
        if (d < D) {
          float x[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (gg[u] != 0.f) {
              load8<T>(rows[u] + d, x[u]);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) x[u][i] = 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[c][i] = fmaf(gg[u], x[u][i], acc[c][i]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = d0 + c * 256 + lane * 8;
      if (d < D) store8<O>(out + d, acc[c]);
    }
  }
}

template <typename T, typename O>
__global__ void __launch_bounds__(256) db_kernel(const T* __restrict__ g, const T* __restrict__ reps,
                                                 int B, int V, O* __restrict__ db) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  float acc = 0.f;
  for (int b = 0; b < B; ++b) acc += scaled_grad<T>(g, reps, static_cast<size_t>(b) * V + v);
  db[v] = cvt_out<O>(acc);
}

template <typename T, typename O>
int launch_dh(const void* grad_reps, const void* reps, const int32_t* idx, const void* weight,
              int B, int S, int D, int V, void* d_hidden, const BwdWorkspace& ws,
              cudaStream_t stream) {
  int nw = 49152 / S;
  if (nw > 32) nw = 32;
  if (nw < 1) return fail(SPARTON_ERR_UNSUPPORTED, "backward supports S <= 49152 (got %d)", S);
  const size_t smem = static_cast<size_t>(nw) * S * sizeof(int);
  cudaError_t e;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(bwd_sort_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bwd_sort_kernel)");
  }
  bwd_sort_kernel<T><<<B, nw * 32, smem, stream>>>(static_cast<const T*>(grad_reps),
                                                   static_cast<const T*>(reps), idx, S, V, ws.offs,
                                                   ws.perm, ws.gperm);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_sort_kernel launch");
  const long long rows = static_cast<long long>(B) * S;
  dh_kernel<T, O><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      static_cast<const T*>(weight), ws.offs, ws.perm, ws.gperm, B, S, D, V,
      static_cast<O*>(d_hidden));
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dh_kernel launch");
  return SPARTON_OK;
}

template <typename T, typename O>
int launch_params(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
                  int B, int S, int D, int V, void* d_weight, void* d_bias, cudaStream_t stream) {
  const T* g = static_cast<const T*>(grad_reps);
  const T* r = static_cast<const T*>(reps);
  cudaError_t e;
  if (d_weight != nullptr) {
    dw_kernel<T, O><<<(V + 7) / 8, 256, 0, stream>>>(g, r, idx, static_cast<const T*>(hidden), B,
                                                     S, D, V, static_cast<O*>(d_weight));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "dw_kernel launch");
  }
  if (d_bias != nullptr) {
    db_kernel<T, O><<<(V + 255) / 256, 256, 0, stream>>>(g, r, B, V, static_cast<O*>(d_bias));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "db_kernel launch");
  }
  return SPARTON_OK;
}

template <typename T>
int launch_in(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
              const void* weight, int B, int S, int D, int V, void* d_hidden, void* d_weight,
              void* d_bias, int dh_dtype, int dp_dtype, const BwdWorkspace& ws,
              cudaStream_t stream) {
  if (d_hidden != nullptr) {
    const int st =
        dh_dtype == SPARTON_DTYPE_F32
            ? launch_dh<T, float>(grad_reps, reps, idx, weight, B, S, D, V, d_hidden, ws, stream)
            : launch_dh<T, T>(grad_reps, reps, idx, weight, B, S, D, V, d_hidden, ws, stream);
    if (st != SPARTON_OK) return st;
  }
  if (d_weight == nullptr && d_bias == nullptr) return SPARTON_OK;
  return dp_dtype == SPARTON_DTYPE_F32
             ? launch_params<T, float>(grad_reps, reps, idx, hidden, B, S, D, V, d_weight, d_bias,
                                       stream)
             : launch_params<T, T>(grad_reps, reps, idx, hidden, B, S, D, V, d_weight, d_bias,
                                   stream);
}

}  // namespace

int launch_bwd(int dtype, const void* grad_reps, const void* reps, const int32_t* idx,
               const void* hidden, const void* weight, int B, int S, int D, int V,
               void* d_hidden, void* d_weight, void* d_bias, int d_hidden_dtype,
               int d_param_dtype, const BwdWorkspace& ws, cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_in<__nv_bfloat16>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                                      d_weight, d_bias, d_hidden_dtype, d_param_dtype, ws, stream);
    case SPARTON_DTYPE_F16:
      return launch_in<__half>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                               d_weight, d_bias, d_hidden_dtype, d_param_dtype, ws, stream);
    case SPARTON_DTYPE_F32:
      return launch_in<float>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                              d_weight, d_bias, d_hidden_dtype, d_param_dtype, ws, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

}  // namespace sparton
