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
//                        (offs[b][s] .. offs[b][s+1]) of (v, g') pairs; it also
//                        writes the vocab-major list of (H row b*S+idx, g') that
//                        dW reads.
//   K3/K4 gather_reduce_kernel, one warp per output row:
//                        dH[b,s,:] = sum over bucket (b,s) of g' * W[v,:]
//                        dW[v,:]   = sum over b of g' * H[b*S + idx[b,v], :]
//                        (+ db[v] = sum over b of g' in the same pass).
//      db_kernel         db alone, when dW is not requested.
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
                    const int32_t* __restrict__ idx, int B, int S, int V, int* __restrict__ offs,
                    int* __restrict__ perm, float* __restrict__ gperm, int* __restrict__ wrow,
                    float* __restrict__ wcoef) {
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
    if (v < v_end) {
      // Vocab-major entry for dW: every (v, b) gets one, with g' = 0 when the
      // head's output is 0 (the row index is then a harmless valid row).
      const size_t t = static_cast<size_t>(v) * B + b;
      wrow[t] = b * S + (key >= 0 ? key : 0);
      wcoef[t] = gp;
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

// --------------------------------------------------------- K3/K4: gather-reduce
// out[r, :] = sum over the entry list of row r of coef[e] * src[row[e], :].
//   kMode 0 (dH): r = b*S + s, list = bucket (b, s) of the CSR, src = W.
//   kMode 1 (dW): r = v, list = the B entries of v, src = H; the coefficient
//                 sum of the list is db[v].
// One warp per output row. A pass covers NC*256 columns (lane l owns columns
// d0 + c*256 + 8l .. +7). Entries are fetched 32 at a time with one coalesced
// load and broadcast by shuffle; for each group of 4 entries every row load of
// the pass is issued before the FMAs, so 4*NC 16-byte loads per lane are in
// flight. Summation order is fixed: deterministic.
template <typename T>
struct Row8;
template <>
struct Row8<__nv_bfloat16> {
  uint4 r;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) {
    r = __ldg(reinterpret_cast<const uint4*>(p));
  }
  __device__ __forceinline__ void zero() { r = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void fma_into(float c, float (&acc)[8]) const {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] = fmaf(c, f.x, acc[2 * i]);
      acc[2 * i + 1] = fmaf(c, f.y, acc[2 * i + 1]);
    }
  }
};
template <>
struct Row8<__half> {
  uint4 r;
  __device__ __forceinline__ void load(const __half* p) {
    r = __ldg(reinterpret_cast<const uint4*>(p));
  }
  __device__ __forceinline__ void zero() { r = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void fma_into(float c, float (&acc)[8]) const {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      acc[2 * i] = fmaf(c, f.x, acc[2 * i]);
      acc[2 * i + 1] = fmaf(c, f.y, acc[2 * i + 1]);
    }
  }
};
template <>
struct Row8<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void fma_into(float c, float (&acc)[8]) const {
    acc[0] = fmaf(c, a.x, acc[0]); acc[1] = fmaf(c, a.y, acc[1]);
    acc[2] = fmaf(c, a.z, acc[2]); acc[3] = fmaf(c, a.w, acc[3]);
    acc[4] = fmaf(c, b.x, acc[4]); acc[5] = fmaf(c, b.y, acc[5]);
    acc[6] = fmaf(c, b.z, acc[6]); acc[7] = fmaf(c, b.w, acc[7]);
  }
};

constexpr int kGatherWarps = 8;
constexpr int kGatherUnroll = 4;

template <typename T, typename O, int NC, int kMode>
__global__ void __launch_bounds__(kGatherWarps * 32)
    gather_reduce_kernel(const T* __restrict__ src, int D, int n_rows, int S, int V, int B,
                         const int* __restrict__ offs, const int* __restrict__ ent_row,
                         const float* __restrict__ ent_coef, O* __restrict__ out,
                         O* __restrict__ out_sum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kGatherWarps + warp;
  if (r >= n_rows) return;
  int e0, e1;
  if (kMode == 0) {
    const int b = r / S, s = r - (r / S) * S;
    const int* o = offs + static_cast<size_t>(b) * (S + 1);
    e0 = b * V + __ldg(o + s);
    e1 = b * V + __ldg(o + s + 1);
  } else {
    e0 = r * B;
    e1 = e0 + B;
  }
  O* orow = out + static_cast<size_t>(r) * D;
  float csum = 0.f;
  for (int d0 = 0; d0 < D; d0 += NC * 256) {
    float acc[NC][8];
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
    for (int eb = e0; eb < e1; eb += 32) {
      const int n = min(32, e1 - eb);
      int my_row = 0;
      float my_coef = 0.f;
      if (lane < n) {
        my_row = __ldg(ent_row + eb + lane);
        my_coef = __ldg(ent_coef + eb + lane);
      }
      if (kMode == 1 && d0 == 0) csum += my_coef;
      for (int j = 0; j < n; j += kGatherUnroll) {
        int rr[kGatherUnroll];
        float cc[kGatherUnroll];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; ++u) {
          rr[u] = __shfl_sync(0xFFFFFFFFu, my_row, j + u);
          cc[u] = __shfl_sync(0xFFFFFFFFu, my_coef, j + u);
        }
        Row8<T> x[kGatherUnroll][NC];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; ++u)
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int d = d0 + c * 256 + lane * 8;
            if (cc[u] != 0.f && d < D)
              x[u][c].load(src + static_cast<size_t>(rr[u]) * D + d);
            else
              x[u][c].zero();
          }
#pragma unroll
        for (int u = 0; u < kGatherUnroll; ++u)
#pragma unroll
          for (int c = 0; c < NC; ++c) x[u][c].fma_into(cc[u], acc[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int d = d0 + c * 256 + lane * 8;
      if (d < D) store8<O>(orow + d, acc[c]);
    }
  }
  if (kMode == 1 && out_sum != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) csum += __shfl_xor_sync(0xFFFFFFFFu, csum, o);
    if (lane == 0) out_sum[r] = cvt_out<O>(csum);
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

template <typename T, typename O, int kMode>
int launch_gather(const T* src, int D, int n_rows, int S, int V, int B, const int* offs,
                  const int* ent_row, const float* ent_coef, O* out, O* out_sum,
                  cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((n_rows + kGatherWarps - 1) / kGatherWarps);
  const int block = kGatherWarps * 32;
  if (D <= 256)
    gather_reduce_kernel<T, O, 1, kMode><<<grid, block, 0, stream>>>(src, D, n_rows, S, V, B, offs,
                                                                     ent_row, ent_coef, out, out_sum);
  else if (D <= 512)
    gather_reduce_kernel<T, O, 2, kMode><<<grid, block, 0, stream>>>(src, D, n_rows, S, V, B, offs,
                                                                     ent_row, ent_coef, out, out_sum);
  else if (D <= 768)
    gather_reduce_kernel<T, O, 3, kMode><<<grid, block, 0, stream>>>(src, D, n_rows, S, V, B, offs,
                                                                     ent_row, ent_coef, out, out_sum);
  else
    gather_reduce_kernel<T, O, 4, kMode><<<grid, block, 0, stream>>>(src, D, n_rows, S, V, B, offs,
                                                                     ent_row, ent_coef, out, out_sum);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gather_reduce_kernel launch");
  return SPARTON_OK;
}

template <typename T>
int launch_sort(const void* grad_reps, const void* reps, const int32_t* idx, int B, int S, int V,
                const BwdWorkspace& ws, cudaStream_t stream) {
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
                                                   static_cast<const T*>(reps), idx, B, S, V,
                                                   ws.offs, ws.perm, ws.gperm, ws.wrow, ws.wcoef);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_sort_kernel launch");
  return SPARTON_OK;
}

template <typename T, typename OH, typename OP>
int launch_all(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
               const void* weight, int B, int S, int D, int V, void* d_hidden, void* d_weight,
               void* d_bias, const BwdWorkspace& ws, cudaStream_t stream) {
  if (d_hidden != nullptr || d_weight != nullptr) {
    const int st = launch_sort<T>(grad_reps, reps, idx, B, S, V, ws, stream);
    if (st != SPARTON_OK) return st;
  }
  if (d_hidden != nullptr) {
    const int st = launch_gather<T, OH, 0>(static_cast<const T*>(weight), D, B * S, S, V, B,
                                           ws.offs, ws.perm, ws.gperm, static_cast<OH*>(d_hidden),
                                           nullptr, stream);
    if (st != SPARTON_OK) return st;
  }
  if (d_weight != nullptr) {
    const int st = launch_gather<T, OP, 1>(static_cast<const T*>(hidden), D, V, S, V, B, nullptr,
                                           ws.wrow, ws.wcoef, static_cast<OP*>(d_weight),
                                           static_cast<OP*>(d_bias), stream);
    if (st != SPARTON_OK) return st;
  } else if (d_bias != nullptr) {
    db_kernel<T, OP><<<(V + 255) / 256, 256, 0, stream>>>(static_cast<const T*>(grad_reps),
                                                          static_cast<const T*>(reps), B, V,
                                                          static_cast<OP*>(d_bias));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "db_kernel launch");
  }
  return SPARTON_OK;
}

template <typename T>
int launch_in(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
              const void* weight, int B, int S, int D, int V, void* d_hidden, void* d_weight,
              void* d_bias, int dh_dtype, int dp_dtype, const BwdWorkspace& ws,
              cudaStream_t stream) {
  const bool hf = dh_dtype == SPARTON_DTYPE_F32, pf = dp_dtype == SPARTON_DTYPE_F32;
  if (hf && pf)
    return launch_all<T, float, float>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                                       d_weight, d_bias, ws, stream);
  if (hf)
    return launch_all<T, float, T>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                                   d_weight, d_bias, ws, stream);
  if (pf)
    return launch_all<T, T, float>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden,
                                   d_weight, d_bias, ws, stream);
  return launch_all<T, T, T>(grad_reps, reps, idx, hidden, weight, B, S, D, V, d_hidden, d_weight,
                             d_bias, ws, stream);
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
