// sparse.cu — sparse forms of the head's output reps [B, V] for indexing:
// the per-row CSR of the entries above a threshold, and the per-row top-k.
//
// Upstream (hhkbble/sparton training/model.py:141-144) `encode` returns the
// dense reps under no_grad, and training/train.py:205-210 logs the fraction
// of entries > 0; an inverted index stores each row's nonzero (vocab id,
// weight) pairs, or its k heaviest.
//
// CSR, three launches:
//   csr_count_kernel  one CTA per (row, chunk of kCsrChunk columns): number of
//                     entries > threshold -> chunk_cnt[b][chunk]
//   csr_scan_kernel   one CTA: exclusive scan of chunk_cnt in row-major order
//                     -> chunk_off, crow[b] (row starts), crow[B] (= nnz)
//   csr_fill_kernel   the count pass again, writing (column, value) at
//                     chunk_off + rank: columns ascending inside every row.
//                     Entries at or past `capacity` are not written (the
//                     caller sees nnz in crow[B]).
// Top-k, a cluster of up to 8 CTAs per row (enough CTAs for two per SM):
//   radix select on order-preserving unsigned keys (8 bits a pass: 2 passes
//   for 16-bit types, 4 for fp32; shared-memory histograms in which the lanes
//   holding the common digit, that of 0.0, add once), the CTAs' histograms
//   summed through
//   distributed shared memory, finds the k-th largest key K and how many of
//   its equals to take; one ordered pass collects the entries above K and the
//   first such equals in vocab order into CTA 0; a bitonic sort in its shared
//   memory orders the k by (value descending, vocab id ascending).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cooperative_groups.h>

#include "dtype.cuh"
#include "internal.h"

namespace sparton {
namespace {

constexpr int kCsrChunk = 4096;
constexpr int kCsrThreads = 256;
constexpr int kTopkThreads = 512;
constexpr int kTileU = 8;  // entries per lane per step of a row walk
constexpr size_t kTopkStageBudget = 200 * 1024;  // shared memory for a staged row part

// Order-preserving unsigned key of an element (larger value -> larger key;
// NaN above +inf, as torch.topk orders it) and its bit width.
template <typename T>
struct Key;
// `of` reads global memory through the read-only path; `at` reads any
// address (the row staged in shared memory).
template <>
struct Key<float> {
  static constexpr int kBits = 32;
  __device__ static __forceinline__ uint32_t conv(uint32_t u) {
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  __device__ static __forceinline__ uint32_t of(const float* p) {
    // The bits are loaded as an integer: no float-typed value carries a NaN.
    return conv(__ldg(reinterpret_cast<const unsigned int*>(p)));
  }
  __device__ static __forceinline__ uint32_t at(const float* p) {
    return conv(*reinterpret_cast<const unsigned int*>(p));
  }
};
template <typename T16>
struct Key16 {
  static constexpr int kBits = 16;
  __device__ static __forceinline__ uint32_t conv(uint32_t u) {
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  }
  __device__ static __forceinline__ uint32_t of(const T16* p) {
    return conv(__ldg(reinterpret_cast<const unsigned short*>(p)));
  }
  __device__ static __forceinline__ uint32_t at(const T16* p) {
    return conv(*reinterpret_cast<const unsigned short*>(p));
  }
};
template <>
struct Key<__half> : Key16<__half> {};
template <>
struct Key<__nv_bfloat16> : Key16<__nv_bfloat16> {};

__device__ __forceinline__ int block_sum(int x, int* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
  __syncthreads();
  if (lane == 0) tmp[warp] = x;
  __syncthreads();
  int t = 0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += tmp[w];
  return t;
}

// Exclusive prefix of `x` over the block (thread order) and the block total.
__device__ __forceinline__ int block_excl_scan(int x, int* tmp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = static_cast<int>(blockDim.x >> 5);
  int incl = x;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) tmp[warp] = incl;
  __syncthreads();
  int before = 0;
  total = 0;
  for (int w = 0; w < nw; ++w) {
    if (w < warp) before += tmp[w];
    total += tmp[w];
  }
  return before + incl - x;
}

// ------------------------------------------------------------------- CSR
// Each warp takes kTileU*32 consecutive columns per step (column
// base + u*32 + lane), all kTileU loads of a lane issued first.
template <typename T>
__global__ void __launch_bounds__(kCsrThreads)
    csr_count_kernel(const T* __restrict__ reps, int V, float thr, int nchunks,
                     int* __restrict__ chunk_cnt) {
  __shared__ int tmp[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y, ch = blockIdx.x;
  const int v0 = ch * kCsrChunk, v1 = min(V, v0 + kCsrChunk);
  const T* row = reps + static_cast<size_t>(b) * V;
  pdl_trigger();
  int n = 0;
  for (int base = v0 + warp * 32 * kTileU; base < v1; base += kCsrThreads * kTileU) {
    T x[kTileU];
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = base + u * 32 + lane;
      x[u] = v < v1 ? row[v] : T{};
    }
#pragma unroll
    for (int u = 0; u < kTileU; ++u) n += (base + u * 32 + lane < v1 && to_f32<T>(x[u]) > thr);
  }
  n = block_sum(n, tmp);
  if (threadIdx.x == 0) chunk_cnt[static_cast<size_t>(b) * nchunks + ch] = n;
}

__global__ void __launch_bounds__(1024)
    csr_scan_kernel(const int* __restrict__ chunk_cnt, int B, int nchunks,
                    int* __restrict__ chunk_off, int64_t* __restrict__ crow) {
  __shared__ int tmp[32];
  const int n = B * nchunks;
  int carry = 0;
  pdl_wait();  // the chunk counts
  pdl_trigger();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + static_cast<int>(threadIdx.x);
    const int x = i < n ? chunk_cnt[i] : 0;
    int total;
    const int ex = block_excl_scan(x, tmp, total);
    if (i < n) {
      chunk_off[i] = carry + ex;
      if (i % nchunks == 0) crow[i / nchunks] = carry + ex;
    }
    carry += total;
  }
  if (threadIdx.x == 0) crow[B] = carry;
}

template <typename T>
__global__ void __launch_bounds__(kCsrThreads)
    csr_fill_kernel(const T* __restrict__ reps, int V, float thr, int nchunks,
                    const int* __restrict__ chunk_off, int64_t capacity, int32_t* __restrict__ cols,
                    T* __restrict__ vals) {
  __shared__ int tmp[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const int b = blockIdx.y, ch = blockIdx.x;
  const int v0 = ch * kCsrChunk, v1 = min(V, v0 + kCsrChunk);
  const T* row = reps + static_cast<size_t>(b) * V;
  pdl_wait();  // the scanned chunk offsets
  int pos = chunk_off[static_cast<size_t>(b) * nchunks + ch];
  for (int base0 = v0; base0 < v1; base0 += kCsrThreads * kTileU) {
    const int base = base0 + warp * 32 * kTileU;
    T x[kTileU];
    unsigned keep[kTileU];
    int warp_n = 0;
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = base + u * 32 + lane;
      x[u] = v < v1 ? row[v] : T{};
    }
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = base + u * 32 + lane;
      keep[u] = __ballot_sync(0xFFFFFFFFu, v < v1 && to_f32<T>(x[u]) > thr);
      warp_n += __popc(keep[u]);
    }
    // Columns before this warp's span in the step, then earlier u, then lower lanes.
    int total;
    const int warp_before = block_excl_scan(lane == 0 ? warp_n : 0, tmp, total);
    int at = pos + __shfl_sync(0xFFFFFFFFu, warp_before, 0);
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      if ((keep[u] >> lane) & 1u) {
        const int i = at + __popc(keep[u] & lt);
        if (i < capacity) {
          cols[i] = base + u * 32 + lane;
          vals[i] = x[u];
        }
      }
      at += __popc(keep[u]);
    }
    pos += total;
  }
}

// ------------------------------------------------------------------ top-k
// A thread-block cluster of P CTAs per row (P = 1 .. 8); CTA c walks the vocab
// range [c*part, (c+1)*part). Shared memory: hist[256], then k_pad (key, id)
// pairs (used in CTA 0).
// kStaged: the CTA first copies its part of the row into shared memory (after
// the pair arrays) and every pass reads it there instead of from L2.
template <typename T, bool kStaged>
__global__ void __launch_bounds__(kTopkThreads)
    topk_kernel(const T* __restrict__ reps, int V, int k, int k_pad, T* __restrict__ out_vals,
                int32_t* __restrict__ out_idx) {
  extern __shared__ uint32_t smem[];
  uint32_t* hist = smem;            // [256]
  uint32_t* skey = smem + 256;      // [k_pad]
  int32_t* sid = reinterpret_cast<int32_t*>(skey + k_pad);  // [k_pad]
  T* srow = reinterpret_cast<T*>(sid + k_pad);              // [part] when kStaged
  __shared__ int tmp[32];
  __shared__ uint32_t s_prefix, s_remaining, s_eq_before, s_gt;
  namespace cg = cooperative_groups;
  const cg::cluster_group cluster = cg::this_cluster();
  const int P = static_cast<int>(cluster.num_blocks());
  const int c = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.y;
  const T* row = reps + static_cast<size_t>(b) * V;
  const int part = (((V + P - 1) / P) + 31) & ~31;
  const int v_lo = min(V, c * part), v_hi = min(V, v_lo + part);
  if (kStaged) {
    for (int i = threadIdx.x; i < v_hi - v_lo; i += kTopkThreads) srow[i] = row[v_lo + i];
    __syncthreads();
  }
  // the key of vocab id v of this CTA's part
  auto key_of = [&](int v) -> uint32_t {
    return kStaged ? Key<T>::at(srow + (v - v_lo)) : Key<T>::of(row + v);
  };
  constexpr int kBits = Key<T>::kBits;
  constexpr uint32_t kZeroKey = 1u << (kBits - 1);  // key of +0.0
  // Each warp takes kTileU*32 consecutive entries per step (entry
  // base + u*32 + lane), all kTileU loads of a lane issued first.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kStep = kTopkThreads * kTileU;
  if (threadIdx.x == 0) s_gt = 0;
  // One CTA per row: a block barrier and this CTA's own shared memory.
  auto csync = [&]() {
    if (P > 1)
      cluster.sync();
    else
      __syncthreads();
  };

  // Radix select over the whole row: after the pass on bits [shift, shift+8),
  // `prefix` holds the top bits of K and `remaining` how many elements with
  // that prefix still belong to the top k. Every CTA sums the cluster's
  // histograms itself (distributed shared memory) and picks the same digit.
  uint32_t prefix = 0, prefix_mask = 0;
  uint32_t remaining = static_cast<uint32_t>(k);
  for (int shift = kBits - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    // Most entries of a SPLADE row are 0: when the key of 0.0 is still in the
    // prefix group, its digit is the common one, otherwise lane 0's.
    const bool zero_in_group = (kZeroKey & prefix_mask) == prefix;
    const uint32_t zero_digit = (kZeroKey >> shift) & 0xFFu;
    for (int base = v_lo + warp * 32 * kTileU; base < v_hi; base += kStep) {
      uint32_t key[kTileU];
#pragma unroll
      for (int u = 0; u < kTileU; ++u) {
        const int v = base + u * 32 + lane;
        key[u] = v < v_hi ? key_of(v) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kTileU; ++u) {
        const int v = base + u * 32 + lane;
        const uint32_t d =
            (v < v_hi && (key[u] & prefix_mask) == prefix) ? (key[u] >> shift) & 0xFFu : 256u;
        // The lanes holding the common digit add once (one ballot); the rest
        // add one each.
        const uint32_t dc = zero_in_group ? zero_digit : __shfl_sync(0xFFFFFFFFu, d, 0);
        const unsigned same = __ballot_sync(0xFFFFFFFFu, d == dc);
        if (d == dc) {
          if (d < 256u && lane == __ffs(same) - 1) atomicAdd(&hist[d], __popc(same));
        } else if (d < 256u) {
          atomicAdd(&hist[d], 1u);
        }
      }
    }
    csync();  // every CTA's histogram is complete
    // Digits in descending order, one per thread: the digit whose bucket
    // holds the remaining-th largest key of the prefix group.
    const int t = static_cast<int>(threadIdx.x);
    uint32_t own = 0, before = 0;
    if (t < 256) {
      if (P == 1) {
        own = hist[255 - t];
      } else {
        for (int r = 0; r < P; ++r) {
          const uint32_t x = *cluster.map_shared_rank(hist + (255 - t), r);
          own += x;
          before += r < c ? x : 0u;
        }
      }
    }
    int total;
    const uint32_t above = static_cast<uint32_t>(block_excl_scan(static_cast<int>(own), tmp, total));
    if (t < 256 && above < remaining && above + own >= remaining) {
      s_prefix = prefix | (static_cast<uint32_t>(255 - t) << shift);
      s_remaining = remaining - above;
      s_eq_before = before;  // after the last pass: equals of K in the CTAs before this one
    }
    csync();  // no CTA reads another's histogram past this point
    prefix = s_prefix;
    remaining = s_remaining;
    prefix_mask |= 0xFFu << shift;
  }
  // K = prefix (all bits); take every key > K and the first `remaining`
  // equals in vocab order (rank = equals in earlier CTAs, then in earlier
  // warps' spans of the step, then earlier u, then lower lanes), written into
  // CTA 0's shared memory.
  const uint32_t K = prefix;
  const int n_gt = k - static_cast<int>(remaining);
  uint32_t* dkey = P > 1 ? cluster.map_shared_rank(skey, 0) : skey;
  int32_t* did = P > 1 ? cluster.map_shared_rank(sid, 0) : sid;
  uint32_t* dgt = P > 1 ? cluster.map_shared_rank(&s_gt, 0) : &s_gt;
  const unsigned lt = (1u << lane) - 1u;
  int eq_seen = static_cast<int>(s_eq_before);
  for (int base0 = v_lo; base0 < v_hi; base0 += kStep) {
    const int base = base0 + warp * 32 * kTileU;
    uint32_t key[kTileU];
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = base + u * 32 + lane;
      key[u] = v < v_hi ? key_of(v) : 0u;
    }
    unsigned eqm[kTileU];
    int warp_eq = 0;
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = base + u * 32 + lane;
      eqm[u] = __ballot_sync(0xFFFFFFFFu, v < v_hi && key[u] == K);
      warp_eq += __popc(eqm[u]);
      if (v < v_hi && key[u] > K) {
        const uint32_t at = atomicAdd(dgt, 1u);
        dkey[at] = key[u];
        did[at] = v;
      }
    }
    int total;
    const int warp_before = block_excl_scan(lane == 0 ? warp_eq : 0, tmp, total);
    int rank = eq_seen + __shfl_sync(0xFFFFFFFFu, warp_before, 0);
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      if ((eqm[u] >> lane) & 1u) {
        const int r = rank + __popc(eqm[u] & lt);
        if (r < static_cast<int>(remaining)) {
          dkey[n_gt + r] = key[u];
          did[n_gt + r] = base + u * 32 + lane;
        }
      }
      rank += __popc(eqm[u]);
    }
    eq_seen += total;
  }
  csync();  // CTA 0 holds all k candidates
  if (c != 0) return;
  for (int i = k + static_cast<int>(threadIdx.x); i < k_pad; i += kTopkThreads) {
    skey[i] = 0;  // below every real key in the descending order
    sid[i] = 0x7FFFFFFF;
  }
  __syncthreads();
  // Bitonic sort of (key desc, id asc) over k_pad entries.
  for (int size = 2; size <= k_pad; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < k_pad; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;  // this run sorts "before"-first
          const uint32_t ki = skey[i], kj = skey[j];
          const int32_t ii = sid[i], ij = sid[j];
          const bool i_before_j = ki > kj || (ki == kj && ii < ij);
          if (i_before_j != desc) {
            skey[i] = kj;
            skey[j] = ki;
            sid[i] = ij;
            sid[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < k; i += kTopkThreads) {
    const int32_t v = sid[i];
    out_idx[static_cast<size_t>(b) * k + i] = v;
    out_vals[static_cast<size_t>(b) * k + i] = row[v];
  }
}

template <typename T>
int launch_csr_typed(const void* reps, int B, int V, float thr, int64_t* crow, int32_t* cols,
                     void* vals, int64_t capacity, const SparseWorkspace& ws,
                     cudaStream_t stream) {
  const int nchunks = (V + kCsrChunk - 1) / kCsrChunk;
  if (B == 0 || nchunks == 0) {  // every row empty
    const cudaError_t e =
        cudaMemsetAsync(crow, 0, (static_cast<size_t>(B) + 1) * sizeof(int64_t), stream);
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "cudaMemsetAsync(crow)");
  }
  const dim3 grid(static_cast<unsigned>(nchunks), static_cast<unsigned>(B));
  csr_count_kernel<T><<<grid, kCsrThreads, 0, stream>>>(static_cast<const T*>(reps), V, thr,
                                                        nchunks, ws.chunk_cnt);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "csr_count_kernel launch");
  e = launch_pdl(csr_scan_kernel, dim3(1), dim3(1024), 0, stream,
                 static_cast<const int*>(ws.chunk_cnt), B, nchunks, ws.chunk_off, crow);
  if (e != cudaSuccess) return cuda_fail(e, "csr_scan_kernel launch");
  if (capacity > 0 && cols != nullptr && vals != nullptr) {
    e = launch_pdl(csr_fill_kernel<T>, grid, dim3(kCsrThreads), 0, stream,
                   static_cast<const T*>(reps), V, thr, nchunks,
                   static_cast<const int*>(ws.chunk_off), capacity, cols, static_cast<T*>(vals));
    if (e != cudaSuccess) return cuda_fail(e, "csr_fill_kernel launch");
  }
  return SPARTON_OK;
}

template <typename T>
int launch_topk_typed(const void* reps, int B, int V, int k, void* vals, int32_t* idx,
                      cudaStream_t stream) {
  if (B == 0 || k == 0) return SPARTON_OK;
  int k_pad = 1;
  while (k_pad < k) k_pad <<= 1;
  const size_t smem_pairs = (256 + 2 * static_cast<size_t>(k_pad)) * sizeof(uint32_t);
  // Enough CTAs for two per SM, each walking at least 16384 entries of its
  // row (shorter spans lose more to the cluster barriers than they gain:
  // [128, 30522] ran 50 µs with one CTA per row, 59 µs with two).
  int P = 1;
  while (P < 8 && static_cast<long long>(B) * P < 2ll * device_sm_count() &&
         V / (2 * P) >= 16384)
    P *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(P), static_cast<unsigned>(B));
  cfg.blockDim = dim3(kTopkThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(P);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Stage the CTA's part of the row in shared memory when it fits (config 2:
  // 61 KB of a 30522-wide bf16 row; config 3: 62 KB per CTA of an 8-CTA cluster).
  auto plan_smem = [&](int p) {
    const size_t part = static_cast<size_t>((((V + p - 1) / p) + 31) & ~31);
    const size_t staged = smem_pairs + part * sizeof(T);
    return staged <= kTopkStageBudget ? staged : 0;
  };
  auto launch = [&](auto kernel, size_t smem) -> cudaError_t {
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(
          kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
    }
    cfg.dynamicSmemBytes = smem;
    if (P > 1 && !cluster_fits(kernel, &cfg, P, smem)) {
      P = 1;
      cfg.gridDim = dim3(1u, static_cast<unsigned>(B));
      attr[0].val.clusterDim.x = 1;
      return cudaErrorNotReady;  // re-plan the shared memory for one CTA per row
    }
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<const T*>(reps), V, k, k_pad,
                              static_cast<T*>(vals), idx);
  };
  cudaError_t e = cudaErrorNotReady;
  for (int attempt = 0; attempt < 2 && e == cudaErrorNotReady; ++attempt) {
    const size_t staged = plan_smem(P);
    e = staged ? launch(topk_kernel<T, true>, staged) : launch(topk_kernel<T, false>, smem_pairs);
  }
  if (e != cudaSuccess) return cuda_fail(e, "topk_kernel launch");
  return SPARTON_OK;
}

}  // namespace

size_t sparse_workspace_bytes(int64_t B, int64_t V) {
  const int64_t nchunks = (V + kCsrChunk - 1) / kCsrChunk;
  const int64_t n = (B > 0 ? B : 1) * (nchunks > 0 ? nchunks : 1);
  return 2 * align256(static_cast<size_t>(n) * sizeof(int));
}

SparseWorkspace sparse_workspace_carve(void* base, int64_t B, int64_t V) {
  const int64_t nchunks = (V + kCsrChunk - 1) / kCsrChunk;
  const int64_t n = (B > 0 ? B : 1) * (nchunks > 0 ? nchunks : 1);
  SparseWorkspace ws;
  ws.chunk_cnt = static_cast<int*>(base);
  ws.chunk_off = reinterpret_cast<int*>(static_cast<char*>(base) +
                                        align256(static_cast<size_t>(n) * sizeof(int)));
  return ws;
}

int launch_reps_csr(int dtype, const void* reps, int B, int V, float threshold, int64_t* crow,
                    int32_t* cols, void* vals, int64_t capacity, const SparseWorkspace& ws,
                    cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_csr_typed<__nv_bfloat16>(reps, B, V, threshold, crow, cols, vals, capacity, ws,
                                             stream);
    case SPARTON_DTYPE_F16:
      return launch_csr_typed<__half>(reps, B, V, threshold, crow, cols, vals, capacity, ws, stream);
    case SPARTON_DTYPE_F32:
      return launch_csr_typed<float>(reps, B, V, threshold, crow, cols, vals, capacity, ws, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

int launch_reps_topk(int dtype, const void* reps, int B, int V, int k, void* vals, int32_t* idx,
                     cudaStream_t stream) {
  switch (dtype) {
    case SPARTON_DTYPE_BF16:
      return launch_topk_typed<__nv_bfloat16>(reps, B, V, k, vals, idx, stream);
    case SPARTON_DTYPE_F16:
      return launch_topk_typed<__half>(reps, B, V, k, vals, idx, stream);
    case SPARTON_DTYPE_F32:
      return launch_topk_typed<float>(reps, B, V, k, vals, idx, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  }
}

}  // namespace sparton
