// bwd.cu — K2..K4: backward of the SPLADE head without atomics.
//
// Upstream (hhkbble/sparton src/sparton/sparton_kernel.py:472-565) runs one
// Triton kernel over (vocab block, batch block) tiles that computes
//   g' = where(score > 0, g * exp(-score), 0)                         (:531)
// and scatters it with fp32 atomics: db[v] += sum_b g' (:536),
// dW[v,:] += sum_b g' * H[b, idx[b,v], :] (:554-557) and, the dominant cost,
// dH[b, idx[b,v], :] += g' * W[v,:] element by element (:559-561).
//
// Here every output element is produced by exactly one warp in a fixed order
// (deterministic, no atomics):
//   K2 sort_*_kernel     stable counting sort of each batch row's vocab ids
//                        with score > 0 by argmax position -> CSR
//                        (offs[b][s]) of (v, g') pairs, v ascending inside
//                        each bucket: chunk counts, a per-row scan, a scatter.
//      dw_list_kernel    tiled transpose of (argmax row, g') to vocab-major
//                        order: the B entries of each vocab id, contiguous.
//   K3 gather_kernel<0>  one warp per (b, s) row: dH[b,s,:] = sum over its
//                        bucket of g' * W[v,:] (W rows gathered, fp32 sums).
//                        Persistent warps claim rows from a counter in the
//                        workspace, position-major, so uneven buckets and the
//                        empty rows past each sequence's end balance out.
//   K4 gather_kernel<1>  one warp per vocab id: dW[v,:] = sum over b of
//                        g' * H[b*S + idx[b,v], :] (neighbouring vocab ids share
//                        H[b] rows in L1); db[v] is the sum of the same g'.
//                        K3 and K4 cut D into column slices, slice-major, when
//                        the gathered matrix (W for K3, H for K4) exceeds the
//                        L2 budget, so the slice being gathered stays in L2.
//      db_kernel         db alone, when dW is not requested.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include <mutex>
#include <type_traits>

#include "dtype.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

// g' of one (b, v) entry; 0 when the head's output is 0 (max logit <= 0).
template <typename T>
__device__ __forceinline__ float scaled_grad(const T* g, const T* reps, size_t o) {
  const float sc = ldg_f32<T>(reps + o);
  return sc > 0.f ? ldg_f32<T>(g + o) * expf(-sc) : 0.f;
}

// acc[i], acc[i+1] += c * f.x, c * f.y as one paired FMA (fma.rn.f32x2 on
// sm_100): the same per-element rounding as two fmaf, half the instructions.
__device__ __forceinline__ void fma2(float c, float2 f, float (&acc)[8], int i) {
  const float2 a = __ffma2_rn(make_float2(c, c), f, make_float2(acc[i], acc[i + 1]));
  acc[i] = a.x;
  acc[i + 1] = a.y;
}

// Eight consecutive elements of a row (16-bit types: one 16-byte load; fp32:
// two) and their FMA into eight fp32 accumulators.
template <typename T>
struct Row8 {  // 16-bit element types
  uint4 r;
  __device__ __forceinline__ void load(const T* p) { r = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ void zero() { r = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void fma_into(float c, float (&acc)[8]) const {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if constexpr (std::is_same<T, __nv_bfloat16>::value)  // bf16 -> fp32: a 16-bit shift
        f = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
      else
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      fma2(c, f, acc, 2 * i);
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
    fma2(c, make_float2(a.x, a.y), acc, 0);
    fma2(c, make_float2(a.z, a.w), acc, 2);
    fma2(c, make_float2(b.x, b.y), acc, 4);
    fma2(c, make_float2(b.z, b.w), acc, 6);
  }
};

// Eight fp32 values stored as eight elements of O (one 16-byte store for 16-bit O);
// kStream: evict-first stores (st.global.cs), which do not displace data the
// kernel still gathers.
template <typename O, bool kStream = false>
__device__ __forceinline__ void store8(O* p, const float (&x)[8]) {
  if constexpr (std::is_same<O, float>::value) {
    const float4 a = make_float4(x[0], x[1], x[2], x[3]), b = make_float4(x[4], x[5], x[6], x[7]);
    if constexpr (kStream) {
      __stcs(reinterpret_cast<float4*>(p), a);
      __stcs(reinterpret_cast<float4*>(p) + 1, b);
    } else {
      reinterpret_cast<float4*>(p)[0] = a;
      reinterpret_cast<float4*>(p)[1] = b;
    }
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<O, __nv_bfloat16>::value) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        memcpy(&w[i], &h, 4);
      } else {
        const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        memcpy(&w[i], &h, 4);
      }
    }
    const uint4 u = make_uint4(w[0], w[1], w[2], w[3]);
    if constexpr (kStream)
      __stcs(reinterpret_cast<uint4*>(p), u);
    else
      *reinterpret_cast<uint4*>(p) = u;
  }
}

// ------------------------------------------------------------------ K2: sort
// Stable counting sort of every batch row's vocab ids with reps > 0 by their
// argmax position, in three short kernels over chunks of `chunk` consecutive
// vocab ids (nw warps x 128 ids; nw from S so that the per-warp tables fit in
// shared memory):
//   sort_count_kernel   one CTA per (chunk, row): cnt[b][c][s] = entries of
//                       chunk c with argmax s (shared-memory histogram);
//   sort_scan_kernel    one CTA per row: cnt[b][c][s] becomes the exclusive
//                       prefix over the chunks before c, and offs[b][s] the
//                       exclusive prefix over positions of the bucket sizes;
//   sort_scatter_kernel one CTA per (chunk, row): per-warp counts per position
//                       (16-bit), their prefix over the warps of the CTA, then
//                       every warp replays its 128 ids in order and writes
//                       (v, g') at offs[b][s] + cnt[b][c][s] + (warp prefix) +
//                       (earlier entries of the warp with that s) + (lower lanes
//                       with that s): v ascending inside every bucket, the same
//                       CSR as a sequential stable sort.
// No cluster barriers or grid-wide waits: each kernel's CTAs are independent.
constexpr int kSortWarpIds = 128;                 // vocab ids per warp in a chunk
constexpr int kSortIters = kSortWarpIds / 32;     // entries per lane
constexpr int kSortSmemBudget = 220 * 1024;       // scatter: nw x S 16-bit + S int32
constexpr int kSortMaxS = kSortSmemBudget / 6;    // nw >= 1

__host__ __device__ inline int sort_warps(int S) {
  int nw = 8;
  while (nw > 1 && (nw * 2 + 4) * S > kSortSmemBudget) nw >>= 1;
  return nw;
}

// Lanes of the warp whose key equals this lane's (keys in [0, 2^nbits), or -1
// for "no entry", which forms its own group): one ballot per key bit. Used
// instead of __match_any_sync, which issues on a slow pipe (the sort kernels
// built on it were bound by that pipe).
__device__ __forceinline__ unsigned same_key_lanes(int key, int nbits) {
  unsigned m = __ballot_sync(0xFFFFFFFFu, key >= 0);
  if (key < 0) m = ~m;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1;
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, bit);
    m &= bit ? bal : ~bal;
  }
  return m;
}

__device__ __forceinline__ int key_bits(int S) { return S > 1 ? 32 - __clz(S - 1) : 0; }

template <typename T>
__device__ __forceinline__ int sort_key(float sc, int s, int S) {
  return (sc > 0.f && s >= 0 && s < S) ? s : -1;
}

// The sort keys of one warp's 128 vocab ids, lane-strided (entry i of this
// lane is vocab id v_begin + 32 i + lane), all loads issued before any use.
template <typename T>
__device__ __forceinline__ void sort_load_keys(const T* reps, const int32_t* idx, size_t row,
                                               int v_begin, int v_end, int S, int lane,
                                               int (&key)[kSortIters], float (&sc)[kSortIters]) {
  int s[kSortIters];
#pragma unroll
  for (int i = 0; i < kSortIters; ++i) {
    const int v = v_begin + 32 * i + lane;
    sc[i] = v < v_end ? ldg_f32<T>(reps + row + v) : 0.f;
    s[i] = v < v_end ? __ldg(idx + row + v) : -1;
  }
#pragma unroll
  for (int i = 0; i < kSortIters; ++i) key[i] = sort_key<T>(sc[i], s[i], S);
}

template <typename T>
__global__ void __launch_bounds__(256)
    sort_count_kernel(const T* __restrict__ reps, const int32_t* __restrict__ idx, int S, int V,
                      int chunk, int n_chunks, int* __restrict__ cnt, unsigned int* status,
                      unsigned int* row_counter) {
  extern __shared__ int hist[];  // [S]
  const int c = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (c == 0 && b == 0 && threadIdx.x == 0) {
    *status = 0u;
    *row_counter = 0u;
  }
  const int c_end = min(V, (c + 1) * chunk);
  const int v_begin = min(c_end, c * chunk + warp * kSortWarpIds);
  const int v_end = min(c_end, v_begin + kSortWarpIds);
  int key[kSortIters];
  float sc[kSortIters];
  sort_load_keys<T>(reps, idx, static_cast<size_t>(b) * V, v_begin, v_end, S, lane, key, sc);
  for (int i = threadIdx.x; i < S; i += blockDim.x) hist[i] = 0;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kSortIters; ++i)
    if (key[i] >= 0) atomicAdd(&hist[key[i]], 1);
  __syncthreads();
  int* out = cnt + (static_cast<size_t>(b) * n_chunks + c) * S;
  for (int i = threadIdx.x; i < S; i += blockDim.x) out[i] = hist[i];
}

// Block-wide exclusive scan of one int per thread (blockDim.x = 1024).
__device__ __forceinline__ int block_exclusive_scan(int x, int* tmp /*[33]*/, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int t = lane < static_cast<int>(blockDim.x >> 5) ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    tmp[lane] = t;  // inclusive per-warp totals
  }
  __syncthreads();
  total = tmp[(blockDim.x >> 5) - 1];
  const int r = incl - x + (warp > 0 ? tmp[warp - 1] : 0);
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(1024)
    sort_scan_kernel(int S, int n_chunks, int* __restrict__ cnt, int* __restrict__ offs) {
  __shared__ int tmp[33];
  pdl_wait();  // the chunk counts
  pdl_trigger();
  const int b = blockIdx.x;
  int* crow = cnt + static_cast<size_t>(b) * n_chunks * S;
  int* orow = offs + static_cast<size_t>(b) * (S + 1);
  int carry = 0;
  for (int s0 = 0; s0 < S; s0 += blockDim.x) {
    const int s = s0 + static_cast<int>(threadIdx.x);
    int run = 0;
    if (s < S) {
      // 16 chunks' counts loaded together, then turned into their prefix
      for (int c0 = 0; c0 < n_chunks; c0 += 16) {
        int x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          x[j] = c0 + j < n_chunks ? __ldcg(crow + static_cast<size_t>(c0 + j) * S + s) : 0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j < n_chunks) crow[static_cast<size_t>(c0 + j) * S + s] = run;
          run += x[j];
        }
      }
    }
    int total = 0;
    const int ex = block_exclusive_scan(run, tmp, total);
    if (s < S) orow[s] = carry + ex;
    carry += total;
  }
  if (threadIdx.x == 0) orow[S] = carry;
}

template <typename T>
__global__ void __launch_bounds__(256)
    sort_scatter_kernel(const T* __restrict__ g, const T* __restrict__ reps,
                        const int32_t* __restrict__ idx, int S, int V, int chunk, int n_chunks,
                        const int* __restrict__ cnt, const int* __restrict__ offs,
                        int2* __restrict__ ent) {
  extern __shared__ int sbase[];  // [S] bucket base of this chunk, then [nw][S] 16-bit counters
  const int c = blockIdx.x, b = blockIdx.y;
  pdl_trigger();
  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t* wcnt = reinterpret_cast<uint16_t*>(sbase + S);
  const size_t row = static_cast<size_t>(b) * V;
  const int c_end = min(V, (c + 1) * chunk);
  const int v_begin = min(c_end, c * chunk + warp * kSortWarpIds);
  const int v_end = min(c_end, v_begin + kSortWarpIds);
  int key[kSortIters];
  float sc[kSortIters], gv[kSortIters];
  sort_load_keys<T>(reps, idx, row, v_begin, v_end, S, lane, key, sc);
#pragma unroll
  for (int i = 0; i < kSortIters; ++i) {
    const int v = v_begin + 32 * i + lane;
    gv[i] = key[i] >= 0 ? ldg_f32<T>(g + row + v) : 0.f;
  }
  const int* obase = offs + static_cast<size_t>(b) * (S + 1);
  const int* cbase = cnt + (static_cast<size_t>(b) * n_chunks + c) * S;
  pdl_wait();  // the scan's offsets (the loads above read only the backward's inputs)
  for (int i = threadIdx.x; i < S; i += blockDim.x) sbase[i] = obase[i] + cbase[i];
  for (int i = threadIdx.x; i < nw * S; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  uint16_t* my = wcnt + warp * S;
  unsigned peers[kSortIters];
  const int nbits = key_bits(S);
#pragma unroll
  for (int i = 0; i < kSortIters; ++i) {
    peers[i] = same_key_lanes(key[i], nbits);
    if (key[i] >= 0 && lane == __ffs(peers[i]) - 1)
      my[key[i]] = static_cast<uint16_t>(my[key[i]] + __popc(peers[i]));
    __syncwarp();
  }
  __syncthreads();
  // per position: exclusive prefix over the warps of this CTA (in place)
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    int run = 0;
    for (int w = 0; w < nw; ++w) {
      const int x = wcnt[w * S + s];
      wcnt[w * S + s] = static_cast<uint16_t>(run);
      run += x;
    }
  }
  __syncthreads();
  int2* erow = ent + row;
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int i = 0; i < kSortIters; ++i) {
    const int k = key[i];
    int slot = 0;
    if (k >= 0) slot = sbase[k] + my[k] + __popc(peers[i] & lt);
    __syncwarp();
    if (k >= 0) {
      const float gp = gv[i] * expf(-sc[i]);
      erow[slot] = make_int2(v_begin + 32 * i + lane, __float_as_int(gp));
      if (lane == __ffs(peers[i]) - 1) my[k] = static_cast<uint16_t>(my[k] + __popc(peers[i]));
    }
    __syncwarp();
  }
}

// Vocab-major list for dW: went[v*B + b] = (b*S + idx[b,v], bits of g'[b,v])
// (g' = 0, with a harmless valid row, when the head's output is 0). Tiles of
// 32 batch rows x 32 vocab ids through shared memory: both sides coalesced.
template <typename T>
__global__ void __launch_bounds__(256)
    dw_list_kernel(const T* __restrict__ g, const T* __restrict__ reps,
                   const int32_t* __restrict__ idx, int B, int S, int V, int2* __restrict__ went,
                   unsigned int* status) {
  __shared__ float cs[32][33];
  __shared__ int rs[32][33];
  const int v0 = blockIdx.x * 32, b0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  pdl_trigger();
  if (status != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *status = 0u;
  for (int i = ty; i < 32; i += 8) {
    const int b = b0 + i, v = v0 + tx;
    float c = 0.f;
    int r = b * S;
    if (b < B && v < V) {
      const size_t o = static_cast<size_t>(b) * V + v;
      const int s = __ldg(idx + o);
      c = scaled_grad<T>(g, reps, o);
      if (s >= 0 && s < S) r += s; else c = 0.f;
    }
    cs[i][tx] = c;
    rs[i][tx] = r;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int v = v0 + i, b = b0 + tx;
    if (v < V && b < B) {
      const size_t o = static_cast<size_t>(v) * B + b;
      went[o] = make_int2(rs[tx][i], __float_as_int(cs[tx][i]));
    }
  }
}

// ----------------------------------------------------------- K3/K4: dH, dW
// out[r, :] = sum over the entry list of row r of coef * src[row, :], 8 warps
// per CTA:
//   kMode 0 (dH): r = b*S + s, entries = bucket (b, s) of the CSR
//                 (src row = v, coef = g'), src = W;
//   kMode 1 (dW): r = v, entries = its B vocab-major entries (src row =
//                 b*S + idx[b,v], coef = g'), src = H; out_sum[r] = db[v].
// Entries are fetched 32 at a time with one coalesced load and broadcast by
// shuffle, and the loads of several entries are issued before their FMAs.
//
// Full rows (one warp per output row): lane l owns columns d0 + c*256 + 8l ..
// +7 of NC*256-column passes; 4 entries, NC 16-byte loads each, in flight per
// lane. For dW, neighbouring vocab ids walk the batch rows in step, so the rows
// of H[b] they share are served from L1.
//
// Column slices, for a gathered working set larger than the L2 budget (all of
// W for dH, whose rows are gathered in random order; for dW the rows of the
// ~16 batch rows that the warps in flight walk together): D is cut into
// slices of 256, 128 or 64 columns and the work items (slice, row) are
// slice-major, so the warps in flight all read one slice of src, which stays
// in L2. A warp takes one (slice, row) item split into G = 256 / slice lane
// groups; each lane loads 8 columns (16 bytes) and group g takes the entries
// j with j % G == g, so every load stays 16 bytes wide; the G partial sums are
// added in a fixed butterfly order at the end (deterministic). The next entry
// batch is prefetched while the current one is gathered.
constexpr int kGWarps = 8;
constexpr int kGUnroll = 4;
// Sliced gathers: the entry lists are read once per slice and the outputs
// written once, so both go through L2 evict-first (ld/st .cs) and leave it to
// the slice of src, which is gathered many times.
constexpr bool kSliceStreamStores = true;
template <typename X>
__device__ __forceinline__ X ld_list(const X* p) {
  return __ldcs(p);
}
// Bytes of gathered data that are expected to stay resident in the 126 MB L2
// next to the other traffic of the kernel, and the batch rows that the dW
// warps in flight span.
constexpr long long kGatherL2Budget = 48ll << 20;
constexpr int kDwRowsInFlight = 16;

// Row bounds of an output row: r and its entries [e0, e1).
template <int kMode>
__device__ __forceinline__ void entry_range(int q, int B, int S, int V, const int* __restrict__ offs,
                                            int& r, int& e0, int& e1) {
  if (kMode == 0) {
    const int s = q / B, b = q - (q / B) * B;
    r = b * S + s;
    const int* o = offs + static_cast<size_t>(b) * (S + 1);
    e0 = b * V + __ldg(o + s);
    e1 = b * V + __ldg(o + s + 1);
  } else {
    r = q;
    e0 = r * B;
    e1 = e0 + B;
  }
}

template <typename T, typename O, int NC, int kMode>
__device__ __forceinline__ void gather_row_full(const T* __restrict__ src, int B, int S, int D,
                                                int V, const int* __restrict__ offs,
                                                const int2* __restrict__ ent, int q,
                                                O* __restrict__ out, O* __restrict__ out_sum,
                                                int lane) {
  int r, e0, e1;
  entry_range<kMode>(q, B, S, V, offs, r, e0, e1);
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
        const int2 e = __ldg(ent + eb + lane);
        my_row = e.x;
        my_coef = __int_as_float(e.y);
      }
      if (kMode == 1 && d0 == 0) csum += my_coef;
      for (int j = 0; j < n; j += kGUnroll) {
        int rr[kGUnroll];
        float cc[kGUnroll];
#pragma unroll
        for (int u = 0; u < kGUnroll; ++u) {
          rr[u] = __shfl_sync(0xFFFFFFFFu, my_row, j + u);
          cc[u] = __shfl_sync(0xFFFFFFFFu, my_coef, j + u);
        }
        Row8<T> x[kGUnroll][NC];
#pragma unroll
        for (int u = 0; u < kGUnroll; ++u)
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int d = d0 + c * 256 + lane * 8;
            if (cc[u] != 0.f && d < D)
              x[u][c].load(src + static_cast<size_t>(rr[u]) * D + d);
            else
              x[u][c].zero();
          }
#pragma unroll
        for (int u = 0; u < kGUnroll; ++u)
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
    if (lane == 0) out_sum[r] = from_f32<O>(csum);
  }
}

// Columns [d_lo, d_lo + width) of one output row, width <= 256 / G.
template <typename T, typename O, int G, int U, int kMode>
__device__ __forceinline__ void gather_row_slice(const T* __restrict__ src, int B, int S, int D,
                                                 int V, const int* __restrict__ offs,
                                                 const int2* __restrict__ ent, int q,
                                                 int d_lo, int width, O* __restrict__ out,
                                                 O* __restrict__ out_sum, int lane) {
  static_assert(G == 1 || G == 2 || G == 4, "lane groups");
  static_assert(U * G <= 32 && 32 % (U * G) == 0, "entries per round must divide 32");
  constexpr int kLanes = 32 / G;
  const int grp = lane / kLanes, sub = lane - grp * kLanes;
  int r, e0, e1;
  entry_range<kMode>(q, B, S, V, offs, r, e0, e1);
  const int d = sub * 8;
  const bool active = d < width;
  const T* scol = src + d_lo + d;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float csum = 0.f;
  int nx_row = 0;
  float nx_coef = 0.f;
  if (lane < e1 - e0) {
    const int2 e = ld_list(ent + e0 + lane);
    nx_row = e.x;
    nx_coef = __int_as_float(e.y);
  }
  for (int eb = e0; eb < e1; eb += 32) {
    const int n = min(32, e1 - eb);
    const int my_row = nx_row;
    const float my_coef = nx_coef;  // 0 on the lanes past the batch's end
    nx_row = 0;
    nx_coef = 0.f;
    if (lane < e1 - eb - 32) {  // the next batch, while this one is gathered
      const int2 e = ld_list(ent + eb + 32 + lane);
      nx_row = e.x;
      nx_coef = __int_as_float(e.y);
    }
    if (kMode == 1) csum += my_coef;
    for (int j = 0; j < n; j += U * G) {
      int rr[U];
      float cc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {  // entry j + u*G + grp (< 32) for this group
        rr[u] = __shfl_sync(0xFFFFFFFFu, my_row, j + u * G + grp);
        cc[u] = __shfl_sync(0xFFFFFFFFu, my_coef, j + u * G + grp);
      }
      Row8<T> x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (cc[u] != 0.f && active)
          x[u].load(scol + static_cast<size_t>(rr[u]) * D);
        else
          x[u].zero();
      }
#pragma unroll
      for (int u = 0; u < U; ++u) x[u].fma_into(cc[u], acc);
    }
  }
#pragma unroll
  for (int o = kLanes; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xFFFFFFFFu, acc[i], o);
  if (grp == 0 && active) store8<O, kSliceStreamStores>(out + static_cast<size_t>(r) * D + d_lo + d, acc);
  if (kMode == 1 && out_sum != nullptr && d_lo == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) csum += __shfl_xor_sync(0xFFFFFFFFu, csum, o);
    if (lane == 0) out_sum[r] = from_f32<O>(csum);
  }
}

// Register cap for 4 CTAs (32 warps) per SM: the gathers are bound by loads
// in flight, and 4 resident CTAs measured 28-30% faster than the 3 that the
// uncapped register count allows. G == 0: full rows in NC passes; G > 0:
// column slices of slice_w = 256 / G columns.
template <typename T, typename O, int NC, int G, int U, int kMode>
__global__ void __launch_bounds__(kGWarps * 32, 4)
    gather_kernel(const T* __restrict__ src, int B, int S, int D, int V, const int* __restrict__ offs,
                  const int2* __restrict__ ent, int n_rows,
                  int slice_w, int n_slices, O* __restrict__ out, O* __restrict__ out_sum,
                  unsigned int* row_counter) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // the sort's CSR (dH) or the vocab-major list (dW)
  if (kMode == 0) {
    // dH: persistent warps claim items q = 0, 1, ... from the workspace counter
    // (the next claim is issued before the current one is gathered). Items are
    // slice-major, then position-major (row q % n_rows -> s = row / B,
    // b = row % B): the heavy rows come first and the empty rows past each
    // sequence's end last.
    const int n_items = n_rows * n_slices;
    int q = 0;
    if (lane == 0) q = static_cast<int>(atomicAdd(row_counter, 1u));
    q = __shfl_sync(0xFFFFFFFFu, q, 0);
    while (q < n_items) {
      int qn = 0;
      if (lane == 0) qn = static_cast<int>(atomicAdd(row_counter, 1u));
      if constexpr (G == 0) {
        gather_row_full<T, O, NC, kMode>(src, B, S, D, V, offs, ent, q, out,
                                         out_sum, lane);
      } else {
        const int sl = q / n_rows;
        const int d_lo = sl * slice_w;
        gather_row_slice<T, O, G, U, kMode>(src, B, S, D, V, offs, ent,
                                            q - sl * n_rows, d_lo, min(slice_w, D - d_lo), out,
                                            out_sum, lane);
      }
      q = __shfl_sync(0xFFFFFFFFu, qn, 0);
    }
  } else if constexpr (G == 0) {
    // dW: one row per warp.
    const int r = blockIdx.x * kGWarps + warp;
    if (r < n_rows)
      gather_row_full<T, O, NC, kMode>(src, B, S, D, V, offs, ent, r, out, out_sum,
                                       lane);
  } else {
    // dW: one (slice, row) per warp; blocks are slice-major (the block scheduler
    // dispatches them in order).
    const int per_slice = (n_rows + kGWarps - 1) / kGWarps;
    const int sl = blockIdx.x / per_slice;
    const int r = (blockIdx.x - sl * per_slice) * kGWarps + warp;
    const int d_lo = sl * slice_w;
    if (r < n_rows)
      gather_row_slice<T, O, G, U, kMode>(src, B, S, D, V, offs, ent, r, d_lo,
                                          min(slice_w, D - d_lo), out, out_sum, lane);
  }
}

template <typename T, typename O>
__global__ void __launch_bounds__(256) db_kernel(const T* __restrict__ g, const T* __restrict__ reps,
                                                 int B, int V, O* __restrict__ db) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  float acc = 0.f;
  for (int b = 0; b < B; ++b) acc += scaled_grad<T>(g, reps, static_cast<size_t>(b) * V + v);
  db[v] = from_f32<O>(acc);
}

// ----------------------------------------------------------------------- host
template <typename K>
int set_smem(K kernel, int bytes, const char* what) {
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, what);
}

// The sort's three launches (K2 above). Shared memory: S ints of histogram
// (count); S ints of bucket bases and nw x S 16-bit counters (scatter).
template <typename T>
int launch_sort(const void* grad_reps, const void* reps, const int32_t* idx, int B, int S, int V,
                const BwdWorkspace& ws, cudaStream_t stream) {
  if (S > kSortMaxS)
    return fail(SPARTON_ERR_UNSUPPORTED, "backward supports S <= %d (got %d)", kSortMaxS, S);
  const int nw = sort_warps(S);
  const int chunk = nw * kSortWarpIds;
  const int n_chunks = (V + chunk - 1) / chunk;
  const size_t smem_count = static_cast<size_t>(S) * sizeof(int);
  const size_t smem_scatter = static_cast<size_t>(S) * (sizeof(int) + nw * sizeof(uint16_t));
  int st = SPARTON_OK;
  if (smem_count > 48 * 1024)
    st = set_smem(sort_count_kernel<T>, static_cast<int>(smem_count),
                  "cudaFuncSetAttribute(sort_count_kernel)");
  if (st == SPARTON_OK && smem_scatter > 48 * 1024)
    st = set_smem(sort_scatter_kernel<T>, static_cast<int>(smem_scatter),
                  "cudaFuncSetAttribute(sort_scatter_kernel)");
  if (st != SPARTON_OK) return st;
  const dim3 grid(static_cast<unsigned>(n_chunks), static_cast<unsigned>(B));
  sort_count_kernel<T><<<grid, static_cast<unsigned>(nw * 32), smem_count, stream>>>(static_cast<const T*>(reps), idx, S, V,
                                                          chunk, n_chunks, ws.sort_cnt,
                                                          ws.status, ws.row_counter);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sort_count_kernel launch");
  const unsigned scan_threads = static_cast<unsigned>(S >= 1024 ? 1024 : (S + 31) / 32 * 32);
  e = launch_pdl(sort_scan_kernel, dim3(static_cast<unsigned>(B)), dim3(scan_threads), 0, stream,
                 S, n_chunks, ws.sort_cnt, ws.offs);
  if (e != cudaSuccess) return cuda_fail(e, "sort_scan_kernel launch");
  e = launch_pdl(sort_scatter_kernel<T>, grid, dim3(static_cast<unsigned>(nw * 32)), smem_scatter,
                 stream, static_cast<const T*>(grad_reps), static_cast<const T*>(reps), idx, S, V,
                 chunk, n_chunks, static_cast<const int*>(ws.sort_cnt),
                 static_cast<const int*>(ws.offs), ws.ent);
  if (e != cudaSuccess) return cuda_fail(e, "sort_scatter_kernel launch");
  return SPARTON_OK;
}

// Launches one gather_kernel instantiation: for dH a persistent grid of
// resident CTAs per SM (occupancy API, cached per device) x SMs, capped by the
// work; for dW one CTA per kGWarps rows of each slice.
template <typename T, typename O, int NC, int G, int U, int kMode>
int launch_gather_nc(const T* src, int B, int S, int D, int V, const int* offs, const int2* ent, int n_rows, O* out, O* out_sum,
                     unsigned int* row_counter, cudaStream_t stream) {
  static std::mutex mu;
  static int per_sm[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const int block = kGWarps * 32;
  int bps = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    bps = dev < 64 ? per_sm[dev] : 0;
    if (bps == 0) {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, gather_kernel<T, O, NC, G, U, kMode>,
                                                        block, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if (bps < 1) bps = 1;
      if (dev < 64) per_sm[dev] = bps;
    }
  }
  const int slice_w = G == 0 ? D : 256 / G;
  const int n_slices = (D + slice_w - 1) / slice_w;
  // dH rows carry very different amounts of work (bucket sizes, empty rows past
  // each sequence's end): persistent CTAs that claim rows dynamically.
  // dW rows all carry B entries: one CTA per kGWarps rows, balanced by the
  // hardware block scheduler.
  const long long need = (static_cast<long long>(n_rows) + kGWarps - 1) / kGWarps * n_slices;
  const long long cap = kMode == 0 ? static_cast<long long>(bps) * device_sm_count() : need;
  const unsigned grid = static_cast<unsigned>(need < cap ? (need > 0 ? need : 1) : cap);
  e = launch_pdl(gather_kernel<T, O, NC, G, U, kMode>, dim3(grid), dim3(block), 0, stream, src, B,
                 S, D, V, offs, ent, n_rows, slice_w, n_slices, out, out_sum, row_counter);
  if (e != cudaSuccess) return cuda_fail(e, "gather_kernel launch");
  return SPARTON_OK;
}

// Full rows when the gathered working set (col_bytes per column of D) fits the
// L2 budget, else the widest slice of 256, 128 or 64 columns whose share does
// (64 at the least).
template <typename T, typename O, int kMode>
int launch_gather(const T* src, long long col_bytes, int B, int S, int D, int V, const int* offs,
                  const int2* ent, int n_rows, O* out, O* out_sum,
                  unsigned int* row_counter, cudaStream_t stream) {
  if (col_bytes * D > kGatherL2Budget && D > 64) {
    if (D > 256 && col_bytes * 256 <= kGatherL2Budget)
      return launch_gather_nc<T, O, 1, 1, 4, kMode>(src, B, S, D, V, offs, ent,
                                                    n_rows, out, out_sum, row_counter, stream);
    if (D > 128 && col_bytes * 128 <= kGatherL2Budget)
      return launch_gather_nc<T, O, 1, 2, 4, kMode>(src, B, S, D, V, offs, ent,
                                                    n_rows, out, out_sum, row_counter, stream);
    return launch_gather_nc<T, O, 1, 4, 8, kMode>(src, B, S, D, V, offs, ent, n_rows,
                                                  out, out_sum, row_counter, stream);
  }
  if (D <= 256)
    return launch_gather_nc<T, O, 1, 0, 0, kMode>(src, B, S, D, V, offs, ent, n_rows,
                                                  out, out_sum, row_counter, stream);
  if (D <= 512)
    return launch_gather_nc<T, O, 2, 0, 0, kMode>(src, B, S, D, V, offs, ent, n_rows,
                                                  out, out_sum, row_counter, stream);
  if (D <= 768)
    return launch_gather_nc<T, O, 3, 0, 0, kMode>(src, B, S, D, V, offs, ent, n_rows,
                                                  out, out_sum, row_counter, stream);
  return launch_gather_nc<T, O, 4, 0, 0, kMode>(src, B, S, D, V, offs, ent, n_rows,
                                                out, out_sum, row_counter, stream);
}

template <typename T, typename O>
int launch_dh(const void* weight, int B, int S, int D, int V, void* d_hidden,
              const BwdWorkspace& ws, cudaStream_t stream) {
  // dH gathers rows of W in random order: its working set is all of W.
  return launch_gather<T, O, 0>(static_cast<const T*>(weight),
                                static_cast<long long>(V) * sizeof(T), B, S, D, V, ws.offs, ws.ent, B * S, static_cast<O*>(d_hidden), nullptr,
                                ws.row_counter, stream);
}

template <typename T, typename O>
int launch_dw(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
              int B, int S, int D, int V, void* d_weight, void* d_bias, const BwdWorkspace& ws,
              cudaStream_t stream) {
  const dim3 lgrid(static_cast<unsigned>((V + 31) / 32), static_cast<unsigned>((B + 31) / 32));
  dw_list_kernel<T><<<lgrid, 256, 0, stream>>>(static_cast<const T*>(grad_reps),
                                               static_cast<const T*>(reps), idx, B, S, V, ws.went,
                                               ws.status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dw_list_kernel launch");
  // dW warps walk the batch rows in step: the working set is the H[b] of the
  // ~kDwRowsInFlight batch rows they span.
  return launch_gather<T, O, 1>(static_cast<const T*>(hidden),
                                static_cast<long long>(kDwRowsInFlight) * S * sizeof(T), B, S, D, V,
                                nullptr, ws.went, V, static_cast<O*>(d_weight), static_cast<O*>(d_bias),
                                nullptr, stream);
}

template <typename T, typename OH, typename OP>
int launch_all(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
               const void* weight, int B, int S, int D, int V, void* d_hidden, void* d_weight,
               void* d_bias, const BwdWorkspace& ws, cudaStream_t stream) {
  if (d_hidden != nullptr) {
    int st = launch_sort<T>(grad_reps, reps, idx, B, S, V, ws, stream);
    if (st == SPARTON_OK) st = launch_dh<T, OH>(weight, B, S, D, V, d_hidden, ws, stream);
    if (st != SPARTON_OK) return st;
  }
  if (d_weight != nullptr) {
    const int st =
        launch_dw<T, OP>(grad_reps, reps, idx, hidden, B, S, D, V, d_weight, d_bias, ws, stream);
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
