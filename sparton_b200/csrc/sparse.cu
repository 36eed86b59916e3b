// sparse.cu — sparse forms of the head's output reps [B, V] for indexing:
// the per-row CSR of the entries above a threshold, and the per-row top-k.
//
// Upstream (hhkbble/sparton training/model.py:141-144) `encode` returns the
// dense reps under no_grad, and training/train.py:205-210 logs the fraction
// of entries > 0; an inverted index stores each row's nonzero (vocab id,
// weight) pairs, or its k heaviest.
//
// CSR, one kernel:
//   csr_kernel  one CTA per chunk of kCsrChunk elements of the flattened reps:
//               counts the entries >
//               threshold, finds the entries of all earlier chunks by a
//               decoupled look-back over the chunks' published counts and
//               prefixes, and writes (column, value) in order; crow[b] (row
//               starts) and crow[B] (= nnz). Entries at or past `capacity` are
//               not written (the caller sees nnz in crow[B]).
// Top-k: rows whose keys fit in shared memory (and k <= 512) take
//   topk_row_kernel, one CTA per row (see there); the others a cluster of up
//   to 8 CTAs per row (enough CTAs for two per SM):
//   radix select on order-preserving unsigned keys (12 bits, then 8 bits a
//   pass, the last the rest: 2 passes for 16-bit types, 4 for fp32), the CTAs'
//   histograms summed through
//   distributed shared memory, finds the k-th largest key K and how many of
//   its equals to take. The first pass reads the row with 16-byte loads; when
//   few entries share or beat the selected top digit, a second read copies
//   them in vocab order into a shared-memory candidate list and the later
//   passes walk only that list. One ordered pass collects the entries above K
//   and the first such equals in vocab order into CTA 0; a bitonic sort in its
//   shared memory orders the k by (value descending, vocab id ascending).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cooperative_groups.h>
#include <atomic>
#include <type_traits>

#include "dtype.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

constexpr int kCsrChunk = 8192;  // elements of the flattened reps per CTA
constexpr int kCsrThreads = 256;
constexpr int kTopkThreads = 512;
constexpr int kTileU = 8;  // entries per lane per step of a row walk
constexpr int kTopkCand = 6144;  // candidate list entries per CTA (48 KB of key + id)
constexpr int kTopkFirstBits = 12;  // digit width of the first radix pass (4096 bins)
constexpr int kTopkBins = 1 << kTopkFirstBits;

// Order-preserving unsigned key of an element (larger value -> larger key;
// NaN above +inf, as torch.topk orders it) and its bit width.
template <typename T>
struct Key;
// `conv` maps the raw bits, `of` loads them through the read-only path.
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
};
template <>
struct Key<__half> : Key16<__half> {};
template <>
struct Key<__nv_bfloat16> : Key16<__nv_bfloat16> {};

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
// Look-back words of the chunks: [tag:30][status:2][value:32]. The tag is the
// call's (the host numbers the calls), so words left by earlier calls never
// match; status 1 = the chunk's own count, 2 = the inclusive prefix through
// the chunk.
constexpr unsigned long long kLbCount = 1ull << 32;
constexpr unsigned long long kLbPrefix = 2ull << 32;
constexpr unsigned long long kLbValue = 0xFFFFFFFFull;
__device__ __forceinline__ unsigned long long lb_word(uint32_t tag, unsigned long long status,
                                                      unsigned long long value) {
  return (static_cast<unsigned long long>(tag) << 34) | status | (value & kLbValue);
}

// The words carry their data (count or prefix) themselves, so relaxed
// single-copy-atomic 64-bit accesses at GPU scope are enough: no fence orders
// anything else.
__device__ __forceinline__ void lb_publish(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long lb_read(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One pass (decoupled look-back) over the flattened reps [B * V], whose row-
// major order is the CSR order: CTA c takes the chunk of kCsrChunk elements at
// c * kCsrChunk. Thread t holds kVecs consecutive vectors of kPer elements
// (16-byte loads when reps is 16-byte aligned, else kPer = 1) and counts its
// entries above the threshold; a block prefix over the threads gives each
// thread's offset inside the chunk, and the chunk publishes its count. Then
// every thread reads the word of one earlier chunk (kCsrThreads of them per
// round, nearest first), the block finds the nearest inclusive prefix among
// them and adds it and the counts after it, and walks further back only if
// none was there. The CTA publishes its own inclusive prefix; each thread puts
// its entries (column = flattened index - row * V) in shared memory at its
// offset, and the CTA copies them to prefix + offset with consecutive threads
// writing consecutive entries: columns ascending inside each row. crow[b] is written by the
// thread whose elements include b * V, crow[B] by the last chunk. Entries at
// or past `capacity` are not written (the caller sees nnz in crow[B]).
// A chunk waits only for chunks of lower index, which the hardware dispatches
// first; each wait is bounded anyway (a timeout records
// SPARTON_DEV_TIMEOUT_SCAN in the workspace header).
template <typename T, int kPer>
__global__ void __launch_bounds__(kCsrThreads)
    csr_kernel(const T* __restrict__ reps, int B, int V, float thr, int nchunks, uint32_t tag,
               unsigned int* __restrict__ header, unsigned long long* __restrict__ flags,
               int64_t capacity, int64_t* __restrict__ crow, int32_t* __restrict__ cols,
               T* __restrict__ vals) {
  constexpr int kWarps = kCsrThreads / 32;
  constexpr int kSpan = kCsrChunk / kCsrThreads;  // elements of a thread
  constexpr int kVecs = kSpan / kPer;
  __shared__ int tmp[32];
  __shared__ int s_stop, s_fail;
  __shared__ long long s_part[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_fail = 0;
  const int id = static_cast<int>(blockIdx.x);
  const long long n = static_cast<long long>(B) * V;
  const long long e0 = static_cast<long long>(id) * kCsrChunk + static_cast<long long>(threadIdx.x) * kSpan;
  // the thread's elements e0 .. e0 + nv - 1, kept as loaded (16-byte words)
  const int nv = static_cast<int>(e0 < n ? (n - e0 < kSpan ? n - e0 : kSpan) : 0);
  constexpr int kWords = kSpan * static_cast<int>(sizeof(T)) / 4;
  constexpr int kPerWord = 4 / static_cast<int>(sizeof(T));
  static_assert(kSpan % kPerWord == 0, "whole 32-bit words per thread");
  uint32_t w[kWords];
  // word q of the thread from element loads (the tail of reps, or unaligned reps)
  auto word_at = [&](int q) -> uint32_t {
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < kPerWord; ++i) {
      const int k = q * kPerWord + i;
      const T t = k < nv ? reps[e0 + k] : T{};
      uint32_t bits;
      if constexpr (sizeof(T) == 4)
        bits = __float_as_uint(to_f32<T>(t));
      else
        bits = *reinterpret_cast<const uint16_t*>(&t);
      r |= bits << (8 * sizeof(T) * i);
    }
    return r;
  };
  if constexpr (kPer > 1) {
    constexpr int kWordsPerVec = kPer * static_cast<int>(sizeof(T)) / 4;
#pragma unroll
    for (int u = 0; u < kVecs; ++u) {
      if ((u + 1) * kPer <= nv) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(reps + e0) + u);
        w[4 * u] = q.x, w[4 * u + 1] = q.y, w[4 * u + 2] = q.z, w[4 * u + 3] = q.w;
      } else {
#pragma unroll
        for (int i = 0; i < kWordsPerVec; ++i) w[u * kWordsPerVec + i] = word_at(u * kWordsPerVec + i);
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < kWords; ++q) w[q] = word_at(q);
  }
  auto elem = [&](int i) -> T { return reinterpret_cast<const T*>(w)[i]; };
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < kSpan; ++i) cnt += (i < nv && to_f32<T>(elem(i)) > thr) ? 1 : 0;
  int total;
  const int before = block_excl_scan(cnt, tmp, total);
  if (threadIdx.x == 0)
    lb_publish(flags + id, lb_word(tag, id == 0 ? kLbPrefix : kLbCount,
                                   static_cast<unsigned long long>(total)));
  long long excl = 0;
  const uint64_t t0 = global_timer_ns();
  const unsigned long long want = static_cast<unsigned long long>(tag) << 34;
  constexpr unsigned long long kTagMask = ~((1ull << 34) - 1);
  for (int pos = id - 1; pos >= 0; pos -= kCsrThreads) {
    const int j = pos - static_cast<int>(threadIdx.x);  // thread 0: the nearest earlier chunk
    unsigned long long f = 0;
    if (j >= 0) {
      f = lb_read(flags + j);
      while ((f & kTagMask) != want) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
          s_fail = 1;
          break;
        }
        f = lb_read(flags + j);
      }
    }
    if (threadIdx.x == 0) s_stop = kCsrThreads;
    __syncthreads();
    if (j >= 0 && ((f >> 32) & 3ull) == 2) atomicMin(&s_stop, static_cast<int>(threadIdx.x));
    __syncthreads();
    const int stop = s_stop;  // the nearest inclusive prefix (kCsrThreads: none)
    long long add = (j >= 0 && static_cast<int>(threadIdx.x) <= stop)
                        ? static_cast<long long>(f & kLbValue) : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) add += __shfl_xor_sync(0xFFFFFFFFu, add, o);
    if (lane == 0) s_part[warp] = add;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) excl += s_part[w];
    const bool done = stop < kCsrThreads || s_fail;
    __syncthreads();  // s_part and s_stop are reused
    if (done) break;
  }
  if (threadIdx.x == 0) {
    if (s_fail)
      atomicCAS(header, 0u, SPARTON_DEV_TIMEOUT_SCAN);
    else if (id > 0)
      lb_publish(flags + id, lb_word(tag, kLbPrefix, static_cast<unsigned long long>(excl + total)));
    if (id == nchunks - 1) crow[B] = excl + total;
  }
  // The chunk's entries go to shared memory first (thread order = column
  // order) and then out to [excl, excl + total) by consecutive threads.
  extern __shared__ __align__(16) unsigned char csr_smem[];
  int32_t* s_cols = reinterpret_cast<int32_t*>(csr_smem);             // [kCsrChunk]
  T* s_vals = reinterpret_cast<T*>(s_cols + kCsrChunk);               // [kCsrChunk]
  if (nv > 0) {
    // row and column of the first element; a row starts where the column wraps
    int row = static_cast<int>(e0 / V);
    int col = static_cast<int>(e0 - static_cast<long long>(row) * V);
    int p = before;
    if (col == 0) crow[row] = excl + p;
#pragma unroll
    for (int i = 0; i < kSpan; ++i) {
      if (i < nv) {
        if (col == V) {
          col = 0;
          crow[++row] = excl + p;
        }
        const T v = elem(i);
        if (to_f32<T>(v) > thr) {
          s_cols[p] = col;
          s_vals[p] = v;
          ++p;
        }
        ++col;
      }
    }
  }
  if (capacity <= excl) return;  // (uniform) nothing of this chunk fits
  __syncthreads();
  for (int q = threadIdx.x; q < total; q += kCsrThreads) {
    const long long at = excl + q;
    if (at < capacity) {
      cols[at] = s_cols[q];
      vals[at] = s_vals[q];
    }
  }
}

// ------------------------------------------------------------------ top-k
// A thread-block cluster of P CTAs per row (P = 1 .. 8); CTA c walks the vocab
// range [c*part, (c+1)*part). Shared memory: hist[4096], k_pad (key, id) pairs
// (used in CTA 0), then a candidate list of up to kTopkCand (key, id) pairs.
//
// Pass 1 reads the CTA's part with 16-byte loads (kPer elements each; kPer = 1
// when reps is not 16-byte aligned) and histograms the top 12 key bits (an
// eighth of an octave for 16-bit types; the later passes take 8 bits, the last
// the rest); lanes
// count the key of 0.0 in a register (most entries of a SPLADE row) and add it
// once. When the cluster's entries at or above the selected digit number at
// most kTopkCand, a second read of the part (from L2) copies them, in vocab
// order, into the CTA's candidate list, and the remaining radix passes and the
// collection walk that list; otherwise they walk the row.
template <typename T, int kPer>
__device__ __forceinline__ void load_keys(const T* base, int vi, uint32_t (&key)[kPer]) {
  if constexpr (kPer == 1) {
    key[0] = Key<T>::of(base + vi);
  } else {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(base) + vi);
    const uint32_t q[4] = {w.x, w.y, w.z, w.w};
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int e = 0; e < 4; ++e) key[e] = Key<T>::conv(q[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        key[2 * e] = Key<T>::conv(q[e] & 0xFFFFu);
        key[2 * e + 1] = Key<T>::conv(q[e] >> 16);
      }
    }
  }
}

// Exclusive prefix of x over the warp's lanes, and the warp total.
__device__ __forceinline__ int warp_excl_scan(int x, int lane, int& total) {
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  return incl - x;
}

template <typename T, int kPer>
__global__ void __launch_bounds__(kTopkThreads)
    topk_kernel(const T* __restrict__ reps, int V, int k, int k_pad, T* __restrict__ out_vals,
                int32_t* __restrict__ out_idx) {
  extern __shared__ uint32_t smem[];
  uint32_t* hist = smem;                                          // [kTopkBins]
  uint32_t* skey = smem + kTopkBins;                              // [k_pad]
  int32_t* sid = reinterpret_cast<int32_t*>(skey + k_pad);        // [k_pad]
  uint32_t* ckey = reinterpret_cast<uint32_t*>(sid + k_pad);      // [kTopkCand]
  int32_t* cid = reinterpret_cast<int32_t*>(ckey + kTopkCand);    // [kTopkCand]
  __shared__ int tmp[32];
  __shared__ uint32_t s_prefix, s_remaining, s_eq_before, s_gt, s_cge;
  namespace cg = cooperative_groups;
  const cg::cluster_group cluster = cg::this_cluster();
  const int P = static_cast<int>(cluster.num_blocks());
  const int c = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.y;
  const T* row = reps + static_cast<size_t>(b) * V;
  const int part = (((V + P - 1) / P) + 31) & ~31;
  const int v_lo = min(V, c * part), v_hi = min(V, v_lo + part);
  constexpr int kBits = Key<T>::kBits;
  constexpr uint32_t kZeroKey = 1u << (kBits - 1);  // key of +0.0
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // One CTA per row: a block barrier and this CTA's own shared memory.
  auto csync = [&]() {
    if (P > 1)
      cluster.sync();
    else
      __syncthreads();
  };
  // The digit whose bucket holds the remaining-th largest key of the prefix
  // group, over nbins digits of width `shift`..: thread t owns the `per`
  // digits nbins-1 - t*per - [0, per) (descending); every CTA sums the
  // cluster's histograms itself and picks the same digit.
  auto select_digit = [&](uint32_t prefix, uint32_t remaining, int shift, int nbins) {
    const int per = nbins > kTopkThreads ? nbins / kTopkThreads : 1;
    const int t = static_cast<int>(threadIdx.x);
    uint32_t cnt[kTopkBins / kTopkThreads], bef[kTopkBins / kTopkThreads];
    uint32_t own = 0;
#pragma unroll
    for (int q = 0; q < kTopkBins / kTopkThreads; ++q) {
      const int dgt = nbins - 1 - (t * per + q);
      cnt[q] = bef[q] = 0;
      if (q < per && dgt >= 0) {
        if (P == 1) {
          cnt[q] = hist[dgt];
        } else {
          for (int r = 0; r < P; ++r) {
            const uint32_t x = *cluster.map_shared_rank(hist + dgt, r);
            cnt[q] += x;
            bef[q] += r < c ? x : 0u;
          }
        }
        own += cnt[q];
      }
    }
    int total;
    uint32_t above = static_cast<uint32_t>(block_excl_scan(static_cast<int>(own), tmp, total));
    if (above < remaining && above + own >= remaining) {
#pragma unroll
      for (int q = 0; q < kTopkBins / kTopkThreads; ++q) {
        if (q < per && above + cnt[q] >= remaining) {
          s_prefix = prefix | (static_cast<uint32_t>(nbins - 1 - (t * per + q)) << shift);
          s_remaining = remaining - above;
          s_eq_before = bef[q];       // after the last pass: equals of K in the CTAs before this one
          s_cge = above + cnt[q];     // entries of the group at or above the digit
          break;
        }
        above += cnt[q];
      }
    }
  };

  // ---- pass 1: the top kTopkFirstBits bits, 16-byte loads
  const size_t g0 = static_cast<size_t>(b) * V + v_lo;
  const size_t a0 = g0 / kPer * kPer;
  const int lo = static_cast<int>(g0 - a0), hi = lo + (v_hi - v_lo);  // element offsets from a0
  const int nvec = v_hi > v_lo ? (hi + kPer - 1) / kPer : 0;
  const T* abase = reps + a0;
  constexpr int kVU = kPer == 1 ? 8 : 2;  // loads per lane per step
  constexpr int kVStep = kTopkThreads * kVU;
  const int shift0 = kBits - kTopkFirstBits;
  for (int i = threadIdx.x; i < kTopkBins; i += kTopkThreads) hist[i] = 0;
  if (threadIdx.x == 0) s_gt = 0;
  __syncthreads();
  {
    uint32_t zc = 0;
    for (int base = warp * 32 * kVU; base < nvec; base += kVStep) {
      uint32_t key[kVU][kPer];
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int vi = base + u * 32 + lane;
        if (vi < nvec) load_keys<T, kPer>(abase, vi, key[u]);
      }
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int vi = base + u * 32 + lane;
        const int off0 = vi * kPer;
        if (vi < nvec && off0 >= lo && off0 + kPer <= hi) {  // a whole vector of the part
#pragma unroll
          for (int e = 0; e < kPer; ++e) {
            if (key[u][e] == kZeroKey)
              ++zc;
            else
              atomicAdd(&hist[key[u][e] >> shift0], 1u);
          }
        } else if (vi < nvec) {
#pragma unroll
          for (int e = 0; e < kPer; ++e) {
            const int off = off0 + e;
            if (off >= lo && off < hi) {
              if (key[u][e] == kZeroKey)
                ++zc;
              else
                atomicAdd(&hist[key[u][e] >> shift0], 1u);
            }
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zc += __shfl_xor_sync(0xFFFFFFFFu, zc, o);
    if (lane == 0 && zc) atomicAdd(&hist[kZeroKey >> shift0], zc);
  }
  csync();  // every CTA's histogram is complete
  select_digit(0u, static_cast<uint32_t>(k), shift0, kTopkBins);
  csync();  // no CTA reads another's histogram past this point
  uint32_t prefix = s_prefix, remaining = s_remaining;
  uint32_t prefix_mask = (kTopkBins - 1u) << shift0;
  const bool use_list = s_cge <= static_cast<uint32_t>(kTopkCand);

  // ---- the candidate list: entries whose top digit is >= the selected one
  int n_list = 0;
  if (use_list) {
    const uint32_t t1 = prefix >> shift0;
    for (int base0 = 0; base0 < nvec; base0 += kVStep) {
      const int base = base0 + warp * 32 * kVU;
      uint32_t key[kVU][kPer];
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int vi = base + u * 32 + lane;
        if (vi < nvec) load_keys<T, kPer>(abase, vi, key[u]);
      }
      uint32_t sel[kVU];
      int lane_off[kVU], wtot = 0;
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int vi = base + u * 32 + lane;
        sel[u] = 0;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const int off = vi * kPer + e;
          if (vi < nvec && off >= lo && off < hi && (key[u][e] >> shift0) >= t1) sel[u] |= 1u << e;
        }
        int tot;
        lane_off[u] = wtot + warp_excl_scan(__popc(sel[u]), lane, tot);
        wtot += tot;
      }
      // order: earlier steps, earlier warps of the step, earlier u, lower lanes
      int btotal;
      const int wbefore = block_excl_scan(lane == 0 ? wtot : 0, tmp, btotal);
      const int at0 = n_list + __shfl_sync(0xFFFFFFFFu, wbefore, 0);
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int vi = base + u * 32 + lane;
        int at = at0 + lane_off[u];
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          if ((sel[u] >> e) & 1u) {
            ckey[at] = key[u][e];
            cid[at] = v_lo + (vi * kPer + e - lo);
            ++at;
          }
        }
      }
      n_list += btotal;
    }
    __syncthreads();
  }
  // The entries the later passes walk, in vocab order: the list, or the part.
  const int n_src = use_list ? n_list : v_hi - v_lo;
  auto key_at = [&](int i) -> uint32_t { return use_list ? ckey[i] : Key<T>::of(row + v_lo + i); };
  auto id_at = [&](int i) -> int { return use_list ? cid[i] : v_lo + i; };
  // Each warp takes kTileU*32 consecutive entries per step (entry
  // base + u*32 + lane), all kTileU loads of a lane issued first.
  constexpr int kStep = kTopkThreads * kTileU;

  // ---- the remaining radix passes
  for (int shift = shift0; shift > 0;) {
    const int width = shift < 8 ? shift : 8;
    shift -= width;
    const uint32_t dmask = (1u << width) - 1u;
    constexpr uint32_t kNoDigit = 0xFFFFu;
    for (int i = threadIdx.x; i < (1 << width); i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    // when the key of 0.0 is still in the prefix group its digit is the
    // common one, otherwise lane 0's
    const bool zero_in_group = (kZeroKey & prefix_mask) == prefix;
    const uint32_t zero_digit = (kZeroKey >> shift) & dmask;
    for (int base = warp * 32 * kTileU; base < n_src; base += kStep) {
      uint32_t key[kTileU];
#pragma unroll
      for (int u = 0; u < kTileU; ++u) {
        const int i = base + u * 32 + lane;
        key[u] = i < n_src ? key_at(i) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kTileU; ++u) {
        const int i = base + u * 32 + lane;
        const uint32_t d =
            (i < n_src && (key[u] & prefix_mask) == prefix) ? (key[u] >> shift) & dmask : kNoDigit;
        // The lanes holding the common digit add once (one ballot); the rest
        // add one each.
        const uint32_t dc = zero_in_group ? zero_digit : __shfl_sync(0xFFFFFFFFu, d, 0);
        const unsigned same = __ballot_sync(0xFFFFFFFFu, d == dc);
        if (d == dc) {
          if (d != kNoDigit && lane == __ffs(same) - 1) atomicAdd(&hist[d], __popc(same));
        } else if (d != kNoDigit) {
          atomicAdd(&hist[d], 1u);
        }
      }
    }
    csync();
    select_digit(prefix, remaining, shift, 1 << width);
    csync();
    prefix = s_prefix;
    remaining = s_remaining;
    prefix_mask |= dmask << shift;
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
  for (int base0 = 0; base0 < n_src; base0 += kStep) {
    const int base = base0 + warp * 32 * kTileU;
    uint32_t key[kTileU];
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int i = base + u * 32 + lane;
      key[u] = i < n_src ? key_at(i) : 0u;
    }
    unsigned eqm[kTileU];
    int warp_eq = 0;
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int i = base + u * 32 + lane;
      eqm[u] = __ballot_sync(0xFFFFFFFFu, i < n_src && key[u] == K);
      warp_eq += __popc(eqm[u]);
      if (i < n_src && key[u] > K) {
        const uint32_t at = atomicAdd(dgt, 1u);
        dkey[at] = key[u];
        did[at] = id_at(i);
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
          did[n_gt + r] = id_at(base + u * 32 + lane);
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

// ------------------------------------------------ top-k, rows in shared memory
// One CTA of kRowThreads per row whose keys fit in shared memory (V * key size
// <= kRowStageBytes) and k <= kRowMaxK:
//   1. the row is read once with 16-byte loads; its order-preserving keys go
//      to shared memory (vector i of the aligned-down row at key offset
//      i * kPer) and the top kTopkFirstBits of each key into a histogram
//      (the key of 0.0 is counted in registers and added once per warp);
//   2. the digit holding the k-th largest key is selected; while more than
//      kRowList entries lie at or above it and key bits remain, one more
//      histogram pass over the staged keys of the selected group narrows it;
//   3. the entries at or above the threshold (at most kRowList) are copied
//      into a list of (key << 32 | ~vocab id) words, each warp reserving its
//      slots with one shared atomic; when ties of the exact k-th key
//      overflow the list instead, the list gets the entries above it and the
//      first equals in vocab order (block prefix counts per step);
//   4. each list entry's rank is the number of entries before it in (key
//      descending, vocab id ascending) order, a strict total order, so the
//      entries of rank < k go straight to their output slots.
constexpr int kRowThreads = 1024;
constexpr int kRowList = 1024;
constexpr int kRowMaxK = 512;
constexpr size_t kRowStageBytes = 128 * 1024;

template <typename T>
using RowKey = typename std::conditional<sizeof(T) == 2, uint16_t, uint32_t>::type;

template <typename T, int kPer>
__global__ void __launch_bounds__(kRowThreads)
    topk_row_kernel(const T* __restrict__ reps, int V, int k, T* __restrict__ out_vals,
                    int32_t* __restrict__ out_idx) {
  using KeyT = RowKey<T>;
  extern __shared__ __align__(16) unsigned char smem_row[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem_row);                          // [kTopkBins]
  unsigned long long* list = reinterpret_cast<unsigned long long*>(hist + kTopkBins);  // [kRowList]
  KeyT* skey = reinterpret_cast<KeyT*>(list + kRowList);                          // [nvec * kPer]
  __shared__ int tmp[32];
  __shared__ uint32_t s_prefix, s_remaining, s_cge, s_n;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31;
  constexpr int kBits = Key<T>::kBits;
  constexpr uint32_t kZeroKey = 1u << (kBits - 1);
  constexpr int kU = 4;  // vectors of a thread in flight
  const int shift0 = kBits - kTopkFirstBits;
  const T* row = reps + static_cast<size_t>(b) * V;
  const size_t g0 = static_cast<size_t>(b) * V;
  const size_t a0 = g0 / kPer * kPer;
  const int lo = static_cast<int>(g0 - a0), hi = lo + V;  // key offsets of the row's entries
  const int nvec = (hi + kPer - 1) / kPer;
  for (int i = threadIdx.x; i < kTopkBins; i += kRowThreads) hist[i] = 0;
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();

  // ---- 1. stage the keys, histogram of the top digit
  {
    uint32_t zc = 0;
    for (int base = threadIdx.x; base < nvec; base += kU * kRowThreads) {
      uint32_t key[kU][kPer];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int vi = base + u * kRowThreads;
        if (vi < nvec) load_keys<T, kPer>(reps + a0, vi, key[u]);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int vi = base + u * kRowThreads;
        if (vi >= nvec) continue;
        if constexpr (kPer == 1) {
          skey[vi] = static_cast<KeyT>(key[u][0]);
        } else if constexpr (sizeof(KeyT) == 2) {
          uint4 w;
          w.x = key[u][0] | (key[u][1] << 16);
          w.y = key[u][2] | (key[u][3] << 16);
          w.z = key[u][4] | (key[u][5] << 16);
          w.w = key[u][6] | (key[u][7] << 16);
          *reinterpret_cast<uint4*>(skey + vi * kPer) = w;
        } else {
          *reinterpret_cast<uint4*>(skey + vi * kPer) =
              make_uint4(key[u][0], key[u][1], key[u][2], key[u][3]);
        }
        const int off0 = vi * kPer;
        if (off0 >= lo && off0 + kPer <= hi) {  // a whole vector of the row
#pragma unroll
          for (int e = 0; e < kPer; ++e) {
            if (key[u][e] == kZeroKey)
              ++zc;
            else
              atomicAdd(&hist[key[u][e] >> shift0], 1u);
          }
        } else {
#pragma unroll
          for (int e = 0; e < kPer; ++e) {
            const int off = off0 + e;
            if (off >= lo && off < hi) {
              if (key[u][e] == kZeroKey)
                ++zc;
              else
                atomicAdd(&hist[key[u][e] >> shift0], 1u);
            }
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zc += __shfl_xor_sync(0xFFFFFFFFu, zc, o);
    if (lane == 0 && zc) atomicAdd(&hist[kZeroKey >> shift0], zc);
  }
  __syncthreads();

  // The digit (of nbins) holding the remaining-th largest key of the prefix
  // group: thread t owns digits nbins-1 - t*per - [0, per), descending.
  auto select_digit = [&](uint32_t prefix, uint32_t remaining, int shift, int nbins) {
    const int per = nbins > kRowThreads ? nbins / kRowThreads : 1;
    const int t = static_cast<int>(threadIdx.x);
    constexpr int kPerMax = kTopkBins / kRowThreads;
    uint32_t cnt[kPerMax];
    uint32_t own = 0;
#pragma unroll
    for (int q = 0; q < kPerMax; ++q) {
      const int dgt = nbins - 1 - (t * per + q);
      cnt[q] = (q < per && dgt >= 0) ? hist[dgt] : 0u;
      own += cnt[q];
    }
    int total;
    uint32_t above = static_cast<uint32_t>(block_excl_scan(static_cast<int>(own), tmp, total));
    if (above < remaining && above + own >= remaining) {
#pragma unroll
      for (int q = 0; q < kPerMax; ++q) {
        if (q < per && above + cnt[q] >= remaining) {
          s_prefix = prefix | (static_cast<uint32_t>(nbins - 1 - (t * per + q)) << shift);
          s_remaining = remaining - above;
          s_cge = above + cnt[q];
          break;
        }
        above += cnt[q];
      }
    }
  };

  // ---- 2. select, narrowing while the candidates overflow the list
  select_digit(0u, static_cast<uint32_t>(k), shift0, kTopkBins);
  __syncthreads();
  uint32_t prefix = s_prefix, remaining = s_remaining;
  uint32_t cge = s_cge;  // entries with key >= prefix
  uint32_t pmask = (kTopkBins - 1u) << shift0;
  int shift = shift0;
  while (cge > static_cast<uint32_t>(kRowList) && shift > 0) {
    const int width = shift < 8 ? shift : 8;
    shift -= width;
    const uint32_t dmask = (1u << width) - 1u;
    __syncthreads();  // the previous select's reads of hist are done
    for (int i = threadIdx.x; i < (1 << width); i += kRowThreads) hist[i] = 0;
    __syncthreads();
    uint32_t zc = 0;
    const bool zero_in_group = (kZeroKey & pmask) == prefix;
    for (int off = lo + threadIdx.x; off < hi; off += kRowThreads) {
      const uint32_t key = skey[off];
      if ((key & pmask) == prefix) {
        if (zero_in_group && key == kZeroKey)
          ++zc;
        else
          atomicAdd(&hist[(key >> shift) & dmask], 1u);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zc += __shfl_xor_sync(0xFFFFFFFFu, zc, o);
    if (lane == 0 && zc) atomicAdd(&hist[(kZeroKey >> shift) & dmask], zc);
    __syncthreads();
    const uint32_t above_group = static_cast<uint32_t>(k) - remaining;
    select_digit(prefix, remaining, shift, 1 << width);
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    cge = above_group + s_cge;
    pmask |= dmask << shift;
  }

  // ---- 3. the list
  if (cge <= static_cast<uint32_t>(kRowList)) {
    // every entry with key >= prefix (lower bits of prefix are 0): a lane
    // checks one staged vector of kPer keys, the warp reserves its slots with
    // one shared atomic
    const int warp = threadIdx.x >> 5;
    for (int base = 32 * warp; base < nvec; base += kRowThreads) {
      const int vi = base + lane;
      uint32_t key[kPer];
      unsigned take = 0u;
      if (vi < nvec) {
        if constexpr (kPer == 1) {
          key[0] = skey[vi];
        } else if constexpr (sizeof(KeyT) == 2) {
          const uint4 w = *reinterpret_cast<const uint4*>(skey + vi * kPer);
          const uint32_t q[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            key[2 * e] = q[e] & 0xFFFFu;
            key[2 * e + 1] = q[e] >> 16;
          }
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(skey + vi * kPer);
          key[0] = w.x, key[1] = w.y, key[2] = w.z, key[3] = w.w;
        }
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const int off = vi * kPer + e;
          if (off >= lo && off < hi && key[e] >= prefix) take |= 1u << e;
        }
      }
      int wtot;
      const int ex = warp_excl_scan(__popc(take), lane, wtot);
      if (wtot == 0) continue;  // (warp-uniform)
      uint32_t at = 0;
      if (lane == 0) at = atomicAdd(&s_n, static_cast<uint32_t>(wtot));
      at = __shfl_sync(0xFFFFFFFFu, at, 0) + ex;
#pragma unroll
      for (int e = 0; e < kPer; ++e)
        if ((take >> e) & 1u)
          list[at++] = (static_cast<unsigned long long>(key[e]) << 32) |
                       (0xFFFFFFFFu - static_cast<uint32_t>(vi * kPer + e - lo));
    }
  } else {
    // K = prefix exactly: the entries above K, then the first `remaining`
    // equals in vocab order (thread t of a step takes 32 consecutive entries
    // of a warp-strided span: rank = equals in earlier steps and threads)
    const uint32_t K = prefix;
    const uint32_t n_gt = static_cast<uint32_t>(k) - remaining;
    int eq_seen = 0;
    for (int off0 = lo; off0 < hi; off0 += kRowThreads * 32) {
      const int mine = off0 + 32 * static_cast<int>(threadIdx.x);
      int c_eq = 0;
      for (int j = 0; j < 32; ++j) {
        const int off = mine + j;
        if (off < hi) {
          const uint32_t key = skey[off];
          if (key > K) {
            const uint32_t at = atomicAdd(&s_n, 1u);
            list[at] = (static_cast<unsigned long long>(key) << 32) |
                       (0xFFFFFFFFu - static_cast<uint32_t>(off - lo));
          }
          c_eq += key == K;
        }
      }
      int total;
      int r = eq_seen + block_excl_scan(c_eq, tmp, total);
      for (int j = 0; j < 32 && r < static_cast<int>(remaining); ++j) {
        const int off = mine + j;
        if (off < hi && skey[off] == K) {
          list[n_gt + r] = (static_cast<unsigned long long>(K) << 32) |
                           (0xFFFFFFFFu - static_cast<uint32_t>(off - lo));
          ++r;
        }
      }
      eq_seen += total;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_n = static_cast<uint32_t>(k);
  }
  __syncthreads();

  // ---- 4. rank = entries before this one; rank < k goes to the output.
  // With a short list, tpe consecutive lanes share an entry, each counting
  // over a part of the list, and add their counts.
  const int m = static_cast<int>(s_n);
  const int tpe = m <= kRowThreads / 4 ? 4 : (m <= kRowThreads / 2 ? 2 : 1);
  for (int t0 = 0; t0 < m * tpe; t0 += kRowThreads) {
    const int t = t0 + static_cast<int>(threadIdx.x);
    const int i = t / tpe, part = t % tpe;
    const bool valid = i < m;
    const unsigned long long c = valid ? list[i] : 0ull;
    int rank = 0;
    if (valid) {
      const int j1 = (part + 1) * m / tpe;
      int j = part * m / tpe;
      for (; j + 4 <= j1; j += 4)
        rank += (list[j] > c) + (list[j + 1] > c) + (list[j + 2] > c) + (list[j + 3] > c);
      for (; j < j1; ++j) rank += list[j] > c;
    }
    for (int o = 1; o < tpe; o <<= 1) rank += __shfl_xor_sync(0xFFFFFFFFu, rank, o);
    if (valid && part == 0 && rank < k) {
      const int v = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(c));
      out_idx[static_cast<size_t>(b) * k + rank] = v;
      out_vals[static_cast<size_t>(b) * k + rank] = row[v];
    }
  }
}

template <typename T>
int launch_csr_typed(const void* reps, int B, int V, float thr, int64_t* crow, int32_t* cols,
                     void* vals, int64_t capacity, const SparseWorkspace& ws,
                     cudaStream_t stream) {
  if (B == 0 || V == 0) {  // every row empty
    const cudaError_t e =
        cudaMemsetAsync(crow, 0, (static_cast<size_t>(B) + 1) * sizeof(int64_t), stream);
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "cudaMemsetAsync(crow)");
  }
  // this call's tag for the look-back words (30 bits, never 0)
  static std::atomic<uint32_t> calls{0};
  const uint32_t tag = (calls.fetch_add(1, std::memory_order_relaxed) % 0x3FFFFFFFu) + 1u;
  const int n = static_cast<int>((static_cast<long long>(B) * V + kCsrChunk - 1) / kCsrChunk);
  const size_t smem = static_cast<size_t>(kCsrChunk) * (sizeof(int32_t) + sizeof(T));
  const bool vec = reinterpret_cast<uintptr_t>(reps) % 16 == 0;
  cudaError_t e = cudaFuncSetAttribute(vec ? csr_kernel<T, 16 / sizeof(T)> : csr_kernel<T, 1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "csr_kernel smem");
  if (vec)
    csr_kernel<T, 16 / sizeof(T)><<<n, kCsrThreads, smem, stream>>>(
        static_cast<const T*>(reps), B, V, thr, n, tag, ws.header, ws.flags, capacity, crow, cols,
        static_cast<T*>(vals));
  else
    csr_kernel<T, 1><<<n, kCsrThreads, smem, stream>>>(static_cast<const T*>(reps), B, V, thr, n, tag,
                                                     ws.header, ws.flags, capacity, crow, cols,
                                                     static_cast<T*>(vals));
  e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "csr_kernel launch");
}

template <typename T>
int launch_topk_typed(const void* reps, int B, int V, int k, void* vals, int32_t* idx,
                      cudaStream_t stream) {
  if (B == 0 || k == 0) return SPARTON_OK;
  int k_pad = 1;
  while (k_pad < k) k_pad <<= 1;
  const size_t smem = (kTopkBins + 2 * static_cast<size_t>(k_pad) + 2 * static_cast<size_t>(kTopkCand)) *
                      sizeof(uint32_t);
  // Enough CTAs for two per SM, each walking at least 16384 entries of its
  // row (shorter spans lose more to the cluster barriers than they gain).
  int P = 1;
  while (P < 8 && static_cast<long long>(B) * P < 2ll * device_sm_count() &&
         V / (2 * P) >= 16384)
    P *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kTopkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // 16-byte loads in the first passes when the rows' storage is 16-byte aligned
  const bool vec = reinterpret_cast<uintptr_t>(reps) % 16 == 0;
  constexpr int kPerVec = 16 / sizeof(T);
  const size_t row_keys = (static_cast<size_t>(V) + 2 * kPerVec) * sizeof(RowKey<T>);
  if (k <= kRowMaxK && row_keys <= kRowStageBytes) {
    // the row's keys fit in shared memory: one CTA per row
    const size_t rsmem = kTopkBins * sizeof(uint32_t) + kRowList * sizeof(unsigned long long) +
                         (row_keys + 15) / 16 * 16;
    auto rkernel = vec ? topk_row_kernel<T, kPerVec> : topk_row_kernel<T, 1>;
    cudaError_t e = cudaFuncSetAttribute(rkernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(rsmem));
    if (e != cudaSuccess) return cuda_fail(e, "topk_row_kernel smem");
    rkernel<<<B, kRowThreads, rsmem, stream>>>(static_cast<const T*>(reps), V, k,
                                               static_cast<T*>(vals), idx);
    e = cudaGetLastError();
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "topk_row_kernel launch");
  }
  auto kernel = vec ? topk_kernel<T, kPerVec> : topk_kernel<T, 1>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "topk_kernel smem");
  if (P > 1) {
    cfg.gridDim = dim3(static_cast<unsigned>(P), static_cast<unsigned>(B));
    attr[0].val.clusterDim.x = static_cast<unsigned>(P);
    if (!cluster_fits(kernel, &cfg, P, smem)) P = 1;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(P), static_cast<unsigned>(B));
  attr[0].val.clusterDim.x = static_cast<unsigned>(P);
  e = cudaLaunchKernelEx(&cfg, kernel, static_cast<const T*>(reps), V, k, k_pad,
                         static_cast<T*>(vals), idx);
  if (e != cudaSuccess) return cuda_fail(e, "topk_kernel launch");
  return SPARTON_OK;
}

}  // namespace

size_t sparse_workspace_bytes(int64_t B, int64_t V) {
  const int64_t n = ((B > 0 ? B : 0) * (V > 0 ? V : 0) + kCsrChunk - 1) / kCsrChunk;
  return 256 + align256(static_cast<size_t>(n > 0 ? n : 1) * sizeof(unsigned long long));
}

SparseWorkspace sparse_workspace_carve(void* base, int64_t B, int64_t V) {
  const int64_t n = ((B > 0 ? B : 0) * (V > 0 ? V : 0) + kCsrChunk - 1) / kCsrChunk;
  SparseWorkspace ws;
  ws.header = static_cast<unsigned int*>(base);
  ws.flags = reinterpret_cast<unsigned long long*>(static_cast<char*>(base) + 256);
  ws.bytes = 256 + static_cast<size_t>(n) * sizeof(unsigned long long);
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
