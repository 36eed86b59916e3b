// sparse.cu — sparse forms of the head's output reps [B, V] for indexing:
// the per-row CSR of the entries above a threshold, and the per-row top-k.
//
// Upstream (hhkbble/sparton training/model.py:141-144) `encode` returns the
// dense reps under no_grad, and training/train.py:205-210 logs the fraction
// of entries > 0; an inverted index stores each row's nonzero (vocab id,
// weight) pairs, or its k heaviest.
//
// CSR, one kernel after a memset of its workspace:
//   csr_kernel  one CTA per chunk of kCsrChunk columns of a row, taken in
//               row-major order from a ticket counter: counts the entries >
//               threshold, finds the entries of all earlier chunks by a
//               decoupled look-back over the chunks' published counts and
//               prefixes, and writes (column, value) in column order; crow[b]
//               (row starts) and crow[B] (= nnz). Entries at or past
//               `capacity` are not written (the caller sees nnz in crow[B]).
// Top-k, a cluster of up to 8 CTAs per row (enough CTAs for two per SM):
//   radix select on order-preserving unsigned keys (8 bits a pass: 2 passes
//   for 16-bit types, 4 for fp32), the CTAs' histograms summed through
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

#include "dtype.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

constexpr int kCsrChunk = 4096;
constexpr int kCsrThreads = 256;
constexpr int kTopkThreads = 512;
constexpr int kTileU = 8;  // entries per lane per step of a row walk
constexpr int kTopkCand = 8192;  // candidate list entries per CTA (64 KB of key + id)

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
// Look-back words of the chunks: [status:2][value:62]; status 0 = nothing yet,
// 1 = the chunk's own count, 2 = the inclusive prefix through the chunk.
constexpr unsigned long long kLbCount = 1ull << 62;
constexpr unsigned long long kLbPrefix = 2ull << 62;
constexpr unsigned long long kLbValue = (1ull << 62) - 1;

__device__ __forceinline__ void lb_publish(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long lb_read(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One pass (decoupled look-back): a CTA takes the next chunk of kCsrChunk
// columns in row-major order from a ticket counter (so every chunk before it
// belongs to a CTA that has already started), loads it into registers, counts
// the entries above the threshold per (step, warp), publishes its count, and
// warp 0 walks back over the earlier chunks' words 32 at a time, adding counts
// until it meets an inclusive prefix; the CTA then publishes its own inclusive
// prefix and writes its entries at (prefix + earlier steps and warps + earlier
// u + lower lanes), i.e. columns ascending inside each row. crow[b] is written
// by the row's first chunk, crow[B] by the last chunk. Entries at or past
// `capacity` are not written (the caller sees nnz in crow[B]). The waits are
// on CTAs that are already running and wait on nothing themselves; each is
// bounded anyway (a timeout records SPARTON_DEV_TIMEOUT_SCAN).
template <typename T>
__global__ void __launch_bounds__(kCsrThreads)
    csr_kernel(const T* __restrict__ reps, int B, int V, float thr, int nchunks,
               unsigned int* __restrict__ header, unsigned long long* __restrict__ flags,
               int64_t capacity, int64_t* __restrict__ crow, int32_t* __restrict__ cols,
               T* __restrict__ vals) {
  constexpr int kWarps = kCsrThreads / 32;
  constexpr int kStepCols = kCsrThreads * kTileU;
  constexpr int kSteps = kCsrChunk / kStepCols;
  __shared__ int s_cnt[kSteps * kWarps];
  __shared__ int s_id;
  __shared__ long long s_excl;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  if (threadIdx.x == 0) s_id = static_cast<int>(atomicAdd(header + 1, 1u));
  __syncthreads();
  const int id = s_id;
  const int b = id / nchunks, ch = id - b * nchunks;
  const int v0 = ch * kCsrChunk, v1 = min(V, v0 + kCsrChunk);
  const T* row = reps + static_cast<size_t>(b) * V;
  T x[kSteps][kTileU];
  unsigned keep[kSteps][kTileU];
#pragma unroll
  for (int st = 0; st < kSteps; ++st)
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = v0 + st * kStepCols + warp * 32 * kTileU + u * 32 + lane;
      x[st][u] = v < v1 ? row[v] : T{};
    }
#pragma unroll
  for (int st = 0; st < kSteps; ++st) {
    int n = 0;
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      const int v = v0 + st * kStepCols + warp * 32 * kTileU + u * 32 + lane;
      keep[st][u] = __ballot_sync(0xFFFFFFFFu, v < v1 && to_f32<T>(x[st][u]) > thr);
      n += __popc(keep[st][u]);
    }
    if (lane == 0) s_cnt[st * kWarps + warp] = n;
  }
  __syncthreads();
  int total = 0;
#pragma unroll
  for (int i = 0; i < kSteps * kWarps; ++i) total += s_cnt[i];
  if (warp == 0) {
    long long excl = 0;
    bool ok = true;
    if (id == 0) {
      if (lane == 0) lb_publish(flags, kLbPrefix | static_cast<unsigned long long>(total));
    } else {
      if (lane == 0) lb_publish(flags + id, kLbCount | static_cast<unsigned long long>(total));
      const uint64_t t0 = global_timer_ns();
      for (int pos = id - 1;; pos -= 32) {
        const int j = pos - lane;  // lane 0 is the nearest earlier chunk
        unsigned long long f = kLbPrefix;  // before chunk 0: an inclusive prefix of 0
        if (j >= 0) {
          f = lb_read(flags + j);
          while ((f >> 62) == 0) {
            if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              ok = false;
              break;
            }
            __nanosleep(64);
            f = lb_read(flags + j);
          }
        }
        if (!__all_sync(0xFFFFFFFFu, ok)) {
          ok = false;
          break;
        }
        const unsigned pre = __ballot_sync(0xFFFFFFFFu, (f >> 62) == 2);
        const int stop = pre ? __ffs(pre) - 1 : 31;  // the nearest inclusive prefix
        long long add = lane <= stop ? static_cast<long long>(f & kLbValue) : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) add += __shfl_xor_sync(0xFFFFFFFFu, add, o);
        excl += add;
        if (pre) break;
      }
      if (lane == 0) {
        if (ok)
          lb_publish(flags + id, kLbPrefix | static_cast<unsigned long long>(excl + total));
        else
          atomicCAS(header, 0u, SPARTON_DEV_TIMEOUT_SCAN);
      }
    }
    if (lane == 0) s_excl = excl;
  }
  __syncthreads();
  const long long excl = s_excl;
  if (threadIdx.x == 0) {
    if (ch == 0) crow[b] = excl;
    if (id == B * nchunks - 1) crow[B] = excl + total;
  }
  if (capacity <= 0) return;
  int before = 0;  // entries of the earlier (step, warp) spans
  for (int i = 0; i < warp; ++i) before += s_cnt[i];
#pragma unroll
  for (int st = 0; st < kSteps; ++st) {
    long long at = excl + before;
#pragma unroll
    for (int u = 0; u < kTileU; ++u) {
      if ((keep[st][u] >> lane) & 1u) {
        const long long i = at + __popc(keep[st][u] & lt);
        if (i < capacity) {
          cols[i] = v0 + st * kStepCols + warp * 32 * kTileU + u * 32 + lane;
          vals[i] = x[st][u];
        }
      }
      at += __popc(keep[st][u]);
    }
    // the rest of this step, then the next step's warps before this one
    for (int i = warp; i < kWarps; ++i) before += s_cnt[st * kWarps + i];
    if (st + 1 < kSteps)
      for (int i = 0; i < warp; ++i) before += s_cnt[(st + 1) * kWarps + i];
  }
}

// ------------------------------------------------------------------ top-k
// A thread-block cluster of P CTAs per row (P = 1 .. 8); CTA c walks the vocab
// range [c*part, (c+1)*part). Shared memory: hist[256], k_pad (key, id) pairs
// (used in CTA 0), then a candidate list of up to kTopkCand (key, id) pairs.
//
// Pass 1 reads the CTA's part with 16-byte loads (kPer elements each; kPer = 1
// when reps is not 16-byte aligned) and histograms the top 8 key bits; lanes
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
  uint32_t* hist = smem;                                          // [256]
  uint32_t* skey = smem + 256;                                    // [k_pad]
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
  // Digits in descending order, one per thread: the digit whose bucket holds
  // the remaining-th largest key of the prefix group (every CTA sums the
  // cluster's histograms itself and picks the same digit).
  auto select_digit = [&](uint32_t prefix, uint32_t remaining, int shift) {
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
      s_cge = above + own;   // entries of the group at or above the digit
    }
  };

  // ---- pass 1: the top 8 bits, 16-byte loads
  const size_t g0 = static_cast<size_t>(b) * V + v_lo;
  const size_t a0 = g0 / kPer * kPer;
  const int lo = static_cast<int>(g0 - a0), hi = lo + (v_hi - v_lo);  // element offsets from a0
  const int nvec = v_hi > v_lo ? (hi + kPer - 1) / kPer : 0;
  const T* abase = reps + a0;
  constexpr int kVU = kPer == 1 ? 8 : 2;  // loads per lane per step
  constexpr int kVStep = kTopkThreads * kVU;
  const int shift0 = kBits - 8;
  for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
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
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const int off = vi * kPer + e;
          if (vi < nvec && off >= lo && off < hi) {
            if (key[u][e] == kZeroKey)
              ++zc;
            else
              atomicAdd(&hist[key[u][e] >> shift0], 1u);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zc += __shfl_xor_sync(0xFFFFFFFFu, zc, o);
    if (lane == 0 && zc) atomicAdd(&hist[kZeroKey >> shift0], zc);
  }
  csync();  // every CTA's histogram is complete
  select_digit(0u, static_cast<uint32_t>(k), shift0);
  csync();  // no CTA reads another's histogram past this point
  uint32_t prefix = s_prefix, remaining = s_remaining;
  uint32_t prefix_mask = 0xFFu << shift0;
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
  for (int shift = kBits - 16; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    // when the key of 0.0 is still in the prefix group its digit is the
    // common one, otherwise lane 0's
    const bool zero_in_group = (kZeroKey & prefix_mask) == prefix;
    const uint32_t zero_digit = (kZeroKey >> shift) & 0xFFu;
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
            (i < n_src && (key[u] & prefix_mask) == prefix) ? (key[u] >> shift) & 0xFFu : 256u;
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
    csync();
    select_digit(prefix, remaining, shift);
    csync();
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
  // status, ticket and look-back words start at zero
  cudaError_t e = cudaMemsetAsync(ws.header, 0, ws.bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(csr workspace)");
  const int n = B * nchunks;
  csr_kernel<T><<<n, kCsrThreads, 0, stream>>>(static_cast<const T*>(reps), B, V, thr, nchunks,
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
  const size_t smem = (256 + 2 * static_cast<size_t>(k_pad) + 2 * static_cast<size_t>(kTopkCand)) *
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
  auto kernel = vec ? topk_kernel<T, 16 / sizeof(T)> : topk_kernel<T, 1>;
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
  const int64_t nchunks = (V + kCsrChunk - 1) / kCsrChunk;
  const int64_t n = (B > 0 ? B : 1) * (nchunks > 0 ? nchunks : 1);
  return 256 + align256(static_cast<size_t>(n) * sizeof(unsigned long long));
}

SparseWorkspace sparse_workspace_carve(void* base, int64_t B, int64_t V) {
  const int64_t nchunks = (V + kCsrChunk - 1) / kCsrChunk;
  SparseWorkspace ws;
  ws.header = static_cast<unsigned int*>(base);
  ws.flags = reinterpret_cast<unsigned long long*>(static_cast<char*>(base) + 256);
  ws.bytes = 256 + static_cast<size_t>(B > 0 ? B : 0) * static_cast<size_t>(nchunks) *
                       sizeof(unsigned long long);
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
