// fwd_tc.cu — K1: the fused SPLADE head forward on sm_100a tensor cores.
//
// What it replaces upstream (hhkbble/sparton src/sparton/sparton_kernel.py):
//   fused_sparton_fwd_with_indices :226-253 loops over vocab chunks; per chunk
//   a torch.compile GEMM (+bias) writes logits [B,S,C] to HBM (:244-247) and the
//   Triton kernel reduce_seq_max_log1p_relu_kernel_with_indices (:84-168)
//   re-reads them for the masked max / argmax over S and log1p(relu(.)).
// Here one persistent kernel does all of it and [B,S,V] never exists.
//
// Orientation. The GEMM is computed transposed: the MMA's M dimension is the
// vocabulary (128 rows of W per tile, one TMEM lane per vocab id) and N runs
// over positions. A thread of the epilogue owns one vocab id and scans its own
// TMEM lane along the positions: the max / argmax needs no cross-thread
// reduction.
//
// Packed positions. The positions [0, round16(extent)) of all batch rows are
// laid end to end in one stream of T packed columns (pack_prepare_kernel in
// mask.cu; workspace layout in internal.h). The kernel cuts the rows into G
// groups by the packed column at which each row starts (group g: rows
// starting in [g*T/G, (g+1)*T/G)); a work unit is (vocab tile of 128, group).
// G is chosen on the device from T, the vocab tile count and the grid, so that
// the units spread evenly over the CTAs: it minimises
//   ceil(units / CTAs) * (tiles per unit + 1/2)
// (the 1/2 stands for the part-filled last tile of a unit). Every CTA computes
// the same G. A unit is processed as tiles of 256 packed columns, so almost
// every MMA has N = 256 whatever the row lengths:
// an MMA's cost has a large part that does not depend on N, and rows of ~150
// positions one MMA tile each ran at ~60% of the 256-column rate. A tile holds
// pieces of up to 16 rows; the producer loads each piece with ONE TMA box of
// exactly its length (16 tensor maps, boxes of 16, 32, ..., 256 rows; pieces
// start at 1024-byte aligned shared offsets, so the 128-byte swizzle matches
// that of a single box). A tile's pieces are worked out once, one per lane of
// the producer warp (from the group's list of rows with columns), and each
// lane issues its own box. The epilogue follows the row boundaries through a
// bitmap of row starts and carries a row's running max across tiles.
//
// Units go round-robin over the CTAs (CTA i takes units i, i + grid, ...), in
// panel order: panels of groups whose hidden states fit in L2, vocab-tile-major
// inside a panel. Every role of a CTA walks the same unit sequence, so no unit
// ids pass between them.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0    TMA producer: W tile [128 x 64] + packed hidden tile [N x 64] per
//             stage, 4 stages, 128-byte swizzle.
//   warp 1    TMEM owner + MMA issuer: tcgen05.mma kind::f16, fp32 accumulator
//             in TMEM, two 256-column accumulators (MMA of the next tile
//             overlaps the epilogue of the previous one).
//   Warps 0 and 1 run their loops with all 32 lanes and issue each TMA copy,
//   MMA and commit from one elected lane (ptx.cuh elect_one).
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time (the next chunk's load
//             in flight while one is scanned), masked running max and
//             first-index argmax over positions (strict >, as upstream
//             :150-156); at the end of each row: bias, relu, log1p and the
//             stores of reps / idx. The tile's bitmap words and the unit's bias
//             are fetched before the wait for the accumulator.
//
// Every wait is bounded (ptx.cuh); on timeout the CTA records a status code,
// drains its in-flight TMA copies and MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <math.h>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

constexpr int kBM = 128;        // vocab rows per tile = MMA M = TMEM lanes
constexpr int kBN = 256;        // packed columns per tile = max MMA N
constexpr int kBK = 64;         // K elements per stage: 128-byte rows
constexpr int kStages = 4;      // TMA -> MMA pipeline depth
constexpr int kRowBytes = kBK * 2;
constexpr int kABytes = kBM * kRowBytes;
constexpr int kBBytes = kBN * kRowBytes;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kNumHiddenMaps = kBN / 16;  // boxes of 16, 32, ..., 256 rows
constexpr int kNumAcc = 2;
constexpr int kTmemCols = kNumAcc * kBN;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kTileWords = kBN / 32;  // bitmap words per tile

// Barrier indices inside the barrier block.
constexpr int kBarFull = 0;
constexpr int kBarEmpty = kBarFull + kStages;
constexpr int kBarTFull = kBarEmpty + kStages;
constexpr int kBarTEmpty = kBarTFull + kNumAcc;
constexpr int kBarDrain = kBarTEmpty + kNumAcc;
constexpr int kNumBars = kBarDrain + 1;

constexpr int kCtrlOffset = kStages * kStageBytes;  // barriers, TMEM address, abort flag
constexpr int kTmemHolderOffset = kCtrlOffset + kNumBars * 8;
constexpr int kAbortOffset = kTmemHolderOffset + 4;
constexpr int kPartOffset = kAbortOffset + 4;  // float[kThreads/32] + int[kThreads/32]
constexpr int kCtrlBytes = 512;
static_assert(kPartOffset + 8 * (kThreads / 32) <= kCtrlOffset + kCtrlBytes,
              "control block overflow");
constexpr int kSmemBytes = kCtrlOffset + kCtrlBytes + 1024;  // + alignment slack

struct alignas(64) HiddenMaps {
  CUtensorMap m[kNumHiddenMaps];  // m[i]: boxes of 16 * (i + 1) rows x 64 columns
};

struct FwdTcParams {
  int B, S, D, V;
  int num_vtiles;
  int num_kblocks;
  const unsigned int* total_cols;
  const int* pcol;
  const int* plen;
  const int* pnz;
  const int* prows;
  const uint32_t* pvalid;
  const uint32_t* prow;
  const void* bias;
  void* reps;
  int32_t* idx;
  unsigned int* status;
};

template <typename T>
__device__ __forceinline__ float to_float(T x);
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half x) {
  return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float x) {
  return __float2half_rn(x);
}

// How the rows are cut into groups for this launch (identical in every CTA).
struct Partition {
  int T;        // packed columns in total
  int G;        // row groups
  int panel_g;  // groups per L2 panel
  long long num_units;
};

// First row whose packed start is >= x (B if none).
__device__ __forceinline__ int first_row_from(const FwdTcParams& p, long long x) {
  int lo = 0, hi = p.B;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(p.pcol + mid) < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// One unit: vocab tile vt, rows [r0, r1), packed columns [c0, c1), entries
// [k0, k1) of prows.
struct Unit {
  int vt, r0, r1, c0, c1, k0, k1;
};

// Walks the units of this CTA: blockIdx.x, + gridDim.x, ... The next unit is
// located (binary searches over the row starts) one unit ahead.
struct UnitIter {
  long long j;
  Unit cur, nxt;
  bool has_next;
  __device__ __forceinline__ void locate(long long u, const FwdTcParams& p, const Partition& q,
                                         Unit& o) const {
    const long long per_panel = static_cast<long long>(p.num_vtiles) * q.panel_g;
    const long long panel = u / per_panel;
    const int r = static_cast<int>(u - panel * per_panel);
    const int g0 = static_cast<int>(panel) * q.panel_g;
    const int pg = min(q.panel_g, q.G - g0);
    const int g = g0 + r % pg;
    o.vt = r / pg;
    o.r0 = g == 0 ? 0 : first_row_from(p, static_cast<long long>(g) * q.T / q.G);
    o.r1 = g == q.G - 1 ? p.B : first_row_from(p, static_cast<long long>(g + 1) * q.T / q.G);
    o.c0 = o.r0 < p.B ? __ldg(p.pcol + o.r0) : q.T;
    o.c1 = o.r1 < p.B ? __ldg(p.pcol + o.r1) : q.T;
    o.k0 = __ldg(p.pnz + o.r0);
    o.k1 = __ldg(p.pnz + o.r1);
  }
  __device__ __forceinline__ bool start(const FwdTcParams& p, const Partition& q) {
    j = blockIdx.x;
    if (j >= q.num_units) return false;
    locate(j, p, q, cur);
    has_next = j + gridDim.x < q.num_units;
    if (has_next) locate(j + gridDim.x, p, q, nxt);
    return true;
  }
  __device__ __forceinline__ bool advance(const FwdTcParams& p, const Partition& q) {
    if (!has_next) return false;
    j += gridDim.x;
    cur = nxt;
    has_next = j + gridDim.x < q.num_units;
    if (has_next) locate(j + gridDim.x, p, q, nxt);
    return true;
  }
};

struct Ctrl {
  uint32_t bar0;  // shared address of barrier 0
  volatile int* abort_flag;
  __device__ __forceinline__ uint32_t bar(int i) const { return bar0 + 8u * i; }
};

__device__ void run_producer(const FwdTcParams& p, const Partition& q, const CUtensorMap* tmW,
                             const CUtensorMap* tmH, uint32_t stage_base, const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t issued_mask = 0, issued_parity = 0;
  bool ok = true;
  const int lane = threadIdx.x & 31;
  UnitIter u;
  for (bool more = u.start(p, q); more && ok; more = u.advance(p, q)) {
    const Unit& un = u.cur;
    // k0: entry in prows of the first row that reaches into the current tile.
    int k0 = un.k0;
    const int k_end = un.k1;
    for (int t0 = un.c0; t0 < un.c1 && ok; t0 += kBN) {
      const int n = min(kBN, un.c1 - t0);  // a multiple of 16
      const int t1 = t0 + n;
      // Lane i describes piece i of the tile: row prows[k0 + i] clipped to
      // [t0, t1). Pieces are >= 16 columns, so a tile has at most 16.
      bool has_piece = false;
      uint32_t dst_off = 0;
      int grow = 0, map_i = 0;
      bool ends_here = false;
      if (lane < kBN / 16 && k0 + lane < k_end) {
        const int b = __ldg(p.prows + k0 + lane);
        const int c0 = __ldg(p.pcol + b), c1 = c0 + __ldg(p.plen + b);
        const int s0 = max(c0, t0), s1 = min(c1, t1);
        has_piece = s0 < s1;
        ends_here = has_piece && c1 <= t1;
        dst_off = static_cast<uint32_t>(kABytes + (s0 - t0) * kRowBytes);
        grow = b * p.S + (s0 - c0);
        map_i = (s1 - s0) / 16 - 1;
      }
      k0 += __popc(__ballot_sync(0xFFFFFFFFu, ends_here));
      const uint32_t bytes = static_cast<uint32_t>(kABytes + n * kRowBytes);
      for (int kb = 0; kb < p.num_kblocks; ++kb) {
        if (!mbar_wait_bounded_warp(c.bar(kBarEmpty + stage), phase ^ 1, c.abort_flag, p.status,
                                    SPARTON_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        const uint32_t full = c.bar(kBarFull + stage);
        const uint32_t a_dst = stage_base + stage * kStageBytes;
        if (lane == 0) {
          mbar_arrive_expect_tx(full, bytes);
          tma_load_2d(a_dst, tmW, full, kb * kBK, un.vt * kBM);
        }
        __syncwarp();
        // One box per row piece; the pieces tile [t0, t1) exactly.
        if (has_piece) tma_load_2d(a_dst + dst_off, tmH + map_i, full, kb * kBK, grow);
        __syncwarp();
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }
  for (int s = 0; s < kStages; ++s) {
    if (!(issued_mask & (1u << s))) continue;
    const uint32_t par = (issued_parity >> s) & 1;
    // Normal end: the MMA's last commits to `empty` have landed before the CTA
    // may exit. Unwinding: every issued copy has landed.
    const uint32_t bar = c.bar((ok ? kBarEmpty : kBarFull) + s);
    if (!mbar_wait_drain(bar, par)) atomicCAS(p.status, 0u, SPARTON_DEV_TIMEOUT_DRAIN);
  }
}

template <uint32_t kFmt>
__device__ void run_mma(const FwdTcParams& p, const Partition& q, uint32_t stage_base,
                        uint32_t tmem_base, const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t tile = 0;
  bool ok = true;
  bool issued = false;
  UnitIter u;
  for (bool more = u.start(p, q); more && ok; more = u.advance(p, q)) {
    const Unit& un = u.cur;
    for (int t0 = un.c0; t0 < un.c1; t0 += kBN) {
      const int acc = tile % kNumAcc;
      const uint32_t aph = (tile / kNumAcc) & 1;
      if (!mbar_wait_bounded_warp(c.bar(kBarTEmpty + acc), aph ^ 1, c.abort_flag, p.status,
                                  SPARTON_DEV_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t n_mma = static_cast<uint32_t>(min(kBN, un.c1 - t0));
      const uint32_t idesc = umma_idesc_f16(kFmt, kBM, n_mma);
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
      for (int kb = 0; kb < p.num_kblocks; ++kb) {
        if (!mbar_wait_bounded_warp(c.bar(kBarFull + stage), phase, c.abort_flag, p.status,
                                    SPARTON_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        if (elect_one()) {
          const uint32_t a_addr = stage_base + stage * kStageBytes;
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_f16(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                     umma_desc_k_sw128(b_addr + kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(c.bar(kBarEmpty + stage));
        }
        __syncwarp();
        issued = true;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(c.bar(kBarTFull + acc));
      __syncwarp();
      ++tile;
    }
  }
  if (!ok && issued) {
    // Unwinding: wait for every MMA this thread issued before TMEM is freed.
    if (elect_one()) umma_commit(c.bar(kBarDrain));
    __syncwarp();
    if (!mbar_wait_drain(c.bar(kBarDrain), 0)) atomicCAS(p.status, 0u, SPARTON_DEV_TIMEOUT_DRAIN);
  }
}

// Folds the columns of one TMEM chunk selected by `mw` into the running masked
// max / first argmax; column q of the chunk is position pos0 + q of the row.
// kIdx false (inference forward, no idx output): the max alone.
template <bool kIdx>
__device__ __forceinline__ void scan_chunk(const uint32_t (&r)[32], uint32_t mw, int pos0,
                                           float& best, int& best_idx) {
  if (mw == 0u) return;
  float cm = -INFINITY;
  if (mw == 0xFFFFFFFFu) {
#pragma unroll
    for (int q = 0; q < 32; ++q) cm = fmaxf(cm, __uint_as_float(r[q]));
  } else {
#pragma unroll
    for (int q = 0; q < 32; ++q) cm = ((mw >> q) & 1u) ? fmaxf(cm, __uint_as_float(r[q])) : cm;
  }
  if (!kIdx) {
    best = fmaxf(best, cm);
    return;
  }
  if (cm > best) {
    int first = 31;
#pragma unroll
    for (int q = 31; q >= 0; --q)
      if (((mw >> q) & 1u) && __uint_as_float(r[q]) == cm) first = q;
    best = cm;
    best_idx = pos0 + first;
  }
}

// Per-thread state of the epilogue inside one unit: the current row and its
// running max. Rows are visited in order; empty rows (no packed columns) are
// written as the empty-row value when the walk passes them.
template <typename T, bool kIdx>
struct RowWalk {
  int b;         // current row (below the group's first row: none yet)
  int nxt;       // the next row with columns (the group's end: none)
  int kk;        // entry in prows after nxt
  int k_end;     // end of the group's entries in prows
  int g_end;
  int row_base;  // packed column of the current row's position 0
  float best;
  int best_idx;
  int v;
  float bias;

  __device__ __forceinline__ void store(const FwdTcParams& p, int row) const {
    if (v < p.V) {
      // max_s(x_s + bias) = max_s(x_s) + bias: the bias is added once, after the
      // max. Upstream's initial value 0 (:112) is the `logit > 0` test.
      const float logit = best + bias;
      const bool pos = logit > 0.f;
      const size_t o = static_cast<size_t>(row) * p.V + v;
      static_cast<T*>(p.reps)[o] = from_float<T>(pos ? log1pf(logit) : 0.f);
      if (kIdx) p.idx[o] = pos ? best_idx : 0;
    }
  }
  // Stores the current row (if any), then every (empty) row before `upto`.
  __device__ __forceinline__ void finish_until(const FwdTcParams& p, int first_row, int upto) {
    if (b >= first_row) store(p, b);
    best = -INFINITY;
    best_idx = 0;
    for (int e = max(b + 1, first_row); e < upto; ++e) store(p, e);
  }
  // A row starts at packed column `col`: it is `nxt`, the next row with
  // columns; the one after it is fetched now, for the next row start.
  __device__ __forceinline__ void next_row(const FwdTcParams& p, int first_row, int col) {
    finish_until(p, first_row, nxt);
    b = nxt;
    row_base = col;
    nxt = kk < k_end ? __ldg(p.prows + kk) : g_end;
    ++kk;
  }
};

// Bits of chunk ch of a tile whose first column sits `sh` bits into the word
// held by lane 0 (lane i holds the tile's word i), limited to the columns
// before the unit's end (`left` columns remain from the chunk's start): the
// stream goes on with the next unit's rows.
__device__ __forceinline__ uint32_t chunk_bits(uint32_t words, int ch, int sh, int left) {
  const uint32_t lo = __shfl_sync(0xFFFFFFFFu, words, ch);
  const uint32_t hi = __shfl_sync(0xFFFFFFFFu, words, ch + 1);
  const uint32_t lim = left >= 32 ? 0xFFFFFFFFu : ((1u << left) - 1u);
  return __funnelshift_r(lo, hi, sh) & lim;
}

// One 32-column chunk at packed column cc: valid bits `mw`, row starts `rs`
// (rows start at multiples of 16, so only bits 0 and 16 can be set).
template <typename T, bool kIdx>
__device__ __forceinline__ void epi_chunk(const FwdTcParams& p, const uint32_t (&r)[32],
                                          uint32_t mw, uint32_t rs, int cc, int first_row,
                                          RowWalk<T, kIdx>& w) {
  if (rs & 1u) w.next_row(p, first_row, cc);
  if (rs & 0x10000u) {
    scan_chunk<kIdx>(r, mw & 0xFFFFu, cc - w.row_base, w.best, w.best_idx);
    w.next_row(p, first_row, cc + 16);
    scan_chunk<kIdx>(r, mw & 0xFFFF0000u, cc - w.row_base, w.best, w.best_idx);
  } else {
    scan_chunk<kIdx>(r, mw, cc - w.row_base, w.best, w.best_idx);
  }
}

template <typename T, bool kIdx>
__device__ void run_epilogue(const FwdTcParams& p, const Partition& q, uint32_t tmem_base,
                             const Ctrl& c, int warp, int lane) {
  const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad+32)
  const int row = quad * 32 + lane;
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
  uint32_t tile = 0;
  UnitIter u;
  for (bool more = u.start(p, q); more; more = u.advance(p, q)) {
    const Unit& un = u.cur;
    const int g_begin = un.r0, g_end = un.r1;
    RowWalk<T, kIdx> w;
    w.b = g_begin - 1;
    w.kk = un.k0;
    w.k_end = un.k1;
    w.g_end = g_end;
    w.nxt = w.kk < w.k_end ? __ldg(p.prows + w.kk) : g_end;
    ++w.kk;
    w.row_base = 0;
    w.best = -INFINITY;
    w.best_idx = 0;
    w.v = un.vt * kBM + row;
    w.bias = (p.bias != nullptr && w.v < p.V) ? to_float<T>(static_cast<const T*>(p.bias)[w.v])
                                               : 0.f;
    bool ok = true;
    for (int t0 = un.c0; t0 < un.c1; t0 += kBN) {
      // Lane i holds bitmap word (t0 >> 5) + i; a tile starts at a multiple of
      // 16, so chunk ch is a funnel shift of words ch and ch + 1.
      const int wsh = t0 & 31;
      const uint32_t vwords = lane <= kTileWords ? __ldg(p.pvalid + (t0 >> 5) + lane) : 0u;
      const uint32_t swords = lane <= kTileWords ? __ldg(p.prow + (t0 >> 5) + lane) : 0u;
      const int acc = tile % kNumAcc;
      const uint32_t aph = (tile / kNumAcc) & 1;
      // The whole warp leaves together (the TMEM loads below are warp-wide),
      // even if a wait gave up in only some of its lanes.
      const bool got = mbar_wait_bounded(c.bar(kBarTFull + acc), aph, c.abort_flag, p.status,
                                         SPARTON_DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xFFFFFFFFu, got)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const int nch = (min(kBN, un.c1 - t0) + 31) >> 5;
      const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * kBN);
      uint32_t ra[32], rb[32];
      tmem_ld_32x32b_x32(taddr, ra);
      for (int ch = 0; ch < nch; ch += 2) {
        tmem_ld_wait(ra);
        if (ch + 1 < nch) tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(32 * (ch + 1)), rb);
        const int left0 = un.c1 - (t0 + 32 * ch);
        epi_chunk<T, kIdx>(p, ra, chunk_bits(vwords, ch, wsh, left0),
                     chunk_bits(swords, ch, wsh, left0), t0 + 32 * ch, g_begin, w);
        if (ch + 1 < nch) {
          tmem_ld_wait(rb);
          if (ch + 2 < nch) tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(32 * (ch + 2)), ra);
          const int left1 = un.c1 - (t0 + 32 * (ch + 1));
          epi_chunk<T, kIdx>(p, rb, chunk_bits(vwords, ch + 1, wsh, left1),
                       chunk_bits(swords, ch + 1, wsh, left1), t0 + 32 * (ch + 1), g_begin, w);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(c.bar(kBarTEmpty + acc));
      ++tile;
    }
    if (!ok) break;
    w.finish_until(p, g_begin, g_end);
  }
}

// Chooses G for this launch; all threads of the CTA take part and every CTA
// gets the same answer. Candidate G = 1 .. min(B, 4 * grid); cost as in the
// header comment; ties go to the smaller G.
__device__ Partition choose_partition(const FwdTcParams& p, float* red_cost, int* red_g) {
  Partition q;
  q.T = static_cast<int>(*p.total_cols);
  const int gmax = max(1, min(p.B, 4 * static_cast<int>(gridDim.x)));
  float best = INFINITY;
  int best_g = 1;
  for (int g = threadIdx.x + 1; g <= gmax; g += blockDim.x) {
    const long long units = static_cast<long long>(p.num_vtiles) * g;
    const long long rounds = (units + gridDim.x - 1) / gridDim.x;
    const float cost = static_cast<float>(rounds) *
                       (static_cast<float>(q.T) / (256.f * static_cast<float>(g)) + 0.5f);
    if (cost < best) {
      best = cost;
      best_g = g;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float oc = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int og = __shfl_xor_sync(0xFFFFFFFFu, best_g, o);
    if (oc < best || (oc == best && og < best_g)) {
      best = oc;
      best_g = og;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_cost[warp] = best;
    red_g[warp] = best_g;
  }
  __syncthreads();
  best = red_cost[0];
  best_g = red_g[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
    if (red_cost[w] < best || (red_cost[w] == best && red_g[w] < best_g)) {
      best = red_cost[w];
      best_g = red_g[w];
    }
  }
  q.G = best_g;
  q.num_units = static_cast<long long>(p.num_vtiles) * q.G;
  // Panel of groups whose hidden states (~T/G packed columns of D * 2 bytes
  // each) fit in ~48 MB of L2.
  const long long group_bytes =
      (static_cast<long long>(q.T) / q.G + 256) * static_cast<long long>(p.D) * 2;
  q.panel_g = static_cast<int>(max(1ll, min(static_cast<long long>(q.G), (48ll << 20) / group_bytes)));
  return q;
}

template <typename T, uint32_t kFmt, bool kIdx>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ HiddenMaps tmH,
                  const FwdTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t stage_base = smem_addr(smem);
  Ctrl c;
  c.bar0 = stage_base + kCtrlOffset;
  c.abort_flag = reinterpret_cast<volatile int*>(smem + kAbortOffset);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kTmemHolderOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(c.bar(kBarFull + s), 1);
      mbar_init(c.bar(kBarEmpty + s), 1);
    }
    for (int a = 0; a < kNumAcc; ++a) {
      mbar_init(c.bar(kBarTFull + a), 1);
      mbar_init(c.bar(kBarTEmpty + a), kEpiWarps);
    }
    mbar_init(c.bar(kBarDrain), 1);
    *c.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    for (int i = 0; i < kNumHiddenMaps; ++i) tma_prefetch_desc(&tmH.m[i]);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  // Everything above overlaps the end of pack_prepare_kernel (programmatic
  // dependent launch); its results are read from here on.
  pdl_wait();
  const Partition q = choose_partition(p, reinterpret_cast<float*>(smem + kPartOffset),
                                       reinterpret_cast<int*>(smem + kPartOffset) + kThreads / 32);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    run_producer(p, q, &tmW, tmH.m, stage_base, c);
    __syncwarp();
  } else if (warp == 1) {
    run_mma<kFmt>(p, q, stage_base, tmem_base, c);
    __syncwarp();
  } else {
    run_epilogue<T, kIdx>(p, q, tmem_base, c, warp, lane);
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ----------------------------------------------------------------------- host
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                uint64_t outer, uint32_t box_inner, uint32_t box_outer) {
  return make_tensor_map_2d(map, dt, base, inner, outer, inner * 2, box_inner, box_outer,
                            CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, uint32_t kFmt, bool kIdx>
int launch_kernel(const CUtensorMap& tmW, const HiddenMaps& tmH, const FwdTcParams& p,
                  unsigned grid, cudaStream_t stream) {
  static std::mutex mu;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      e = cudaFuncSetAttribute(fwd_tc_kernel<T, kFmt, kIdx>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd_tc_kernel)");
      attr_done[dev] = true;
    }
  }
  e = launch_pdl(fwd_tc_kernel<T, kFmt, kIdx>, dim3(grid), dim3(kThreads), kSmemBytes, stream, tmW,
                 tmH, p);
  if (e != cudaSuccess) return cuda_fail(e, "fwd_tc_kernel launch");
  return SPARTON_OK;
}

template <typename T, uint32_t kFmt>
int launch_typed(CUtensorMapDataType dt, const void* hidden, const void* weight, const void* bias,
                 int B, int S, int D, int V, void* reps, int32_t* idx, const FwdWorkspace& ws,
                 cudaStream_t stream) {
  CUtensorMap tmW;
  HiddenMaps tmH;
  int st = make_map_2d(&tmW, dt, weight, static_cast<uint64_t>(D), static_cast<uint64_t>(V), kBK,
                       kBM);
  if (st != SPARTON_OK) return st;
  for (int i = 0; i < kNumHiddenMaps; ++i) {
    st = make_map_2d(&tmH.m[i], dt, hidden, static_cast<uint64_t>(D),
                     static_cast<uint64_t>(B) * static_cast<uint64_t>(S), kBK,
                     static_cast<uint32_t>(16 * (i + 1)));
    if (st != SPARTON_OK) return st;
  }

  FwdTcParams p;
  p.B = B;
  p.S = S;
  p.D = D;
  p.V = V;
  p.num_vtiles = (V + kBM - 1) / kBM;
  p.num_kblocks = (D + kBK - 1) / kBK;
  p.total_cols = ws.total_cols;
  p.pcol = ws.pcol;
  p.plen = ws.plen;
  p.pnz = ws.pnz;
  p.prows = ws.prows;
  p.pvalid = ws.pvalid;
  p.prow = ws.prow;
  p.bias = bias;
  p.reps = reps;
  p.idx = idx;
  p.status = ws.status;

  // The number of units (vocab tiles x groups) is chosen on the device; there
  // are at most num_vtiles * B of them.
  const long long max_units = static_cast<long long>(p.num_vtiles) * B;
  const long long grid_ll = max_units < device_sm_count() ? max_units : device_sm_count();
  const unsigned grid = static_cast<unsigned>(grid_ll > 0 ? grid_ll : 1);
  // Without an idx output (the inference forward) the epilogue keeps the max
  // only and stores reps alone.
  return idx != nullptr ? launch_kernel<T, kFmt, true>(tmW, tmH, p, grid, stream)
                        : launch_kernel<T, kFmt, false>(tmW, tmH, p, grid, stream);
}

}  // namespace

int launch_fwd_tc(int dtype, const void* hidden, const void* weight, const void* bias, int B,
                  int S, int D, int V, void* reps, int32_t* idx, const FwdWorkspace& ws,
                  cudaStream_t stream) {
  if (dtype == SPARTON_DTYPE_BF16)
    return launch_typed<__nv_bfloat16, 1u>(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, hidden, weight, bias, B,
                                           S, D, V, reps, idx, ws, stream);
  if (dtype == SPARTON_DTYPE_F16)
    return launch_typed<__half, 0u>(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hidden, weight, bias, B, S, D,
                                    V, reps, idx, ws, stream);
  return fail(SPARTON_ERR_UNSUPPORTED, "tensor-core forward supports bf16 and f16 only");
}

}  // namespace sparton
