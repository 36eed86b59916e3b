// gemm_tc.cu — a plain tcgen05 GEMM for the contractions around the head:
//   C[M,N] = sum_k A[m,k] * B[n,k]  (+ bias[n]),  16-bit inputs, fp32 sums.
//
// Upstream computes these with torch (cuBLAS) calls: the dense layer of the MLM
// transform in front of the head and its two backward products
// (hhkbble/sparton training/model.py:25-35: RobertaTransform.dense, BERT's
// predictions.transform.dense, used at :82-85), and the InfoNCE scores
// q_reps @ d_reps.T with their backward (training/train.py:73-77). Here they run
// on the same machinery as the head's forward kernel (fwd_tc.cu): TMA tiles into
// a 4-stage mbarrier ring, one elected thread issuing tcgen05.mma kind::f16 into
// double-buffered TMEM accumulators, four epilogue warps reading TMEM.
//
// Operand layouts. Each operand is dense row-major in memory in one of two ways:
//   "rows" (K-major): A as [M][K], B as [N][K]: the contraction index is
//                     contiguous, as for y = x @ W.T with x [M,K], W [N,K];
//   "cols" (MN-major): A as [K][M], B as [K][N]: the output index is
//                     contiguous, as for dx = dy @ W (B = W [K=N_out][N=K_in])
//                     or dW = dy.T @ x (A = dy [K][M], B = x [K][N]).
// TMA loads either form with 128-byte swizzle: a K-major tile is boxes of
// [64 rows x 64 k] 8 KB apart (one swizzled [rows x 64 k] tile); an MN-major
// tile is boxes of [64 rows (contiguous) x 64 k]
// placed 8 KB apart, which is the canonical MN-major layout the tcgen05 shared
// memory descriptor describes with leading byte offset 8 KB (between 64-element
// MN blocks) and stride byte offset 1 KB (between groups of 8 k).
//
// Work units are (output tile of 128 x 256, split of the K range). With one
// split the epilogue adds the bias and stores C in its dtype; with several
// (few output tiles, long K: the InfoNCE scores, the dense weight's gradient)
// every split stores its fp32 partial tile into the workspace and
// gemm_reduce_kernel adds the splits in a fixed order (deterministic), adds
// the bias and stores C. The split count depends only on the shape.
//
// Every wait is bounded (ptx.cuh); a CTA that gives up records a status code in
// the workspace header, drains its copies and MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>
#include <string.h>

#include "dtype.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace sparton {
namespace {

constexpr int kBM = 128;   // output rows per tile = MMA M = TMEM lanes
constexpr int kBN = 256;   // output columns per tile = max MMA N
constexpr int kBK = 64;    // k per stage: 128-byte rows
constexpr int kMaxStages = 6;  // the ring holds p.stages stages (4, 5 or 6: see plan)
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBoxBytes = 64 * kBK * 2;  // one MN-major box: 64 rows x 64 k
constexpr int kNumAcc = 2;
constexpr int kTmemCols = kNumAcc * kBN;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;

constexpr int kBarFull = 0;
constexpr int kBarEmpty = kBarFull + kMaxStages;
constexpr int kBarTFull = kBarEmpty + kMaxStages;
constexpr int kBarTEmpty = kBarTFull + kNumAcc;
constexpr int kBarDrain = kBarTEmpty + kNumAcc;
constexpr int kNumBars = kBarDrain + 1;
// Stage ring: p.stages stages of kABytes + bn * 128 bytes each in kRingBytes
// (4 x 48 KB at bn = 256, 5 x 40 KB at 192, 6 x 32 KB at 128).
constexpr int kRingBytes = 200 * 1024;
constexpr int kCtrlOffset = kRingBytes;
constexpr int kTmemHolderOffset = kCtrlOffset + kNumBars * 8;
constexpr int kAbortOffset = kTmemHolderOffset + 4;
constexpr int kCtrlBytes = 256;
// Epilogue staging for outputs whose rows are not 16-byte aligned: one 32 x 33
// fp32 tile per epilogue warp, so a row is stored by consecutive lanes.
constexpr int kStageTileOffset = kCtrlOffset + kCtrlBytes;
constexpr int kStageTileBytes = kEpiWarps * 32 * 33 * 4;
// The tile's bias (<= kBN values of the 16-bit type), one copy per epilogue
// warp, fetched before the warp waits for the accumulator.
constexpr int kBiasOffset = kStageTileOffset + kStageTileBytes;
constexpr int kBiasBytes = kEpiWarps * kBN * 2;
constexpr int kSmemBytes = kBiasOffset + kBiasBytes + 1024;

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, splits, kb_per_split;
  int bn;             // output columns per tile: 256, 192 or 128 (a multiple of 64)
  int stages;         // stages in the TMA -> MMA ring
  int stage_bytes;    // kABytes + bn * 128
  long long units;
  const void* bias;   // [N] in the output's element type family (T), or NULL
  void* C;            // [M][ldc] of type O (splits == 1)
  long long ldc;
  float* partial;     // [splits][M][N] fp32 (splits > 1)
  bool vec_store;     // rows of C start on 16-byte boundaries
  bool vec_bias;      // bias starts on a 16-byte boundary
  bool vec_partial;   // N % 4 == 0: partial rows take 16-byte stores
  unsigned int* status;
};

struct Ctrl {
  uint32_t bar0;
  volatile int* abort_flag;
  __device__ __forceinline__ uint32_t bar(int i) const { return bar0 + 8u * i; }
};

struct UnitPos {
  int m0, n0, kb0, kb1, split;
};

__device__ __forceinline__ UnitPos unit_pos(const GemmParams& p, long long u) {
  const long long tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
  UnitPos o;
  o.split = static_cast<int>(u / tiles);
  const int t = static_cast<int>(u - static_cast<long long>(o.split) * tiles);
  o.m0 = (t / p.n_tiles) * kBM;
  o.n0 = (t % p.n_tiles) * p.bn;
  o.kb0 = o.split * p.kb_per_split;
  o.kb1 = min(p.k_blocks, o.kb0 + p.kb_per_split);
  return o;
}

// Loads the A (kAmn: MN-major) and B (kBmn) tiles of k block kb into a stage.
template <bool kAmn, bool kBmn>
__device__ __forceinline__ void load_stage(const CUtensorMap* tmA, const CUtensorMap* tmB,
                                           uint32_t a_dst, uint32_t full, const UnitPos& u,
                                           int kb, int bn) {
  const int k0 = kb * kBK;
  // Both layouts arrive as 64-row (or 64-column) boxes of 8 KB: a K-major box
  // of 64 rows x 64 k is 8 row groups of 1 KB, so consecutive boxes form the
  // same swizzled tile as one tall box, and several boxes keep the copy engine
  // busy in parallel.
#pragma unroll
  for (int i = 0; i < kBM / 64; ++i) {
    if (kAmn)
      tma_load_2d(a_dst + i * kBoxBytes, tmA, full, u.m0 + 64 * i, k0);
    else
      tma_load_2d(a_dst + i * kBoxBytes, tmA, full, k0, u.m0 + 64 * i);
  }
  const uint32_t b_dst = a_dst + kABytes;
#pragma unroll
  for (int i = 0; i < kBN / 64; ++i) {
    if (64 * i < bn) {
      if (kBmn)
        tma_load_2d(b_dst + i * kBoxBytes, tmB, full, u.n0 + 64 * i, k0);
      else
        tma_load_2d(b_dst + i * kBoxBytes, tmB, full, k0, u.n0 + 64 * i);
    }
  }
}

template <bool kAmn, bool kBmn>
__device__ void run_producer(const GemmParams& p, const CUtensorMap* tmA, const CUtensorMap* tmB,
                             uint32_t stage_base, const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t issued_mask = 0, issued_parity = 0;
  bool ok = true;
  for (long long u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
    const UnitPos up = unit_pos(p, u);
    for (int kb = up.kb0; kb < up.kb1; ++kb) {
      if (!mbar_wait_bounded_warp(c.bar(kBarEmpty + stage), phase ^ 1, c.abort_flag, p.status,
                                  SPARTON_DEV_TIMEOUT_PRODUCER)) {
        ok = false;
        break;
      }
      if (elect_one()) {
        const uint32_t full = c.bar(kBarFull + stage);
        // out-of-range parts of a box are zero-filled and counted
        mbar_arrive_expect_tx(full, static_cast<uint32_t>(kABytes + p.bn * kBK * 2));
        load_stage<kAmn, kBmn>(tmA, tmB, stage_base + stage * p.stage_bytes, full, up, kb, p.bn);
      }
      __syncwarp();
      issued_mask |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  for (int s = 0; s < p.stages; ++s) {
    if (!(issued_mask & (1u << s))) continue;
    const uint32_t par = (issued_parity >> s) & 1;
    const uint32_t bar = c.bar((ok ? kBarEmpty : kBarFull) + s);
    if (!mbar_wait_drain(bar, par)) atomicCAS(p.status, 0u, SPARTON_DEV_TIMEOUT_DRAIN);
  }
}

// Shared-memory descriptor of one MMA's operand slice (16 k) at k step kk.
template <bool kMn>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
  if (!kMn) return umma_desc_k_sw128(base + kk * 32);
  // MN-major, 128-byte swizzle: 8-row k groups 1 KB apart (stride byte offset),
  // 64-element MN blocks kBoxBytes apart (leading byte offset); 16 k = 2 KB.
  uint64_t d = umma_desc_k_sw128(base + kk * 2048);
  d &= ~(static_cast<uint64_t>(0x3FFFu) << 16);
  d |= static_cast<uint64_t>(kBoxBytes >> 4) << 16;
  return d;
}

template <uint32_t kFmt, bool kAmn, bool kBmn>
__device__ void run_mma(const GemmParams& p, uint32_t stage_base, uint32_t tmem_base,
                        const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t tile = 0;
  bool ok = true, issued = false;
  for (long long u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
    const UnitPos up = unit_pos(p, u);
    const int acc = tile % kNumAcc;
    const uint32_t aph = (tile / kNumAcc) & 1;
    if (!mbar_wait_bounded_warp(c.bar(kBarTEmpty + acc), aph ^ 1, c.abort_flag, p.status,
                                SPARTON_DEV_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    tc_fence_after_sync();
    const uint32_t n_mma = static_cast<uint32_t>(min(p.bn, (p.N - up.n0 + 15) / 16 * 16));
    const uint32_t idesc = umma_idesc_f16(kFmt, kBM, n_mma) | (kAmn ? (1u << 15) : 0u) |
                           (kBmn ? (1u << 16) : 0u);
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
    for (int kb = up.kb0; kb < up.kb1; ++kb) {
      if (!mbar_wait_bounded_warp(c.bar(kBarFull + stage), phase, c.abort_flag, p.status,
                                  SPARTON_DEV_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      if (elect_one()) {
        const uint32_t a_addr = stage_base + stage * p.stage_bytes;
        const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16(d_tmem, operand_desc<kAmn>(a_addr, kk), operand_desc<kBmn>(b_addr, kk), idesc,
                   (kb > up.kb0 || kk > 0) ? 1u : 0u);
        umma_commit(c.bar(kBarEmpty + stage));
      }
      __syncwarp();
      issued = true;
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
    if (elect_one()) umma_commit(c.bar(kBarTFull + acc));
    __syncwarp();
    ++tile;
  }
  if (!ok && issued) {
    if (elect_one()) umma_commit(c.bar(kBarDrain));
    __syncwarp();
    if (!mbar_wait_drain(c.bar(kBarDrain), 0)) atomicCAS(p.status, 0u, SPARTON_DEV_TIMEOUT_DRAIN);
  }
}

// Stores 32 consecutive outputs of row m starting at column n (n < N).
template <typename O>
__device__ __forceinline__ void store_row_chunk(const GemmParams& p, int m, int n,
                                                const float (&v)[32]) {
  O* dst = static_cast<O*>(p.C) + static_cast<size_t>(m) * p.ldc + n;
  const int cnt = min(32, p.N - n);
  if (p.vec_store && cnt == 32) {
    constexpr int kPer = 16 / sizeof(O);
#pragma unroll
    for (int i = 0; i < 32; i += kPer) {
      uint4 w;
      uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
      if constexpr (sizeof(O) == 4) {
#pragma unroll
        for (int j = 0; j < 4; ++j) wp[j] = __float_as_uint(v[i + j]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) wp[j] = pack2<O>(v[i + 2 * j], v[i + 2 * j + 1]);
      }
      *reinterpret_cast<uint4*>(dst + i) = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < cnt) dst[i] = from_f32<O>(v[i]);
  }
}

// Stores the warp's 32 rows x 32 columns (lane l holds row `l` of the chunk,
// starting at base; rows ld elements apart, 16-byte aligned) through a shared
// tile so that each store instruction writes whole 16-byte segments of a few
// rows (8 rows of 64 bytes for 16-bit O, 4 of 128 for fp32) instead of one
// segment of 32 rows: full sectors and a quarter of the L2 write requests.
// The tile's segments are XOR-swizzled by row (no more than 2-way bank
// conflicts). Warp-collective; rows at or past rows_valid are not written.
template <typename O>
__device__ __forceinline__ void store_chunk_rows(O* base, long long ld, int rows_valid,
                                                 uint8_t* tile, const float (&v)[32], int lane) {
  constexpr int kRowBytes = 32 * static_cast<int>(sizeof(O));
  constexpr int kSeg = kRowBytes / 16;   // 16-byte segments per row
  constexpr int kRowsPer = 32 / kSeg;    // rows per store instruction
  constexpr int kPer = 16 / static_cast<int>(sizeof(O));  // values per segment
#pragma unroll
  for (int sg = 0; sg < kSeg; ++sg) {
    uint4 w;
    uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
    if constexpr (sizeof(O) == 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) wp[j] = __float_as_uint(v[sg * kPer + j]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) wp[j] = pack2<O>(v[sg * kPer + 2 * j], v[sg * kPer + 2 * j + 1]);
    }
    *reinterpret_cast<uint4*>(tile + lane * kRowBytes + 16 * (sg ^ (lane % kSeg))) = w;
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < kSeg; ++q) {
    const int r = q * kRowsPer + lane / kSeg, sg = lane % kSeg;
    const uint4 w = *reinterpret_cast<const uint4*>(tile + r * kRowBytes + 16 * (sg ^ (r % kSeg)));
    if (r < rows_valid)
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(base + r * ld) + 16 * sg) = w;
  }
  __syncwarp();
}

// Stores the warp's 32 rows x 32 columns (lane l holds row m0 + l) through a
// shared tile, one row per step by consecutive lanes: coalesced stores for
// outputs whose rows are not 16-byte aligned (C with an odd row length).
template <typename O>
__device__ __forceinline__ void store_chunk_staged(const GemmParams& p, float* tile, int m0, int n,
                                                   const float (&v)[32], int lane) {
#pragma unroll
  for (int i = 0; i < 32; ++i) tile[lane * 33 + i] = v[i];
  __syncwarp();
  const int cnt = min(32, p.N - n);
  O* base = static_cast<O*>(p.C) + n + lane;
  for (int r = 0; r < 32 && m0 + r < p.M; ++r)
    if (lane < cnt) base[static_cast<size_t>(m0 + r) * p.ldc] = from_f32<O>(tile[r * 33 + lane]);
  __syncwarp();
}

template <typename T, typename O>
__device__ void run_epilogue(const GemmParams& p, uint32_t tmem_base, const Ctrl& c, int warp,
                             int lane, float* stage_tile, T* sbias) {
  const int quad = warp & 3;
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
  const bool has_bias = p.bias != nullptr && p.splits == 1;
  // The bias of unit u's columns, 8 per lane (lane l: columns 8l .. 8l + 7 of
  // the tile; zero past N), fetched one tile ahead so that its load overlaps
  // the wait for the accumulator.
  auto fetch_bias = [&](long long u) -> uint4 {
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if (!has_bias || u >= p.units) return r;
    const int n0 = unit_pos(p, u).n0;
    const int nb = min(p.bn, p.N - n0), j = lane * 8;
    const T* bsrc = static_cast<const T*>(p.bias) + n0 + j;
    if (p.vec_bias && j + 8 <= nb) return __ldg(reinterpret_cast<const uint4*>(bsrc));
    T* e = reinterpret_cast<T*>(&r);
    for (int i = 0; i < 8; ++i)
      if (j + i < nb) e[i] = bsrc[i];
    return r;
  };
  uint4 bias_next = fetch_bias(blockIdx.x);
  uint32_t tile = 0;
  for (long long u = blockIdx.x; u < p.units; u += gridDim.x) {
    const UnitPos up = unit_pos(p, u);
    const int acc = tile % kNumAcc;
    const uint32_t aph = (tile / kNumAcc) & 1;
    const bool got = mbar_wait_bounded(c.bar(kBarTFull + acc), aph, c.abort_flag, p.status,
                                       SPARTON_DEV_TIMEOUT_EPILOGUE);
    if (!__all_sync(0xFFFFFFFFu, got)) break;
    if (has_bias) {
      // this tile's bias into the warp's shared copy, the next tile's on its way
      *reinterpret_cast<uint4*>(sbias + lane * 8) = bias_next;
      __syncwarp();
      bias_next = fetch_bias(u + gridDim.x);
    }
    tc_fence_after_sync();
    const int m = up.m0 + quad * 32 + lane;
    const int nch = (min(p.bn, p.N - up.n0) + 31) >> 5;
    for (int ch = 0; ch < nch; ++ch) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(lane_base + static_cast<uint32_t>(acc * kBN + 32 * ch), r);
      tmem_ld_wait(r);
      const int n = up.n0 + 32 * ch;
      const bool row_ok = m < p.M;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      const int cnt = min(32, p.N - n);
      if (p.splits > 1) {
        // (no early exit: the TMEM load of the next chunk is warp-collective)
        const int m0w = up.m0 + quad * 32;  // the warp's first row
        float* dst = p.partial + (static_cast<size_t>(up.split) * p.M + (row_ok ? m : 0)) * p.N + n;
        if (p.vec_partial && cnt == 32) {
          store_chunk_rows<float>(p.partial + (static_cast<size_t>(up.split) * p.M + m0w) * p.N + n,
                                  p.N, p.M - m0w, reinterpret_cast<uint8_t*>(stage_tile), v, lane);
        } else if (!row_ok) {
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < cnt) dst[i] = v[i];
        }
      } else {
        if (p.bias != nullptr) {
          // shared copy, the same addresses in every lane (broadcast reads)
          const uint4* bp = reinterpret_cast<const uint4*>(sbias + 32 * ch);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w = bp[q];
            const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * q + i] += to_f32<T>(e[i]);
          }
        }
        if (p.vec_store && cnt == 32) {
          const int m0w = up.m0 + quad * 32;
          store_chunk_rows<O>(static_cast<O*>(p.C) + static_cast<size_t>(m0w) * p.ldc + n, p.ldc,
                              p.M - m0w, reinterpret_cast<uint8_t*>(stage_tile), v, lane);
        } else if (p.vec_store) {
          if (row_ok) store_row_chunk<O>(p, m, n, v);
        } else {
          store_chunk_staged<O>(p, stage_tile, up.m0 + quad * 32, n, v, lane);
        }
      }
    }
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(c.bar(kBarTEmpty + acc));
    ++tile;
  }
}

template <typename T, typename O, uint32_t kFmt, bool kAmn, bool kBmn>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t stage_base = smem_addr(smem);
  Ctrl c;
  c.bar0 = stage_base + kCtrlOffset;
  c.abort_flag = reinterpret_cast<volatile int*>(smem + kAbortOffset);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kTmemHolderOffset);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
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
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;
  if (warp == 0) {
    run_producer<kAmn, kBmn>(p, &tmA, &tmB, stage_base, c);
    __syncwarp();
  } else if (warp == 1) {
    run_mma<kFmt, kAmn, kBmn>(p, stage_base, tmem_base, c);
    __syncwarp();
  } else {
    run_epilogue<T, O>(p, tmem_base, c, warp, lane,
                       reinterpret_cast<float*>(smem + kStageTileOffset) + (warp - 2) * 32 * 33,
                       reinterpret_cast<T*>(smem + kBiasOffset) + (warp - 2) * kBN);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// C[m, n] = sum over splits (in order) of partial[s][m][n] (+ bias[n]); the
// loads of eight splits are issued before they are added.
template <typename T, typename O>
__global__ void __launch_bounds__(256) gemm_reduce_kernel(const float* __restrict__ partial,
                                                          int splits, int M, int N,
                                                          const T* __restrict__ bias, O* C,
                                                          long long ldc) {
  pdl_wait();  // the split partials
  const long long total = static_cast<long long>(M) * N;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += 256ll * gridDim.x) {
    float s = 0.f;
    for (int k0 = 0; k0 < splits; k0 += 8) {
      float x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = k0 + j < splits ? __ldcs(partial + (k0 + j) * total + i) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += x[j];
    }
    const int m = static_cast<int>(i / N), n = static_cast<int>(i - static_cast<long long>(m) * N);
    if (bias != nullptr) s += to_f32<T>(bias[n]);
    C[static_cast<size_t>(m) * ldc + n] = from_f32<O>(s);
  }
}

// ----------------------------------------------------------------------- host
// Splits of the K range when the output has few tiles: about one unit per SM
// of a B200 (148; a constant, so the split count and the workspace size depend
// on the shape only), each split at least 4 k blocks.
constexpr long long kTargetUnits = 148;

// Output tile width bn: 256 unless the tiles fill the GPU in several rounds,
// then the width (256, 192 or 128) with the fewest rounds x (bn + 64) (64
// columns' worth of per-tile cost), so that the last round is not mostly idle.
void plan(int M, int N, int K, int& m_tiles, int& n_tiles, int& k_blocks, int& splits,
          int& kb_per, int& bn) {
  m_tiles = (M + kBM - 1) / kBM;
  k_blocks = (K + kBK - 1) / kBK;
  bn = kBN;
  if (static_cast<long long>(m_tiles) * ((N + kBN - 1) / kBN) >= kTargetUnits) {
    long long best = -1;
    for (int w : {256, 192, 128}) {
      const long long t = static_cast<long long>(m_tiles) * ((N + w - 1) / w);
      const long long cost = (t + kTargetUnits - 1) / kTargetUnits * (w + 64);
      if (best < 0 || cost < best) {
        best = cost;
        bn = w;
      }
    }
  }
  n_tiles = (N + bn - 1) / bn;
  const long long tiles = static_cast<long long>(m_tiles) * n_tiles;
  long long s = 1;
  if (2 * tiles <= kTargetUnits && k_blocks >= 8) {
    s = kTargetUnits / tiles;
    s = s < k_blocks / 4 ? s : k_blocks / 4;
    if (s < 1) s = 1;
  }
  kb_per = static_cast<int>((k_blocks + s - 1) / s);
  splits = (k_blocks + kb_per - 1) / kb_per;  // every split has >= 1 k block
}

struct GemmArgs {
  const void* A;
  const void* B;
  long long lda, ldb;  // elements per stored row of A and B (>= their contiguous extent)
  const void* bias;
  int M, N, K;
  void* C;
  long long ldc;
  void* workspace;
};

// K-major: rows of `ld` elements, logical [mn][K], box [box_rows x 64 k];
// MN-major: rows of `ld` elements, logical [K][mn], box [64 k x 64 mn]. The
// map's extent is the stored one (ld), so a padded operand reads its padding.
int make_operand_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, bool mn_major,
                     int mn, int K, long long ld, int box_rows) {
  if (mn_major)
    return make_tensor_map_2d(map, dt, base, static_cast<uint64_t>(ld), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(ld) * 2, 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  return make_tensor_map_2d(map, dt, base, static_cast<uint64_t>(ld), static_cast<uint64_t>(mn),
                            static_cast<uint64_t>(ld) * 2, kBK, static_cast<uint32_t>(box_rows),
                            CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, typename O, uint32_t kFmt, bool kAmn, bool kBmn>
int launch_typed(CUtensorMapDataType dt, const GemmArgs& a, cudaStream_t stream) {
  GemmParams p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  plan(a.M, a.N, a.K, p.m_tiles, p.n_tiles, p.k_blocks, p.splits, p.kb_per_split, p.bn);
  p.units = static_cast<long long>(p.m_tiles) * p.n_tiles * p.splits;
  p.stage_bytes = kABytes + p.bn * kBK * 2;
  p.stages = kRingBytes / p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  p.bias = a.bias;
  p.C = a.C;
  p.ldc = a.ldc;
  p.status = static_cast<unsigned int*>(a.workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + 256);
  p.vec_store = (reinterpret_cast<uintptr_t>(a.C) % 16 == 0) && ((a.ldc * sizeof(O)) % 16 == 0);
  p.vec_bias = reinterpret_cast<uintptr_t>(a.bias) % 16 == 0;
  p.vec_partial = a.N % 4 == 0;
  CUtensorMap tmA, tmB;
  int st = make_operand_map(&tmA, dt, a.A, kAmn, a.M, a.K, a.lda, 64);
  if (st != SPARTON_OK) return st;
  st = make_operand_map(&tmB, dt, a.B, kBmn, a.N, a.K, a.ldb, 64);
  if (st != SPARTON_OK) return st;

  static std::mutex mu;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      e = cudaFuncSetAttribute(gemm_tc_kernel<T, O, kFmt, kAmn, kBmn>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_tc_kernel)");
      attr_done[dev] = true;
    }
  }
  e = cudaMemsetAsync(a.workspace, 0, 256, stream);  // status word
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  const long long sms = device_sm_count();
  const unsigned grid = static_cast<unsigned>(p.units < sms ? p.units : sms);
  gemm_tc_kernel<T, O, kFmt, kAmn, kBmn><<<grid, kThreads, kSmemBytes, stream>>>(tmA, tmB, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_tc_kernel launch");
  if (p.splits > 1) {
    const long long total = static_cast<long long>(a.M) * a.N;
    long long blocks = (total + 255) / 256;
    if (blocks > 4 * sms) blocks = 4 * sms;
    e = launch_pdl(gemm_reduce_kernel<T, O>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                   stream, static_cast<const float*>(p.partial), p.splits, a.M, a.N,
                   static_cast<const T*>(a.bias), static_cast<O*>(a.C), a.ldc);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_reduce_kernel launch");
  }
  return SPARTON_OK;
}

template <typename T, uint32_t kFmt, bool kAmn, bool kBmn>
int launch_out(CUtensorMapDataType dt, int c_dtype, const GemmArgs& a, cudaStream_t s) {
  if (c_dtype == SPARTON_DTYPE_F32) return launch_typed<T, float, kFmt, kAmn, kBmn>(dt, a, s);
  return launch_typed<T, T, kFmt, kAmn, kBmn>(dt, a, s);
}

template <typename T, uint32_t kFmt>
int launch_layouts(CUtensorMapDataType dt, int c_dtype, bool a_mn, bool b_mn, const GemmArgs& a,
                   cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_out<T, kFmt, false, false>(dt, c_dtype, a, s);
  if (!a_mn && b_mn) return launch_out<T, kFmt, false, true>(dt, c_dtype, a, s);
  if (a_mn && !b_mn) return launch_out<T, kFmt, true, false>(dt, c_dtype, a, s);
  return launch_out<T, kFmt, true, true>(dt, c_dtype, a, s);
}

// dst[r][c] = src[r][c] for c < cols, 0 for cols <= c < ld; dst rows (ld
// elements) start on 16-byte boundaries, src rows (cols elements) on 2-byte
// ones. One warp per (row, segment of 2048 columns), 8 destination elements (16
// bytes) per lane and step.
constexpr int kPadSeg = 2048;

template <typename T>
__global__ void __launch_bounds__(256) pad_rows_kernel(const T* __restrict__ src, int rows,
                                                       int cols, T* __restrict__ dst, int ld) {
  const long long warp = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const long long nwarps = (gridDim.x * static_cast<long long>(blockDim.x)) >> 5;
  const int lane = threadIdx.x & 31;
  const int segs = (ld + kPadSeg - 1) / kPadSeg;
  for (long long w = warp; w < static_cast<long long>(rows) * segs; w += nwarps) {
    const int r = static_cast<int>(w / segs), seg = static_cast<int>(w - static_cast<long long>(r) * segs);
    const T* s = src + static_cast<size_t>(r) * cols;
    T* d = dst + static_cast<size_t>(r) * ld;
    const int c_end = min(ld, (seg + 1) * kPadSeg);
    for (int c0 = seg * kPadSeg + lane * 8; c0 < c_end; c0 += 256) {
      T v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = c0 + i < cols ? s[c0 + i] : from_f32<T>(0.f);
      uint4 w4;
      memcpy(&w4, v, 16);
      *reinterpret_cast<uint4*>(d + c0) = w4;
    }
  }
}

}  // namespace

int launch_pad_rows(int dtype, const void* src, int rows, int cols, void* dst, int ld,
                    cudaStream_t stream) {
  const long long need =
      (static_cast<long long>(rows) * ((ld + kPadSeg - 1) / kPadSeg) + 7) / 8;
  const unsigned grid = static_cast<unsigned>(need < 8ll * device_sm_count() ? (need > 0 ? need : 1)
                                                                             : 8 * device_sm_count());
  if (dtype == SPARTON_DTYPE_BF16)
    pad_rows_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(src), rows, cols, static_cast<__nv_bfloat16*>(dst), ld);
  else if (dtype == SPARTON_DTYPE_F16)
    pad_rows_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(src), rows, cols,
                                                     static_cast<__half*>(dst), ld);
  else
    return fail(SPARTON_ERR_UNSUPPORTED, "sparton_pad_rows takes bf16 or f16");
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "pad_rows_kernel launch");
}

size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  int mt, nt, kb, splits, kbp, bn;
  plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), mt, nt, kb, splits, kbp, bn);
  return 256 + (splits > 1 ? static_cast<size_t>(splits) * M * N * 4 : 0);
}

int launch_gemm(int dtype, int c_dtype, bool a_mn, bool b_mn, const void* A, long long lda,
                const void* B, long long ldb, const void* bias, int M, int N, int K, void* C,
                long long ldc, void* workspace, cudaStream_t stream) {
  const GemmArgs a{A, B, lda, ldb, bias, M, N, K, C, ldc, workspace};
  if (dtype == SPARTON_DTYPE_BF16)
    return launch_layouts<__nv_bfloat16, 1u>(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, c_dtype, a_mn, b_mn,
                                             a, stream);
  if (dtype == SPARTON_DTYPE_F16)
    return launch_layouts<__half, 0u>(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, c_dtype, a_mn, b_mn, a,
                                      stream);
  return fail(SPARTON_ERR_UNSUPPORTED, "the tensor-core GEMM takes bf16 or f16 operands");
}

}  // namespace sparton
