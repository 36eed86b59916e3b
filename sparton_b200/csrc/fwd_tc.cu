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
// vocabulary (128 rows of W per tile, one TMEM lane per vocab id) and N is the
// token dimension (up to 256 positions of one batch row). A thread of the
// epilogue therefore owns one vocab id and scans its own TMEM lane along the
// sequence: the max / argmax over S needs no cross-thread reduction.
//
// Work unit = (vocab tile of 128, batch row b). The unit covers positions
// [0, E_b) in s-tiles of <= 256, where E_b is the last valid position + 1.
// The MMA N of an s-tile is its width rounded up to 16, and the hidden rows
// of one K step arrive in ONE TMA box of exactly that many rows (16 tensor
// maps, boxes of 16, 32, ..., 256 rows), so padded positions cost nothing and
// a stage is two TMA requests. Units go round-robin over the CTAs (CTA i
// takes units i, i + grid, ...). Order: panels of `panel_b` batch rows whose
// hidden states fit in L2; inside a panel, groups of `group_b` rows; inside a
// group, vocab-tile-major. Every role of a CTA walks the same unit sequence,
// so no unit ids pass between them.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0    TMA producer: W tile [128 x 64] + hidden tile [N x 64] per
//             stage, 4 stages, 128-byte swizzle.
//   warp 1    TMEM owner + MMA issuer: tcgen05.mma kind::f16, fp32 accumulator
//             in TMEM, two 256-column accumulators (MMA of the next s-tile
//             overlaps the epilogue of the previous one).
//   Warps 0 and 1 run their loops with all 32 lanes and issue each TMA copy,
//   MMA and commit from one elected lane (ptx.cuh elect_one).
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time (the next chunk's load
//             in flight while one is scanned), masked running max and
//             first-index argmax over positions (strict >, as upstream
//             :150-156), then bias, relu, log1p and the stores of reps / idx.
//             The s-tile's mask words and the unit's bias are fetched before
//             the wait for the accumulator, off the critical path.
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
constexpr int kBN = 256;        // max positions per s-tile = MMA N
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
constexpr int kTileWords = kBN / 32;  // mask words per s-tile
// Batch rows per unit group inside an L2 panel (0: the whole panel).
constexpr int kRowGroup = 0;

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
constexpr int kCtrlBytes = 512;
static_assert(kAbortOffset + 4 <= kCtrlOffset + kCtrlBytes, "control block overflow");
constexpr int kSmemBytes = kCtrlOffset + kCtrlBytes + 1024;  // + alignment slack

struct alignas(64) HiddenMaps {
  CUtensorMap m[kNumHiddenMaps];  // m[i]: boxes of 16 * (i + 1) rows x 64 columns
};

struct FwdTcParams {
  int B, S, D, V;
  int num_vtiles;
  int num_kblocks;
  int panel_b;
  int group_b;
  long long num_units;
  const uint32_t* bits;
  int S32;
  const int* extent;
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

__device__ __forceinline__ void decode_unit(long long j, const FwdTcParams& p, int& vt, int& b) {
  const long long per_panel = static_cast<long long>(p.num_vtiles) * p.panel_b;
  const long long panel = j / per_panel;
  const long long r = j - panel * per_panel;
  const int b0 = static_cast<int>(panel * p.panel_b);
  const int pb = min(p.panel_b, p.B - b0);
  // Row groups of group_b rows (the last may be shorter); every group before
  // the one holding r is full.
  const long long per_group = static_cast<long long>(p.num_vtiles) * p.group_b;
  const int g = static_cast<int>(r / per_group);
  const int rr = static_cast<int>(r - g * per_group);
  const int gb = min(p.group_b, pb - g * p.group_b);
  vt = rr / gb;
  b = b0 + g * p.group_b + rr % gb;
}

// Walks the units of this CTA (blockIdx.x, + gridDim.x, ...). The next unit's
// batch row and extent are fetched one unit ahead, so the dependent global
// load is off the critical path of the role that walks it.
struct UnitIter {
  long long j;
  int vt, b, E;  // current unit
  int nvt, nb, nE;  // next unit (nE = -1: none)
  __device__ __forceinline__ void load_next(const FwdTcParams& p) {
    const long long jn = j + gridDim.x;
    nE = -1;
    if (jn < p.num_units) {
      decode_unit(jn, p, nvt, nb);
      nE = __ldg(p.extent + nb);
    }
  }
  __device__ __forceinline__ bool start(const FwdTcParams& p) {
    j = blockIdx.x;
    if (j >= p.num_units) return false;
    decode_unit(j, p, vt, b);
    E = __ldg(p.extent + b);
    load_next(p);
    return true;
  }
  __device__ __forceinline__ bool advance(const FwdTcParams& p) {
    if (nE < 0) return false;
    j += gridDim.x;
    vt = nvt;
    b = nb;
    E = nE;
    load_next(p);
    return true;
  }
};

struct Ctrl {
  uint32_t bar0;  // shared address of barrier 0
  volatile int* abort_flag;
  __device__ __forceinline__ uint32_t bar(int i) const { return bar0 + 8u * i; }
};

__device__ void run_producer(const FwdTcParams& p, const CUtensorMap* tmW, const CUtensorMap* tmH,
                             uint32_t stage_base, const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t issued_mask = 0, issued_parity = 0;
  bool ok = true;
  UnitIter u;
  for (bool more = u.start(p); more && ok; more = u.advance(p)) {
    const int vt = u.vt, b = u.b, E = u.E;
    for (int s0 = 0; s0 < E && ok; s0 += kBN) {
      const int n16 = (min(kBN, E - s0) + 15) >> 4;  // hidden rows / 16
      const uint32_t bytes = static_cast<uint32_t>(kABytes + n16 * 16 * kRowBytes);
      const CUtensorMap* map = tmH + (n16 - 1);
      const int row0 = b * p.S + s0;
      for (int kb = 0; kb < p.num_kblocks; ++kb) {
        if (!mbar_wait_bounded_warp(c.bar(kBarEmpty + stage), phase ^ 1, c.abort_flag, p.status,
                                    SPARTON_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const uint32_t full = c.bar(kBarFull + stage);
          mbar_arrive_expect_tx(full, bytes);
          const uint32_t a_dst = stage_base + stage * kStageBytes;
          tma_load_2d(a_dst, tmW, full, kb * kBK, vt * kBM);
          tma_load_2d(a_dst + kABytes, map, full, kb * kBK, row0);
        }
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
__device__ void run_mma(const FwdTcParams& p, uint32_t stage_base, uint32_t tmem_base,
                        const Ctrl& c) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t tile = 0;
  bool ok = true;
  bool issued = false;
  UnitIter u;
  for (bool more = u.start(p); more && ok; more = u.advance(p)) {
    const int E = u.E;
    for (int s0 = 0; s0 < E; s0 += kBN) {
      const int acc = tile % kNumAcc;
      const uint32_t aph = (tile / kNumAcc) & 1;
      if (!mbar_wait_bounded_warp(c.bar(kBarTEmpty + acc), aph ^ 1, c.abort_flag, p.status,
                                  SPARTON_DEV_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t n_mma = static_cast<uint32_t>((min(kBN, E - s0) + 15) & ~15);
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

// Folds 32 consecutive positions (one TMEM chunk, mask word `mw`, first
// position `pos0`) into the running masked max / first argmax.
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
  if (cm > best) {
    int first = 31;
#pragma unroll
    for (int q = 31; q >= 0; --q)
      if (((mw >> q) & 1u) && __uint_as_float(r[q]) == cm) first = q;
    best = cm;
    best_idx = pos0 + first;
  }
}

template <typename T>
__device__ void run_epilogue(const FwdTcParams& p, uint32_t tmem_base, const Ctrl& c, int warp,
                             int lane) {
  const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad+32)
  const int row = quad * 32 + lane;
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
  uint32_t tile = 0;
  UnitIter u;
  for (bool more = u.start(p); more; more = u.advance(p)) {
    const int b = u.b, E = u.E;
    const int v = u.vt * kBM + row;
    const uint32_t* bits_row = p.bits + static_cast<size_t>(b) * p.S32;
    const float bias = (p.bias != nullptr && v < p.V)
                           ? to_float<T>(static_cast<const T*>(p.bias)[v])
                           : 0.f;
    float best = -INFINITY;
    int best_idx = 0;
    bool ok = true;
    for (int s0 = 0; s0 < E; s0 += kBN) {
      // Lane i holds mask word i of this s-tile (positions s0 + 32i ...).
      const int w0 = s0 >> 5;
      const uint32_t words =
          (lane < kTileWords && w0 + lane < p.S32) ? __ldg(bits_row + w0 + lane) : 0u;
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
      const int nch = (min(kBN, E - s0) + 31) >> 5;
      const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * kBN);
      uint32_t ra[32], rb[32];
      tmem_ld_32x32b_x32(taddr, ra);
      for (int ch = 0; ch < nch; ch += 2) {
        tmem_ld_wait(ra);
        if (ch + 1 < nch) tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(32 * (ch + 1)), rb);
        scan_chunk(ra, __shfl_sync(0xFFFFFFFFu, words, ch), s0 + 32 * ch, best, best_idx);
        if (ch + 1 < nch) {
          tmem_ld_wait(rb);
          if (ch + 2 < nch) tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(32 * (ch + 2)), ra);
          scan_chunk(rb, __shfl_sync(0xFFFFFFFFu, words, ch + 1), s0 + 32 * (ch + 1), best,
                     best_idx);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(c.bar(kBarTEmpty + acc));
      ++tile;
    }
    if (!ok) break;
    if (v < p.V) {
      // max_s(x_s + bias) = max_s(x_s) + bias: the bias is added once, after the
      // max. Upstream's initial value 0 (:112) is the `logit > 0` test.
      const float logit = best + bias;
      const bool pos = logit > 0.f;
      const size_t o = static_cast<size_t>(b) * p.V + v;
      static_cast<T*>(p.reps)[o] = from_float<T>(pos ? log1pf(logit) : 0.f);
      p.idx[o] = pos ? best_idx : 0;
    }
  }
}

template <typename T, uint32_t kFmt>
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
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    run_producer(p, &tmW, tmH.m, stage_base, c);
    __syncwarp();
  } else if (warp == 1) {
    run_mma<kFmt>(p, stage_base, tmem_base, c);
    __syncwarp();
  } else {
    run_epilogue<T>(p, tmem_base, c, warp, lane);
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
  // Panel of batch rows whose hidden states (S*D*2 bytes each) fit in ~48 MB of L2.
  const long long row_bytes = static_cast<long long>(S) * D * 2;
  long long pb = (48ll << 20) / (row_bytes > 0 ? row_bytes : 1);
  if (pb < 1) pb = 1;
  if (pb > B) pb = B;
  p.panel_b = static_cast<int>(pb);
  p.group_b = (kRowGroup > 0 && kRowGroup < p.panel_b) ? kRowGroup : p.panel_b;
  p.num_units = static_cast<long long>(p.num_vtiles) * B;
  p.bits = ws.bits;
  p.S32 = ws.S32;
  p.extent = ws.extent;
  p.bias = bias;
  p.reps = reps;
  p.idx = idx;
  p.status = ws.status;

  static std::mutex mu;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      e = cudaFuncSetAttribute(fwd_tc_kernel<T, kFmt>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd_tc_kernel)");
      attr_done[dev] = true;
    }
  }
  const long long grid_ll = p.num_units < device_sm_count() ? p.num_units : device_sm_count();
  const unsigned grid = static_cast<unsigned>(grid_ll > 0 ? grid_ll : 1);
  fwd_tc_kernel<T, kFmt><<<grid, kThreads, kSmemBytes, stream>>>(tmW, tmH, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fwd_tc_kernel launch");
  return SPARTON_OK;
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
