// peer_reduce.cu — the sum over a vocabulary-sharded group of every rank's
// partial d_hidden, over NVLink peer memory, restricted to the rows that can
// be nonzero.
//
// In a vocabulary-sharded head (north_star: each GPU owns rows of the decoder)
// every rank's backward produces a partial d_hidden[B,S,D] (fp32), and the
// gradient is their sum. Only positions before each row's extent can receive
// gradient; the rest of d_hidden is zero on every rank. The forward's
// workspace already lays those positions out as T packed columns (pcol[b],
// plen[b] = round16(extent[b]); mask.cu), identically on every rank, but T
// lives on the device, and a library collective (NCCL) needs its count on the
// host. These kernels read T on the device and move only the packed rows:
//
//   signal (part ready)  each rank tells every peer, by a flag in the peer's
//                        memory, that its partial is complete (stream order:
//                        after the backward's d_hidden gather);
//   reduce               rank q owns packed rows [T q / N, T (q+1) / N): it
//                        waits for every peer's flag, loads those rows of every
//                        rank's partial (peer loads over NVLink, its own
//                        locally), adds them in rank order in fp32, rounds once
//                        to the output dtype and stores them in its `red`
//                        buffer (a reduce-scatter);
//   signal (red ready)   each rank tells every peer its rows are reduced;
//   gather               every rank waits for every peer's flag and copies
//                        each packed row from its owner's `red` buffer into its
//                        own d_hidden [B,S,D], writing zeros at the positions
//                        past the packed rows (an all-gather).
//
// The peer buffers (partials, reduced rows, flags) are mapped into every rank
// by CUDA IPC; their device addresses arrive here as plain pointers. Flags
// carry a step number (epoch) and are written with release and read with
// acquire semantics at system scope, after a system-scope fence. Every wait
// is bounded (kPeerWaitNs); a wait that gives up records
// SPARTON_DEV_TIMEOUT_PEER in the status word and the kernel returns.
// Nothing here uses multicast memory or TMA.
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "dtype.cuh"
#include "internal.h"
#include "ptx.cuh"

#include <string.h>

namespace sparton {
namespace {

constexpr int kMaxPeers = 8;
constexpr uint64_t kPeerWaitNs = 10000000000ull;  // 10 s: peers may be a step behind

struct PeerPtrs {
  const float* part[kMaxPeers];  // [B*S][D] fp32 partial d_hidden of each rank
  void* red[kMaxPeers];          // [B*S][D] reduced rows (output dtype) of each rank
  unsigned int* flags[kMaxPeers];  // [2][kMaxPeers] u32 of each rank
};

struct ReduceParams {
  int rank, world;
  unsigned int epoch;
  int B, S, D;
  const unsigned int* total_cols;  // T, from the forward's workspace
  const int* pcol;
  const int* plen;
  void* out;                       // local d_hidden [B*S][D] (gather phase)
  unsigned int* status;
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 16 bytes from (possibly) another GPU's memory, not cached in L1: the data
// was written by that GPU after this kernel may have started.
__device__ __forceinline__ float4 ld_peer_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cv.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_peer_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cv.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Thread 0 of the CTA waits until every rank's flag `slot` holds `epoch`; the
// CTA then proceeds (true) or, after a timeout, returns false everywhere.
__device__ bool wait_peers(const ReduceParams& p, const unsigned int* my_flags, int slot) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = global_timer_ns();
    for (int r = 0; r < p.world; ++r) {
      while (ld_acquire_sys(my_flags + slot * kMaxPeers + r) != p.epoch) {
        if (global_timer_ns() - t0 > kPeerWaitNs) {
          atomicCAS(p.status, 0u, SPARTON_DEV_TIMEOUT_PEER);
          ok = 0;
          break;
        }
        __nanosleep(256);
      }
      if (!ok) break;
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void peer_signal_kernel(const PeerPtrs ptrs, int rank, int world, int slot,
                                   unsigned int epoch) {
  // Everything this rank wrote before this launch (stream order) becomes
  // visible to the peers before they can see the flag.
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < world) st_release_sys(ptrs.flags[r] + slot * kMaxPeers + rank, epoch);
}

// Packed row i -> (batch row b, position s): b = last row with pcol[b] <= i.
__device__ __forceinline__ int packed_row(const ReduceParams& p, int i, int& s) {
  int lo = 0, hi = p.B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.pcol + mid) <= i) lo = mid; else hi = mid - 1;
  }
  s = i - __ldg(p.pcol + lo);
  return lo;
}

// Reduce-scatter: one warp per owned packed row; each lane owns 4 columns of
// a 128-column chunk, and the chunk's loads from every rank are issued before
// any is added (up to kMaxPeers x 2 chunks of 16 bytes in flight per lane).
template <typename O>
__device__ __forceinline__ void store4(O* dst, const float4& a) {
  if constexpr (sizeof(O) == 4) {
    *reinterpret_cast<float4*>(dst) = a;
  } else {
    uint2 w;
    w.x = pack2<O>(a.x, a.y);
    w.y = pack2<O>(a.z, a.w);
    *reinterpret_cast<uint2*>(dst) = w;
  }
}

template <typename O>
__global__ void __launch_bounds__(256) peer_reduce_kernel(const PeerPtrs ptrs, const ReduceParams p) {
  if (!wait_peers(p, ptrs.flags[p.rank], 0)) return;
  const int T = static_cast<int>(*p.total_cols);
  const int i0 = static_cast<int>(static_cast<long long>(T) * p.rank / p.world);
  const int i1 = static_cast<int>(static_cast<long long>(T) * (p.rank + 1) / p.world);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  O* red = static_cast<O*>(ptrs.red[p.rank]);
  for (int i = i0 + warp; i < i1; i += nwarps) {
    int s;
    const int b = packed_row(p, i, s);
    if (s >= p.S) continue;  // the round-up of a row whose extent is not a multiple of 16
    const size_t row = static_cast<size_t>(b) * p.S + s;
    for (int d0 = lane * 4; d0 < p.D; d0 += 256) {
      const int d1 = d0 + 128;
      const bool two = d1 < p.D;
      float4 v0[kMaxPeers], v1[kMaxPeers];
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) {
        if (r < p.world) {
          const float* src = ptrs.part[r] + row * p.D;
          v0[r] = ld_peer_f4(src + d0);
          v1[r] = two ? ld_peer_f4(src + d1) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) {  // rank order: deterministic sums
        if (r < p.world) {
          a0.x += v0[r].x; a0.y += v0[r].y; a0.z += v0[r].z; a0.w += v0[r].w;
          a1.x += v1[r].x; a1.y += v1[r].y; a1.z += v1[r].z; a1.w += v1[r].w;
        }
      }
      store4<O>(red + row * p.D + d0, a0);
      if (two) store4<O>(red + row * p.D + d1, a1);
    }
  }
}

// Owner of packed row i: q with floor(T q / N) <= i < floor(T (q+1) / N).
__device__ __forceinline__ int row_owner(int i, int T, int world) {
  int q = static_cast<int>(static_cast<long long>(i) * world / (T > 0 ? T : 1));
  if (q >= world) q = world - 1;
  while (q > 0 && static_cast<long long>(T) * q / world > i) --q;
  while (q + 1 < world && static_cast<long long>(T) * (q + 1) / world <= i) ++q;
  return q;
}

// All-gather: one warp per row of d_hidden; packed rows come from their
// owner's reduced rows (four 16-byte loads in flight per lane), the rest is
// zero.
template <typename O>
__global__ void __launch_bounds__(256) peer_gather_kernel(const PeerPtrs ptrs, const ReduceParams p) {
  if (!wait_peers(p, ptrs.flags[p.rank], 1)) return;
  const int T = static_cast<int>(*p.total_cols);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(p.B) * p.S;
  constexpr int kPer = 16 / sizeof(O);  // elements per 16-byte chunk
  O* out = static_cast<O*>(p.out);
  for (long long row = warp; row < rows; row += nwarps) {
    const int b = static_cast<int>(row / p.S);
    const int s = static_cast<int>(row - static_cast<long long>(b) * p.S);
    const bool packed = s < __ldg(p.plen + b);
    const int owner = packed ? row_owner(__ldg(p.pcol + b) + s, T, p.world) : 0;
    const O* src = static_cast<const O*>(ptrs.red[owner]) + row * p.D;
    O* dst = out + row * p.D;
    for (int d0 = lane * kPer; d0 < p.D; d0 += 4 * 32 * kPer) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = d0 + u * 32 * kPer;
        v[u] = (packed && d < p.D) ? ld_peer_u4(src + d) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = d0 + u * 32 * kPer;
        if (d < p.D) *reinterpret_cast<uint4*>(dst + d) = v[u];
      }
    }
  }
}

template <typename O>
int launch_typed(const PeerPtrs& ptrs, const ReduceParams& p, cudaStream_t stream) {
  peer_signal_kernel<<<1, 32, 0, stream>>>(ptrs, p.rank, p.world, 0, p.epoch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_signal_kernel launch");
  const unsigned grid = static_cast<unsigned>(device_sm_count() * 2);
  peer_reduce_kernel<O><<<grid, 256, 0, stream>>>(ptrs, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_reduce_kernel launch");
  peer_signal_kernel<<<1, 32, 0, stream>>>(ptrs, p.rank, p.world, 1, p.epoch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_signal_kernel launch");
  peer_gather_kernel<O><<<grid, 256, 0, stream>>>(ptrs, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_gather_kernel launch");
  return SPARTON_OK;
}

}  // namespace
}  // namespace sparton

using namespace sparton;

extern "C" int sparton_hidden_allreduce(void* const* parts, void* const* reds,
                                        uint32_t* const* flags, int rank, int world,
                                        uint32_t epoch, const void* fwd_workspace, int64_t B,
                                        int64_t S, int64_t D, void* d_hidden, int out_dtype,
                                        uint32_t* status, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "rank %d / world %d (1 <= world <= %d)", rank,
                world, kMaxPeers);
  if (epoch == 0) return fail(SPARTON_ERR_INVALID_ARGUMENT, "epoch must be > 0");
  if (B < 1 || S < 1 || D < 4 || D % 8 != 0 || B * S > (1ll << 31) - 1)
    return fail(SPARTON_ERR_UNSUPPORTED, "sizes out of range (B=%lld S=%lld D=%lld)",
                (long long)B, (long long)S, (long long)D);
  if (out_dtype != SPARTON_DTYPE_BF16 && out_dtype != SPARTON_DTYPE_F16 &&
      out_dtype != SPARTON_DTYPE_F32)
    return fail(SPARTON_ERR_UNSUPPORTED, "unknown output dtype %d", out_dtype);
  if (parts == nullptr || reds == nullptr || flags == nullptr || fwd_workspace == nullptr ||
      d_hidden == nullptr || status == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  PeerPtrs ptrs = {};
  for (int r = 0; r < world; ++r) {
    if (parts[r] == nullptr || reds[r] == nullptr || flags[r] == nullptr)
      return fail(SPARTON_ERR_INVALID_ARGUMENT, "peer buffers of rank %d are NULL", r);
    if ((reinterpret_cast<uintptr_t>(parts[r]) | reinterpret_cast<uintptr_t>(reds[r])) & 15)
      return fail(SPARTON_ERR_INVALID_ARGUMENT, "peer buffers must be 16-byte aligned");
    ptrs.part[r] = static_cast<const float*>(parts[r]);
    ptrs.red[r] = reds[r];
    ptrs.flags[r] = flags[r];
  }
  if (reinterpret_cast<uintptr_t>(d_hidden) & 15)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "d_hidden must be 16-byte aligned");
  const int st = check_device();
  if (st != SPARTON_OK) return st;
  const FwdWorkspace fw = fwd_workspace_carve(const_cast<void*>(fwd_workspace), B, S);
  ReduceParams p;
  p.rank = rank;
  p.world = world;
  p.epoch = epoch;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.D = static_cast<int>(D);
  p.total_cols = fw.total_cols;
  p.pcol = fw.pcol;
  p.plen = fw.plen;
  p.out = d_hidden;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (out_dtype == SPARTON_DTYPE_BF16) return launch_typed<__nv_bfloat16>(ptrs, p, s);
  if (out_dtype == SPARTON_DTYPE_F16) return launch_typed<__half>(ptrs, p, s);
  return launch_typed<float>(ptrs, p, s);
}

// --------------------------------------------------------------- CUDA IPC
namespace {
PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 3020, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  });
  return fn;
}
}  // namespace

extern "C" int sparton_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  auto range = address_range_fn();
  if (range == nullptr) return fail(SPARTON_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return fail(SPARTON_ERR_CUDA, "cuMemGetAddressRange failed (CUresult %d)", static_cast<int>(r));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uint64_t>(ptr) - static_cast<uint64_t>(base);
  return SPARTON_OK;
}

extern "C" int sparton_ipc_open(const void* handle, uint64_t offset, void** ptr) {
  if (handle == nullptr || ptr == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<char*>(base) + offset;
  return SPARTON_OK;
}

extern "C" int sparton_ipc_close(void* ptr, uint64_t offset) {
  if (ptr == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "ptr is NULL");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return SPARTON_OK;
}
