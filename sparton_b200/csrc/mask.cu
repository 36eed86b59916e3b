// mask.cu — reduces the attention mask [B,S] to what the forward kernels use:
// one validity bit per position (32 positions per word) and the extent of each
// row (last valid position + 1). Upstream multiplies every logit by the mask
// value inside its reduce kernel (hhkbble/sparton
// src/sparton/sparton_kernel.py:140-148); a position with mask 0 then holds 0,
// which never beats the running max's initial value 0 (:112-113, :154). Here a
// zero mask entry excludes the position, which is the same result for 0/1
// masks, and the extent lets the GEMM skip the padded tail entirely.
//
// pack_prepare_kernel then lays the rows' positions end to end for the
// tensor-core forward (workspace layout in internal.h): row b takes
// round16(extent[b]) packed columns and consecutive rows follow each other. It
// writes the validity bit of every packed column and a bit at each row's first
// column, and the list of rows that have columns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace sparton {
namespace {

template <typename M>
__device__ __forceinline__ bool is_valid(M m) {
  return m != M(0);
}
template <>
__device__ __forceinline__ bool is_valid<__half>(__half m) {
  return __half2float(m) != 0.f;
}
template <>
__device__ __forceinline__ bool is_valid<__nv_bfloat16>(__nv_bfloat16 m) {
  return __bfloat162float(m) != 0.f;
}

// One block per batch row. Also resets the workspace header (the status word
// and the reserved words after it) so the main kernel starts clean.
template <typename M>
__global__ void __launch_bounds__(256) mask_prepare_kernel(const M* __restrict__ mask, int S, int S32,
                                                           uint32_t* __restrict__ bits,
                                                           int* __restrict__ extent,
                                                           unsigned int* header) {
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (b == 0 && threadIdx.x < 3) header[threadIdx.x] = 0u;
  const M* row = mask + static_cast<size_t>(b) * S;
  int last = 0;
  for (int w = warp; w < S32; w += blockDim.x >> 5) {
    const int s = w * 32 + lane;
    const bool valid = s < S && is_valid<M>(row[s]);
    const uint32_t word = __ballot_sync(0xFFFFFFFFu, valid);
    if (lane == 0) bits[static_cast<size_t>(b) * S32 + w] = word;
    if (word != 0u) last = max(last, w * 32 + 32 - __clz(word));
  }
  __shared__ int red[8];
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xFFFFFFFFu, last, o));
  if (lane == 0) red[warp] = last;
  __syncthreads();
  if (threadIdx.x == 0) {
    int m = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = max(m, red[i]);
    extent[b] = m;
  }
}

constexpr int kPackThreads = 1024;

// Exclusive prefix of x over the block (kPackThreads threads); *total gets the
// block sum. `sh` holds kPackThreads / 32 + 1 ints.
__device__ __forceinline__ int block_scan_excl(int x, int* sh, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = x;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sh[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kPackThreads / 32 ? sh[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    sh[lane] = t;  // inclusive warp totals
  }
  __syncthreads();
  const int excl = incl - x + (warp > 0 ? sh[warp - 1] : 0);
  *total = sh[kPackThreads / 32 - 1];
  __syncthreads();
  return excl;
}

__global__ void __launch_bounds__(kPackThreads)
    pack_prepare_kernel(int B, int S32, const int* __restrict__ extent,
                        const uint32_t* __restrict__ bits, int* pcol, int* plen, int* pnz,
                        int* prows, uint32_t* pvalid, uint32_t* prow, unsigned int* total_cols) {
  __shared__ int sh[kPackThreads / 32 + 1];
  const int tid = threadIdx.x;
  pdl_wait();  // extents and bits of mask_prepare_kernel
  pdl_trigger();
  // 1. packed length and start of every row; the rows with columns, in order.
  int carry = 0, carry_nz = 0;
  for (int base = 0; base < B; base += kPackThreads) {
    const int b = base + tid;
    const int len = b < B ? ((extent[b] + 15) & ~15) : 0;
    int tot = 0, tot_nz = 0;
    const int ex = block_scan_excl(len, sh, &tot);
    const int ex_nz = block_scan_excl(len > 0 ? 1 : 0, sh, &tot_nz);
    if (b < B) {
      plen[b] = len;
      pcol[b] = carry + ex;
      pnz[b] = carry_nz + ex_nz;
      if (len > 0) prows[carry_nz + ex_nz] = b;
    }
    carry += tot;
    carry_nz += tot_nz;
  }
  const int total = carry;
  if (tid == 0) {
    pnz[B] = carry_nz;
    *total_cols = static_cast<unsigned int>(total);
  }
  // 2. clear the bitmaps (with the zero tail that the forward's reads may touch).
  const int words = (total + 31) / 32 + 16;
  for (int i = tid; i < words; i += kPackThreads) {
    pvalid[i] = 0u;
    prow[i] = 0u;
  }
  __syncthreads();
  // 3. bits of every row, 16 packed columns at a time (row starts and lengths
  // are multiples of 16, so a word holds pieces of at most two rows).
  for (int b = tid; b < B; b += kPackThreads) {
    const int len = plen[b];
    if (len == 0) continue;
    const int c0 = pcol[b];
    const uint32_t* brow = bits + static_cast<size_t>(b) * S32;
    for (int x = 0; x < len; x += 16) {
      const int col = c0 + x;
      const int word = col >> 5, shift = col & 31;
      const uint32_t v16 = (__ldg(brow + (x >> 5)) >> (x & 31)) & 0xFFFFu;
      if (v16 != 0u) atomicOr(pvalid + word, v16 << shift);
      if (x == 0) atomicOr(prow + word, 1u << shift);
    }
  }
}

template <typename M>
int launch_typed(const void* mask, int B, int S, const FwdWorkspace& ws, cudaStream_t stream) {
  mask_prepare_kernel<M><<<B, 256, 0, stream>>>(static_cast<const M*>(mask), S, ws.S32, ws.bits,
                                                ws.extent, ws.status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "mask_prepare_kernel launch");
  e = launch_pdl(pack_prepare_kernel, dim3(1), dim3(kPackThreads), 0, stream, B, ws.S32,
                 static_cast<const int*>(ws.extent), static_cast<const uint32_t*>(ws.bits),
                 ws.pcol, ws.plen, ws.pnz, ws.prows, ws.pvalid, ws.prow, ws.total_cols);
  if (e != cudaSuccess) return cuda_fail(e, "pack_prepare_kernel launch");
  return SPARTON_OK;
}

}  // namespace

int launch_mask_prepare(const void* mask, int mask_dtype, int B, int S, const FwdWorkspace& ws,
                        cudaStream_t stream) {
  switch (mask_dtype) {
    case SPARTON_MASK_U8:
      return launch_typed<uint8_t>(mask, B, S, ws, stream);
    case SPARTON_MASK_I32:
      return launch_typed<int32_t>(mask, B, S, ws, stream);
    case SPARTON_MASK_I64:
      return launch_typed<long long>(mask, B, S, ws, stream);
    case SPARTON_MASK_F32:
      return launch_typed<float>(mask, B, S, ws, stream);
    case SPARTON_MASK_F16:
      return launch_typed<__half>(mask, B, S, ws, stream);
    case SPARTON_MASK_BF16:
      return launch_typed<__nv_bfloat16>(mask, B, S, ws, stream);
    default:
      return fail(SPARTON_ERR_UNSUPPORTED, "unknown mask dtype %d", mask_dtype);
  }
}

}  // namespace sparton
