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
// round16(extent[b]) packed columns, consecutive rows follow each other, and
// the stream is cut into groups of whole rows by the packed column at which
// each row starts (group = start / group_cols). Per group it writes the
// validity bit of every packed column and a bit at each row's first column.
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

// Group of the row whose packed columns start at global offset `start`.
__device__ __forceinline__ int group_of_start(int start, int group_cols) { return start / group_cols; }

// Last group g with gstart[g] <= b (groups are never empty).
__device__ __forceinline__ int find_group(const int* gstart, int G, int b) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (gstart[mid] <= b) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kPackThreads)
    pack_prepare_kernel(int B, int S32, int group_cols, const int* __restrict__ extent,
                        const uint32_t* __restrict__ bits, int* pcol, int* plen, int* gstart,
                        int* gcols, int* gword, int* prows, int* gnz, uint32_t* pvalid,
                        uint32_t* prow, unsigned int* num_groups) {
  __shared__ int sh[kPackThreads / 32 + 1];
  const int tid = threadIdx.x;
  // 1. packed length of every row and its global start (exclusive prefix).
  int carry = 0;
  for (int base = 0; base < B; base += kPackThreads) {
    const int b = base + tid;
    const int len = b < B ? ((extent[b] + 15) & ~15) : 0;
    int tot = 0;
    const int ex = block_scan_excl(len, sh, &tot);
    if (b < B) {
      plen[b] = len;
      pcol[b] = carry + ex;
    }
    carry += tot;
  }
  const int total = carry;
  __syncthreads();
  // 2. group starts. A row is at most group_cols long, so consecutive rows'
  // groups differ by at most 1 and no group is empty.
  const int G = B > 0 ? group_of_start(pcol[B - 1], group_cols) + 1 : 0;
  for (int b = tid; b < B; b += kPackThreads) {
    const int g = group_of_start(pcol[b], group_cols);
    const int gp = b > 0 ? group_of_start(pcol[b - 1], group_cols) : -1;
    if (g != gp) gstart[g] = b;
  }
  if (tid == 0) {
    gstart[G] = B;
    *num_groups = static_cast<unsigned int>(G);
  }
  __syncthreads();
  // 3. columns of each group; its global start parked in gword for step 4.
  for (int g = tid; g < G; g += kPackThreads) {
    const int p0 = pcol[gstart[g]];
    const int p1 = gstart[g + 1] < B ? pcol[gstart[g + 1]] : total;
    gcols[g] = p1 - p0;
    gword[g] = p0;
  }
  __syncthreads();
  // 4. row start relative to its group.
  for (int b = tid; b < B; b += kPackThreads) {
    const int start = pcol[b];
    pcol[b] = start - gword[group_of_start(start, group_cols)];
  }
  __syncthreads();
  // 5. first bitmap word of each group (groups padded to whole 256-column tiles).
  carry = 0;
  for (int base = 0; base < G; base += kPackThreads) {
    const int g = base + tid;
    const int w = g < G ? (gcols[g] + 255) / 256 * 8 : 0;
    int tot = 0;
    const int ex = block_scan_excl(w, sh, &tot);
    if (g < G) gword[g] = carry + ex;
    carry += tot;
  }
  const int words = carry;
  if (tid == 0) gword[G] = words;
  for (int i = tid; i < words; i += kPackThreads) {
    pvalid[i] = 0u;
    prow[i] = 0u;
  }
  __syncthreads();
  // 6. the rows with columns, in order, and where each group's start in that list.
  carry = 0;
  for (int base = 0; base < B; base += kPackThreads) {
    const int b = base + tid;
    const int nz = (b < B && plen[b] > 0) ? 1 : 0;
    int tot = 0;
    const int ex = block_scan_excl(nz, sh, &tot);
    if (nz) prows[carry + ex] = b;
    if (b < B) {
      const int g = find_group(gstart, G, b);
      if (gstart[g] == b) gnz[g] = carry + ex;
    }
    carry += tot;
  }
  if (tid == 0) gnz[G] = carry;
  // 7. bits of every row, 16 packed columns at a time (row starts and lengths
  // are multiples of 16, so a word holds pieces of at most two rows).
  for (int b = tid; b < B; b += kPackThreads) {
    const int len = plen[b];
    if (len == 0) continue;
    const int g = find_group(gstart, G, b);
    const int c0 = pcol[b], w0 = gword[g];
    const uint32_t* brow = bits + static_cast<size_t>(b) * S32;
    for (int x = 0; x < len; x += 16) {
      const int col = c0 + x;
      const int word = w0 + (col >> 5), shift = col & 31;
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
  pack_prepare_kernel<<<1, kPackThreads, 0, stream>>>(
      B, ws.S32, static_cast<int>(fwd_group_cols(S)), ws.extent, ws.bits, ws.pcol, ws.plen,
      ws.gstart, ws.gcols, ws.gword, ws.prows, ws.gnz, ws.pvalid, ws.prow, ws.num_groups);
  e = cudaGetLastError();
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
