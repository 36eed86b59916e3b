// mask.cu — reduces the attention mask [B,S] to what the forward kernels use:
// one validity bit per position (32 positions per word) and the extent of each
// row (last valid position + 1). Upstream multiplies every logit by the mask
// value inside its reduce kernel (hhkbble/sparton
// src/sparton/sparton_kernel.py:140-148); a position with mask 0 then holds 0,
// which never beats the running max's initial value 0 (:112-113, :154). Here a
// zero mask entry excludes the position, which is the same result for 0/1
// masks, and the extent lets the GEMM skip the padded tail entirely.
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

template <typename M>
int launch_typed(const void* mask, int B, int S, const FwdWorkspace& ws, cudaStream_t stream) {
  mask_prepare_kernel<M><<<B, 256, 0, stream>>>(static_cast<const M*>(mask), S, ws.S32, ws.bits,
                                                ws.extent, ws.status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "mask_prepare_kernel launch");
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
