// fwd_noalloc.cu — sparton_fwd_noalloc: the forward for callers that cannot
// allocate device memory.
//
// sparton_fwd needs a small scratch buffer from its caller (per-row validity
// bits, row extents and the status word). Some
// callers cannot provide one at the point where they run the head: a Go or Java
// service that binds this C ABI through cgo / JNI and has no CUDA allocator of
// its own; a serving process whose framework has already reserved (nearly) all
// device memory for its own pool, so a cudaMalloc would fail; or a latency
// sensitive loop that must not call cudaMalloc, which can synchronise the whole
// device. For them, this entry point keeps the scratch in a fixed array
// compiled into the library and allocates nothing.
//
// The array (SPARTON_FWD_NOALLOC_SCRATCH_BYTES) lives in a file-scope
// __device__ variable: every GPU that loads the library holds one copy until
// the process exits. Host code must not pass the variable's name to a kernel
// (on the host it is only a stand-in symbol); its device address is looked up
// with cudaGetSymbolAddress the first time the entry point runs on a device,
// with that device current, and cached per device.
#include <mutex>

#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_fwd_scratch[SPARTON_FWD_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of this device's copy of g_fwd_scratch (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sparton::cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64)
    return sparton::fail(SPARTON_ERR_DEVICE, "sparton_fwd_noalloc supports device ordinals < 64");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fwd_scratch);
    if (e != cudaSuccess) return sparton::cuda_fail(e, "cudaGetSymbolAddress(fwd scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return SPARTON_OK;
}

}  // namespace

extern "C" int sparton_fwd_noalloc(const void* hidden, const void* weight, const void* bias,
                                   const void* mask, int mask_dtype, int dtype, int64_t B,
                                   int64_t S, int64_t D, int64_t V, void* reps, int32_t* idx,
                                   void* stream) {
  if (B < 0 || S < 0 || D < 0 || V < 0)
    return sparton::fail(SPARTON_ERR_INVALID_ARGUMENT, "negative size (B=%lld S=%lld D=%lld V=%lld)",
                         (long long)B, (long long)S, (long long)D, (long long)V);
  if (B > (1ll << 24) || S > (1ll << 24))
    return sparton::fail(SPARTON_ERR_UNSUPPORTED, "sizes out of range (B=%lld S=%lld)",
                         (long long)B, (long long)S);
  const size_t need = sparton::fwd_workspace_bytes(B, S);
  if (need > SPARTON_FWD_NOALLOC_SCRATCH_BYTES)
    return sparton::fail(SPARTON_ERR_UNSUPPORTED,
                         "sparton_fwd_noalloc: B=%lld S=%lld needs %zu bytes of scratch but the "
                         "library's fixed scratch holds %zu; use sparton_fwd with a workspace",
                         (long long)B, (long long)S, need,
                         (size_t)SPARTON_FWD_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  const int st = scratch_address(&ws);
  if (st != SPARTON_OK) return st;
  // The forward resets everything in the scratch that must start at zero (the
  // status word) and overwrites the bits / extents it reads.
  return sparton_fwd(hidden, weight, bias, mask, mask_dtype, dtype, B, S, D, V, reps, idx, ws,
                     SPARTON_FWD_NOALLOC_SCRATCH_BYTES, stream);
}
