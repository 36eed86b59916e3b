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
// with cudaGetSymbolAddress on every call, with the calling device current.
// The lookup is not cached: after a cudaDeviceReset (or any teardown of the
// primary context) the module is loaded again and the array may sit at a
// different address, so a cached pointer could go stale.
#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_fwd_scratch[SPARTON_FWD_NOALLOC_SCRATCH_BYTES];

// Device address of the current device's copy of g_fwd_scratch.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_fwd_scratch);
  if (e != cudaSuccess) return sparton::cuda_fail(e, "cudaGetSymbolAddress(fwd scratch)");
  *out = p;
  return SPARTON_OK;
}

}  // namespace

extern "C" int sparton_fwd_noalloc(const void* hidden, const void* weight, const void* bias,
                                   const void* mask, int mask_dtype, int dtype, int64_t B,
                                   int64_t S, int64_t D, int64_t V, void* reps, int32_t* idx,
                                   void* stream) {
  // The same argument checks as sparton_fwd, before anything touches the
  // device: a bad size or dtype, or a device that is not sm_100, is reported
  // as such rather than as a failed symbol lookup.
  int st = sparton::check_sizes(B, S, D, V);
  if (st != SPARTON_OK) return st;
  st = sparton::check_dtype(dtype);
  if (st != SPARTON_OK) return st;
  const size_t need = sparton::fwd_workspace_bytes(B, S);
  if (need > SPARTON_FWD_NOALLOC_SCRATCH_BYTES)
    return sparton::fail(SPARTON_ERR_UNSUPPORTED,
                         "sparton_fwd_noalloc: B=%lld S=%lld needs %zu bytes of scratch but the "
                         "library's fixed scratch holds %zu; use sparton_fwd with a workspace",
                         (long long)B, (long long)S, need,
                         (size_t)SPARTON_FWD_NOALLOC_SCRATCH_BYTES);
  st = sparton::check_device();
  if (st != SPARTON_OK) return st;
  void* ws = nullptr;
  st = scratch_address(&ws);
  if (st != SPARTON_OK) return st;
  // The forward resets everything in the scratch that must start at zero (the
  // status word) and overwrites the bits / extents it reads.
  return sparton_fwd(hidden, weight, bias, mask, mask_dtype, dtype, B, S, D, V, reps, idx, ws,
                     SPARTON_FWD_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int sparton_fwd_noalloc_status(void* stream, uint32_t* code) {
  if (code == nullptr) return sparton::fail(SPARTON_ERR_INVALID_ARGUMENT, "code is NULL");
  const int st = sparton::check_device();
  if (st != SPARTON_OK) return st;
  void* ws = nullptr;
  const int s2 = scratch_address(&ws);
  if (s2 != SPARTON_OK) return s2;
  return sparton_read_device_status(ws, stream, code);
}
