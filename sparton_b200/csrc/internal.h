// internal.h — declarations shared by the CUDA translation units of the
// library: workspace layouts, launchers and error reporting. Not installed.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stddef.h>
#include <stdint.h>

#include "../../include/sparton_b200.h"

namespace sparton {

// Records a printf-style message as this thread's last error and returns
// `status` so call sites can `return fail(...)`.
int fail(int status, const char* fmt, ...);

// Turns a CUDA error into SPARTON_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t err, const char* what);

// Argument checks shared by the entry points (capi.cu); each records a message
// and returns a status on failure.
int check_sizes(int64_t B, int64_t S, int64_t D, int64_t V);  // head sizes B, S, D, V
int check_dtype(int dtype);                                    // a sparton_dtype value
int check_device();                                            // current device is sm_100

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// 2-D TMA tensor map over a row-major [outer][inner] array with `row_bytes`
// between rows; box = [box_outer][box_inner] elements.
int make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                       uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                       CUtensorMapSwizzle swizzle);

// Number of SMs on the current device (cached per device).
int device_sm_count();

// True when the current device is compute capability 10.x (B200 / sm_100).
bool device_is_sm100();

// ------------------------------------------------------------ forward workspace
// [0,256)      header: u32 status, u32 packed columns in total (T), reserved
// extent       B x int32      last valid position + 1 of each row (0 = empty)
// bits         B x S32 x u32  validity bit of every position, S32 = ceil(S/32)
// Position packing for the tensor-core forward (written by pack_prepare): the
// positions [0, round16(extent)) of all batch rows are laid end to end in one
// stream of T "packed columns", row after row.
// pcol         B x int32      packed column of row b's position 0
// plen         B x int32      packed columns of row b: extent rounded up to 16
// pnz          (B+1) x int32  rows with columns before row b (pnz[B] = count)
// prows        B x int32      the rows with columns, in order
// pvalid       Wmax x u32     validity bit of every packed column
// prow         Wmax x u32     bit set at the first packed column of every row
//              Wmax = ceil(B * round16(S) / 32) + 16 (the tail stays zero)
struct FwdWorkspace {
  unsigned int* status;
  unsigned int* total_cols;
  int* extent;
  uint32_t* bits;
  int S32;
  int* pcol;
  int* plen;
  int* pnz;
  int* prows;
  uint32_t* pvalid;
  uint32_t* prow;
  int64_t wmax;
};

inline int64_t fwd_packed_words(int64_t B, int64_t S) {
  return (B * ((S + 15) / 16 * 16) + 31) / 32 + 16;
}

inline size_t fwd_workspace_bytes(int64_t B, int64_t S) {
  const int64_t S32 = (S + 31) / 32;
  const int64_t W = fwd_packed_words(B, S);
  return 256 + align256(static_cast<size_t>(B) * 4) + align256(static_cast<size_t>(B * S32) * 4) +
         3 * align256(static_cast<size_t>(B) * 4) + align256(static_cast<size_t>(B + 1) * 4) +
         2 * align256(static_cast<size_t>(W) * 4);
}

inline FwdWorkspace fwd_workspace_carve(void* ws, int64_t B, int64_t S) {
  FwdWorkspace w;
  char* base = static_cast<char*>(ws);
  w.status = reinterpret_cast<unsigned int*>(base);
  w.total_cols = reinterpret_cast<unsigned int*>(base) + 1;
  size_t off = 256;
  w.extent = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B) * 4);
  w.bits = reinterpret_cast<uint32_t*>(base + off);
  w.S32 = static_cast<int>((S + 31) / 32);
  off += align256(static_cast<size_t>(B * w.S32) * 4);
  w.pcol = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B) * 4);
  w.plen = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B) * 4);
  w.prows = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B) * 4);
  w.pnz = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B + 1) * 4);
  w.wmax = fwd_packed_words(B, S);
  w.pvalid = reinterpret_cast<uint32_t*>(base + off);
  off += align256(static_cast<size_t>(w.wmax) * 4);
  w.prow = reinterpret_cast<uint32_t*>(base + off);
  return w;
}

// ----------------------------------------------------------- backward workspace
// [0,256)      header: u32 status, u32 next dH row to claim (both zeroed by the
//              sort kernel at the start of every backward)
// offs         B x (S+1) int32   bucket start of every position (CSR by position)
// perm         B x V int32       vocab ids grouped by argmax position
// gperm        B x V float       g' of those entries, same order
// wrow         V x B int32       per vocab id: hidden row b*S + idx[b,v] of every b
// wcoef        V x B float       per vocab id: g' of every b (0 when reps is 0)
// sort_cnt     B x chunks x S int32  per (row, chunk of vocab ids, position):
//              entries, then their prefix over the chunks (the sort's scratch;
//              chunks = ceil(V / bwd_sort_chunk(S)))
struct BwdWorkspace {
  unsigned int* status;
  unsigned int* row_counter;
  int* offs;
  int2* ent;   // [B][V] (v, bits of g') in CSR order by argmax position
  int2* went;  // [V][B] (b*S + idx[b,v], bits of g'), vocab-major
  int* sort_cnt;
};

// Vocab ids per chunk of the backward's sort: 128 per warp, 8 warps unless
// S 16-bit counters per warp plus S int32 bucket bases would exceed 220 KB of
// shared memory (bwd.cu sort_warps).
inline int64_t bwd_sort_chunk(int64_t S) {
  int64_t nw = 8;
  while (nw > 1 && (nw * 2 + 4) * S > 220 * 1024) nw >>= 1;
  return nw * 128;
}

inline size_t bwd_sort_cnt_bytes(int64_t B, int64_t S, int64_t V) {
  const int64_t chunks = (V + bwd_sort_chunk(S) - 1) / bwd_sort_chunk(S);
  return align256(static_cast<size_t>(B * chunks * S) * 4);
}

inline size_t bwd_workspace_bytes(int64_t B, int64_t S, int64_t V) {
  return 256 + align256(static_cast<size_t>(B * (S + 1)) * 4) +
         2 * align256(static_cast<size_t>(B * V) * 8) + bwd_sort_cnt_bytes(B, S, V);
}

inline BwdWorkspace bwd_workspace_carve(void* ws, int64_t B, int64_t S, int64_t V) {
  BwdWorkspace w;
  char* base = static_cast<char*>(ws);
  w.status = reinterpret_cast<unsigned int*>(base);
  w.row_counter = reinterpret_cast<unsigned int*>(base) + 1;
  size_t off = 256;
  w.offs = reinterpret_cast<int*>(base + off);
  off += align256(static_cast<size_t>(B * (S + 1)) * 4);
  w.ent = reinterpret_cast<int2*>(base + off);
  off += align256(static_cast<size_t>(B * V) * 8);
  w.went = reinterpret_cast<int2*>(base + off);
  off += align256(static_cast<size_t>(B * V) * 8);
  w.sort_cnt = reinterpret_cast<int*>(base + off);
  return w;
}

// ------------------------------------------------------------------ launchers
// Each returns SPARTON_OK or a status after recording a message.

int launch_mask_prepare(const void* mask, int mask_dtype, int B, int S, const FwdWorkspace& ws,
                        cudaStream_t stream);

// bf16 / f16: tcgen05 + TMA persistent kernel.
int launch_fwd_tc(int dtype, const void* hidden, const void* weight, const void* bias, int B,
                  int S, int D, int V, void* reps, int32_t* idx, const FwdWorkspace& ws,
                  cudaStream_t stream);

// f32: exact fp32 FMA kernel.
int launch_fwd_f32(const float* hidden, const float* weight, const float* bias, int B, int S,
                   int D, int V, float* reps, int32_t* idx, const FwdWorkspace& ws,
                   cudaStream_t stream);

// Regularisers (reg.cu): workspace of block partials, fused forward / backward.
size_t reg_workspace_bytes(int64_t V);
int launch_reg_fwd(int dtype, const void* reps, int B, int V, float scale_l1, float scale_flops,
                   float* colsum, float* totals, void* workspace, cudaStream_t stream);
int launch_reg_bwd(int dtype, const void* reps, const float* colsum, const float* g_l1,
                   const float* g_flops, float scale_l1, float scale_flops, int B, int V,
                   void* grad, cudaStream_t stream);

// Sparse forms of reps (sparse.cu): CSR of the entries above a threshold and
// the per-row top-k.
struct SparseWorkspace {
  unsigned int* header;       // [0] device status (SPARTON_DEV_*)
  unsigned long long* flags;  // [ceil(B * V / 8192)] the chunks' look-back words (tagged per call)
  size_t bytes;               // header + flags
};
constexpr int kTopkMax = 4096;
size_t sparse_workspace_bytes(int64_t B, int64_t V);
SparseWorkspace sparse_workspace_carve(void* base, int64_t B, int64_t V);
int launch_reps_csr(int dtype, const void* reps, int B, int V, float threshold, int64_t* crow,
                    int32_t* cols, void* vals, int64_t capacity, const SparseWorkspace& ws,
                    cudaStream_t stream);
int launch_reps_topk(int dtype, const void* reps, int B, int V, int k, void* vals, int32_t* idx,
                     cudaStream_t stream);

// Launch of a kernel that depends on the previous work of its stream, with
// programmatic dependent launch (PDL): the launch may begin while the
// predecessor's last CTAs are still running, and the kernel waits for the
// predecessor's results with pdl_wait() (griddepcontrol.wait) before it reads
// them. For short kernels in a chain (sort, CSR, regularisers) this hides the
// launch gap. A kernel that calls pdl_wait() is also correct when launched
// without the attribute (the wait then returns at once).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Device side of launch_pdl: wait until the grids this one depends on have
// completed and their memory operations are visible.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Called at the start of a kernel that has a launch_pdl successor: once every
// CTA of this grid has called it (i.e. the last wave is running), the
// successor may begin launching into the freed slots; it still waits in
// pdl_wait() for this grid to complete before reading its results.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether clusters of P CTAs with `smem` bytes each can be resident, asked once
// per (device, P, smem) of the occupancy API and remembered.
template <typename K>
inline bool cluster_fits(K kernel, const cudaLaunchConfig_t* cfg, int P, size_t smem) {
  struct Entry {
    int dev, P;
    size_t smem;
    bool fits;
  };
  static std::mutex mu;
  static Entry cache[32];
  static int n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].dev == dev && cache[i].P == P && cache[i].smem == smem) return cache[i].fits;
  int clusters = 0;
  const bool fits =
      cudaOccupancyMaxActiveClusters(&clusters, kernel, cfg) == cudaSuccess && clusters >= 1;
  if (!fits) (void)cudaGetLastError();
  cache[n < 32 ? n++ : 31] = Entry{dev, P, smem, fits};
  return fits;
}

// MLM transform, GELU + LayerNorm part (transform.cu).
size_t transform_workspace_bytes(int64_t rows, int64_t D);
int launch_transform_fwd(int dtype, const void* y, const void* gamma, const void* beta, float eps,
                         int rows, int D, void* h, float* mean, float* rstd, cudaStream_t stream);
int launch_transform_bwd(int dtype, const void* dh, const void* y, const void* gamma,
                         const float* mean, const float* rstd, int rows, int D, void* dy,
                         void* d_gamma, void* d_beta, void* d_bias, void* workspace,
                         cudaStream_t stream);

// Plain tensor-core GEMM (gemm_tc.cu): C[M,N] = sum_k A[m,k] B[n,k] (+ bias[n]);
// a_mn / b_mn: the operand is stored MN-major ([K][M] / [K][N]) instead of
// K-major ([M][K] / [N][K]). dtype: bf16 / f16 operands (and bias); c_dtype:
// dtype or F32; lda / ldb: elements per stored row of A / B (>= the operand's
// contiguous extent: K for K-major, M / N for MN-major; padding is read as part
// of the operand and must be zero). The workspace holds a 256-byte header and
// the split partials.
size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
// dst [rows][ld] = src [rows][cols] with zero columns cols..ld-1 (16-bit types).
int launch_pad_rows(int dtype, const void* src, int rows, int cols, void* dst, int ld,
                    cudaStream_t stream);
int launch_gemm(int dtype, int c_dtype, bool a_mn, bool b_mn, const void* A, long long lda,
                const void* B, long long ldb, const void* bias, int M, int N, int K, void* C,
                long long ldc, void* workspace, cudaStream_t stream);

int launch_bwd(int dtype, const void* grad_reps, const void* reps, const int32_t* idx,
               const void* hidden, const void* weight, int B, int S, int D, int V,
               void* d_hidden, void* d_weight, void* d_bias, int d_hidden_dtype,
               int d_param_dtype, const BwdWorkspace& ws, cudaStream_t stream);

}  // namespace sparton
