// capi.cu — the extern "C" boundary declared in include/sparton_b200.h.
// Validates every argument before anything is launched (upstream relies on
// Python asserts: hhkbble/sparton src/sparton/sparton_kernel.py:179-182,
// :578-580, :650, :673), carves the caller's workspace and dispatches to the
// launchers.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "internal.h"

namespace sparton {

namespace {
thread_local char g_last_error[512] = "";

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
}  // namespace

int check_sizes(int64_t B, int64_t S, int64_t D, int64_t V) {
  if (B < 0 || S < 0 || D < 0 || V < 0)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "negative size (B=%lld S=%lld D=%lld V=%lld)",
                (long long)B, (long long)S, (long long)D, (long long)V);
  // B * round16(S): the forward's packed position stream (one column per
  // position, rows rounded up to 16) is indexed with 32-bit integers.
  if (B > 65535 || S > (1 << 24) || D > (1 << 16) || V > (1 << 28) ||
      B * ((S + 15) / 16 * 16) > (1ll << 31) - 1 || B * V > (1ll << 31) - 1)
    return fail(SPARTON_ERR_UNSUPPORTED,
                "sizes out of range (B=%lld S=%lld D=%lld V=%lld; need B<=65535, B*round16(S) and "
                "B*V < 2^31)",
                (long long)B, (long long)S, (long long)D, (long long)V);
  if (D % 8 != 0)
    return fail(SPARTON_ERR_UNSUPPORTED, "hidden size D=%lld must be a multiple of 8", (long long)D);
  return SPARTON_OK;
}

int check_dtype(int dtype) {
  if (dtype != SPARTON_DTYPE_F32 && dtype != SPARTON_DTYPE_F16 && dtype != SPARTON_DTYPE_BF16)
    return fail(SPARTON_ERR_UNSUPPORTED, "unknown dtype %d", dtype);
  return SPARTON_OK;
}

int check_device() {
  if (!device_is_sm100())
    return fail(SPARTON_ERR_DEVICE, "the current CUDA device is not compute capability 10.x (sm_100)");
  return SPARTON_OK;
}

namespace {
int check_workspace(const void* ws, size_t have, size_t need) {
  if (ws == nullptr || have < need)
    return fail(SPARTON_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given%s", need, have,
                ws == nullptr ? " (NULL)" : "");
  if (!aligned(ws, 256)) return fail(SPARTON_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  return SPARTON_OK;
}

#define SPARTON_TRY(expr)           \
  do {                              \
    const int st_ = (expr);         \
    if (st_ != SPARTON_OK) return st_; \
  } while (0)

}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(SPARTON_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

namespace {
struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool known = false;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

DeviceInfo current_device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DeviceInfo{};
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (!g_dev[dev].known) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return DeviceInfo{};
    g_dev[dev].sms = sms;
    g_dev[dev].major = major;
    g_dev[dev].known = true;
  }
  return g_dev[dev];
}
}  // namespace

int device_sm_count() {
  const DeviceInfo d = current_device_info();
  return d.sms > 0 ? d.sms : 1;
}

bool device_is_sm100() { return current_device_info().major == 10; }

}  // namespace sparton

using namespace sparton;

extern "C" {

int sparton_abi_version(void) { return SPARTON_ABI_VERSION; }

const char* sparton_last_error(void) { return g_last_error; }

size_t sparton_fwd_workspace_size(int64_t B, int64_t S, int64_t D, int64_t V) {
  (void)D;
  (void)V;
  if (B < 0 || S < 0) return 0;
  return fwd_workspace_bytes(B, S);
}

int sparton_mask_prepare(const void* mask, int mask_dtype, int64_t B, int64_t S, void* workspace,
                         size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, S, 8, 0));
  if (mask_dtype < SPARTON_MASK_U8 || mask_dtype > SPARTON_MASK_BF16)
    return fail(SPARTON_ERR_UNSUPPORTED, "unknown mask dtype %d", mask_dtype);
  SPARTON_TRY(check_workspace(workspace, workspace_size, fwd_workspace_bytes(B, S)));
  if (B == 0) return SPARTON_OK;
  if (mask == nullptr && S > 0) return fail(SPARTON_ERR_INVALID_ARGUMENT, "mask is NULL");
  SPARTON_TRY(check_device());
  const FwdWorkspace ws = fwd_workspace_carve(workspace, B, S);
  return launch_mask_prepare(mask, mask_dtype, static_cast<int>(B), static_cast<int>(S), ws,
                             static_cast<cudaStream_t>(stream));
}

int sparton_fwd_prepared(const void* hidden, const void* weight, const void* bias, int dtype,
                         int64_t B, int64_t S, int64_t D, int64_t V, void* reps, int32_t* idx,
                         void* workspace, size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, S, D, V));
  SPARTON_TRY(check_dtype(dtype));
  SPARTON_TRY(check_workspace(workspace, workspace_size, fwd_workspace_bytes(B, S)));
  if (B == 0 || V == 0) return SPARTON_OK;
  if (reps == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "reps output is NULL");
  if ((S > 0 && (hidden == nullptr || D == 0)) || weight == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "hidden / weight is NULL or D == 0");
  if (!aligned(hidden, 16) || !aligned(weight, 16))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "hidden and weight must be 16-byte aligned");
  SPARTON_TRY(check_device());
  const FwdWorkspace ws = fwd_workspace_carve(workspace, B, S);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int b = static_cast<int>(B), s = static_cast<int>(S), d = static_cast<int>(D),
            v = static_cast<int>(V);
  if (dtype == SPARTON_DTYPE_F32)
    return launch_fwd_f32(static_cast<const float*>(hidden), static_cast<const float*>(weight),
                          static_cast<const float*>(bias), b, s, d, v, static_cast<float*>(reps),
                          idx, ws, st);
  if (S == 0) {
    // No positions at all: every output is the empty-row value (0, index 0).
    cudaError_t e = cudaMemsetAsync(reps, 0, static_cast<size_t>(B * V) * 2, st);
    if (e == cudaSuccess && idx != nullptr)
      e = cudaMemsetAsync(idx, 0, static_cast<size_t>(B * V) * 4, st);
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "cudaMemsetAsync");
  }
  return launch_fwd_tc(dtype, hidden, weight, bias, b, s, d, v, reps, idx, ws, st);
}

int sparton_fwd(const void* hidden, const void* weight, const void* bias, const void* mask,
                int mask_dtype, int dtype, int64_t B, int64_t S, int64_t D, int64_t V, void* reps,
                int32_t* idx, void* workspace, size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, S, D, V));
  SPARTON_TRY(check_dtype(dtype));
  SPARTON_TRY(sparton_mask_prepare(mask, mask_dtype, B, S, workspace, workspace_size, stream));
  return sparton_fwd_prepared(hidden, weight, bias, dtype, B, S, D, V, reps, idx, workspace,
                              workspace_size, stream);
}

size_t sparton_bwd_workspace_size(int64_t B, int64_t S, int64_t D, int64_t V) {
  (void)D;
  if (B < 0 || S < 0 || V < 0) return 0;
  return bwd_workspace_bytes(B, S, V);
}

int sparton_bwd(const void* grad_reps, const void* reps, const int32_t* idx, const void* hidden,
                const void* weight, int dtype, int64_t B, int64_t S, int64_t D, int64_t V,
                void* d_hidden, void* d_weight, void* d_bias, int d_hidden_dtype,
                int d_param_dtype, void* workspace, size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, S, D, V));
  SPARTON_TRY(check_dtype(dtype));
  if ((d_hidden_dtype != dtype && d_hidden_dtype != SPARTON_DTYPE_F32) ||
      (d_param_dtype != dtype && d_param_dtype != SPARTON_DTYPE_F32))
    return fail(SPARTON_ERR_UNSUPPORTED, "gradient dtypes must equal dtype or be F32");
  SPARTON_TRY(check_workspace(workspace, workspace_size, bwd_workspace_bytes(B, S, V)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t hsz = d_hidden_dtype == SPARTON_DTYPE_F32 ? 4 : 2;
  const size_t psz = d_param_dtype == SPARTON_DTYPE_F32 ? 4 : 2;
  if (B == 0 || V == 0 || S == 0) {
    // Nothing flows back: write the zero gradients the caller asked for.
    cudaError_t e = cudaSuccess;
    if (d_hidden != nullptr && B * S * D > 0)
      e = cudaMemsetAsync(d_hidden, 0, static_cast<size_t>(B * S * D) * hsz, st);
    if (e == cudaSuccess && d_weight != nullptr && V * D > 0)
      e = cudaMemsetAsync(d_weight, 0, static_cast<size_t>(V * D) * psz, st);
    if (e == cudaSuccess && d_bias != nullptr && V > 0)
      e = cudaMemsetAsync(d_bias, 0, static_cast<size_t>(V) * psz, st);
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "cudaMemsetAsync");
  }
  if (grad_reps == nullptr || reps == nullptr || idx == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "grad_reps / reps / idx is NULL");
  if ((d_hidden != nullptr && weight == nullptr) || (d_weight != nullptr && hidden == nullptr))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "hidden / weight is NULL");
  if (D == 0) return fail(SPARTON_ERR_INVALID_ARGUMENT, "D == 0");
  const void* ptrs[5] = {hidden, weight, d_hidden, d_weight, nullptr};
  for (const void* p : ptrs)
    if (p != nullptr && !aligned(p, 16))
      return fail(SPARTON_ERR_INVALID_ARGUMENT, "hidden / weight / gradients must be 16-byte aligned");
  SPARTON_TRY(check_device());
  const BwdWorkspace ws = bwd_workspace_carve(workspace, B, S, V);
  return launch_bwd(dtype, grad_reps, reps, idx, hidden, weight, static_cast<int>(B),
                    static_cast<int>(S), static_cast<int>(D), static_cast<int>(V), d_hidden,
                    d_weight, d_bias, d_hidden_dtype, d_param_dtype, ws, st);
}

size_t sparton_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0 || M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return 0;
  return gemm_workspace_bytes(M, N, K);
}

int sparton_gemm(const void* A, int a_layout, int64_t lda, const void* B, int b_layout,
                 int64_t ldb, const void* bias, int dtype, int64_t M, int64_t N, int64_t K, void* C,
                 int c_dtype, int64_t ldc, void* workspace, size_t workspace_size, void* stream) {
  if (dtype != SPARTON_DTYPE_BF16 && dtype != SPARTON_DTYPE_F16)
    return fail(SPARTON_ERR_UNSUPPORTED, "sparton_gemm takes bf16 or f16 operands (dtype %d)",
                dtype);
  if (c_dtype != dtype && c_dtype != SPARTON_DTYPE_F32)
    return fail(SPARTON_ERR_UNSUPPORTED, "c_dtype must equal dtype or be F32");
  if ((a_layout != SPARTON_LAYOUT_ROWS && a_layout != SPARTON_LAYOUT_COLS) ||
      (b_layout != SPARTON_LAYOUT_ROWS && b_layout != SPARTON_LAYOUT_COLS))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "unknown operand layout");
  if (M < 0 || N < 0 || K < 0 || M > (1 << 30) || N > (1 << 30) || K > (1 << 30))
    return fail(SPARTON_ERR_UNSUPPORTED, "sizes out of range (M=%lld N=%lld K=%lld)",
                (long long)M, (long long)N, (long long)K);
  if (ldc < N) return fail(SPARTON_ERR_INVALID_ARGUMENT, "ldc=%lld < N=%lld", (long long)ldc,
                           (long long)N);
  // TMA: every stored row of an operand starts on a 16-byte boundary.
  const int64_t a_inner = a_layout == SPARTON_LAYOUT_ROWS ? K : M;
  const int64_t b_inner = b_layout == SPARTON_LAYOUT_ROWS ? K : N;
  if (lda == 0) lda = a_inner;
  if (ldb == 0) ldb = b_inner;
  if (lda < a_inner || ldb < b_inner)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "lda=%lld / ldb=%lld below the rows' extent",
                (long long)lda, (long long)ldb);
  if (lda % 8 != 0 || ldb % 8 != 0 || lda > (1ll << 31) || ldb > (1ll << 31))
    return fail(SPARTON_ERR_UNSUPPORTED,
                "stored operand rows must hold a multiple of 8 elements (A: %lld, B: %lld); pad "
                "the contiguous dimension",
                (long long)lda, (long long)ldb);
  SPARTON_TRY(check_workspace(workspace, workspace_size, gemm_workspace_bytes(M, N, K)));
  if (M == 0 || N == 0) return SPARTON_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr)))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "A / B / C is NULL");
  if (!aligned(A, 16) || !aligned(B, 16))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "A and B must be 16-byte aligned");
  SPARTON_TRY(check_device());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    // Empty contraction: C = bias broadcast (or 0); written by the reduction-free
    // path with no operand reads.
    return fail(SPARTON_ERR_UNSUPPORTED, "K == 0 is not supported");
  }
  return launch_gemm(dtype, c_dtype, a_layout == SPARTON_LAYOUT_COLS,
                     b_layout == SPARTON_LAYOUT_COLS, A, lda, B, ldb, bias, static_cast<int>(M),
                     static_cast<int>(N), static_cast<int>(K), C, ldc, workspace, st);
}

int sparton_pad_rows(const void* src, int dtype, int64_t rows, int64_t cols, void* dst,
                     int64_t ld, void* stream) {
  if (dtype != SPARTON_DTYPE_BF16 && dtype != SPARTON_DTYPE_F16)
    return fail(SPARTON_ERR_UNSUPPORTED, "sparton_pad_rows takes bf16 or f16 (dtype %d)", dtype);
  if (rows < 0 || cols < 0 || ld < cols || rows > (1ll << 31) - 1 || ld > (1ll << 31) - 1)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "bad sizes (rows=%lld cols=%lld ld=%lld)",
                (long long)rows, (long long)cols, (long long)ld);
  if (ld % 8 != 0 || !aligned(dst, 16))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "dst rows must be 16-byte aligned (ld %% 8 == 0)");
  if (rows == 0 || ld == 0) return SPARTON_OK;
  if (dst == nullptr || (cols > 0 && src == nullptr))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "src / dst is NULL");
  SPARTON_TRY(check_device());
  return launch_pad_rows(dtype, src, static_cast<int>(rows), static_cast<int>(cols), dst,
                         static_cast<int>(ld), static_cast<cudaStream_t>(stream));
}

int sparton_read_device_status(const void* workspace, void* stream, uint32_t* code) {
  if (workspace == nullptr || code == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "workspace / code is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(code, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "reading device status");
}


size_t sparton_reg_workspace_size(int64_t B, int64_t V) {
  (void)B;
  if (V < 0) return 0;
  return reg_workspace_bytes(V);
}

int sparton_reg_fwd(const void* reps, int dtype, int64_t B, int64_t V, float scale_l1,
                    float scale_flops, float* colsum, float* out, void* workspace,
                    size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, 0, 8, V));
  SPARTON_TRY(check_dtype(dtype));
  SPARTON_TRY(check_workspace(workspace, workspace_size, reg_workspace_bytes(V)));
  if (out == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "out is NULL");
  if (V > 0 && colsum == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "colsum is NULL");
  if (B * V > 0 && reps == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "reps is NULL");
  SPARTON_TRY(check_device());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (V == 0) {
    const cudaError_t e = cudaMemsetAsync(out, 0, 2 * sizeof(float), st);
    return e == cudaSuccess ? SPARTON_OK : cuda_fail(e, "cudaMemsetAsync");
  }
  return launch_reg_fwd(dtype, reps, static_cast<int>(B), static_cast<int>(V), scale_l1,
                        scale_flops, colsum, out, workspace, st);
}

int sparton_reg_bwd(const void* reps, const float* colsum, const float* g_l1,
                    const float* g_flops, float scale_l1, float scale_flops, int dtype, int64_t B,
                    int64_t V, void* grad, void* stream) {
  SPARTON_TRY(check_sizes(B, 0, 8, V));
  SPARTON_TRY(check_dtype(dtype));
  if (B * V == 0) return SPARTON_OK;
  if (reps == nullptr || colsum == nullptr || grad == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "reps / colsum / grad is NULL");
  SPARTON_TRY(check_device());
  return launch_reg_bwd(dtype, reps, colsum, g_l1, g_flops, scale_l1, scale_flops,
                        static_cast<int>(B), static_cast<int>(V), grad,
                        static_cast<cudaStream_t>(stream));
}

size_t sparton_sparse_workspace_size(int64_t B, int64_t V) {
  if (B < 0 || V < 0) return 0;
  return sparse_workspace_bytes(B, V);
}

int sparton_reps_csr(const void* reps, int dtype, int64_t B, int64_t V, float threshold,
                     int64_t* crow, int32_t* cols, void* vals, int64_t capacity, void* workspace,
                     size_t workspace_size, void* stream) {
  SPARTON_TRY(check_sizes(B, 0, 8, V));
  SPARTON_TRY(check_dtype(dtype));
  SPARTON_TRY(check_workspace(workspace, workspace_size, sparse_workspace_bytes(B, V)));
  if (crow == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "crow is NULL");
  if (capacity < 0) return fail(SPARTON_ERR_INVALID_ARGUMENT, "negative capacity");
  if (capacity > 0 && (cols == nullptr || vals == nullptr))
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "cols / vals is NULL with capacity %lld",
                (long long)capacity);
  if (B * V > 0 && reps == nullptr) return fail(SPARTON_ERR_INVALID_ARGUMENT, "reps is NULL");
  SPARTON_TRY(check_device());
  return launch_reps_csr(dtype, reps, static_cast<int>(B), static_cast<int>(V), threshold, crow,
                         cols, vals, capacity, sparse_workspace_carve(workspace, B, V),
                         static_cast<cudaStream_t>(stream));
}

int sparton_reps_topk(const void* reps, int dtype, int64_t B, int64_t V, int64_t k, void* vals,
                      int32_t* idx, void* stream) {
  SPARTON_TRY(check_sizes(B, 0, 8, V));
  SPARTON_TRY(check_dtype(dtype));
  if (k < 0 || k > V)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "k=%lld must lie in [0, V=%lld]", (long long)k,
                (long long)V);
  if (k > kTopkMax)
    return fail(SPARTON_ERR_UNSUPPORTED, "k=%lld above the supported %d", (long long)k, kTopkMax);
  if (B * k == 0) return SPARTON_OK;
  if (reps == nullptr || vals == nullptr || idx == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "reps / vals / idx is NULL");
  SPARTON_TRY(check_device());
  return launch_reps_topk(dtype, reps, static_cast<int>(B), static_cast<int>(V),
                          static_cast<int>(k), vals, idx, static_cast<cudaStream_t>(stream));
}

size_t sparton_transform_workspace_size(int64_t rows, int64_t D) {
  if (rows < 0 || D < 0) return 0;
  return transform_workspace_bytes(rows, D);
}

int sparton_transform_fwd(const void* y, const void* gamma, const void* beta, float eps, int dtype,
                          int64_t rows, int64_t D, void* h, float* mean, float* rstd,
                          void* stream) {
  SPARTON_TRY(check_dtype(dtype));
  if (rows < 0 || D < 1 || rows > (1ll << 31) - 1 || D > (1 << 16) || rows * D > (1ll << 40))
    return fail(SPARTON_ERR_UNSUPPORTED, "sizes out of range (rows=%lld D=%lld)",
                (long long)rows, (long long)D);
  if (rows == 0) return SPARTON_OK;
  if (y == nullptr || gamma == nullptr || beta == nullptr || h == nullptr || mean == nullptr ||
      rstd == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  if (!(eps >= 0.f)) return fail(SPARTON_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  SPARTON_TRY(check_device());
  return launch_transform_fwd(dtype, y, gamma, beta, eps, static_cast<int>(rows),
                              static_cast<int>(D), h, mean, rstd,
                              static_cast<cudaStream_t>(stream));
}

int sparton_transform_bwd(const void* dh, const void* y, const void* gamma, const float* mean,
                          const float* rstd, int dtype, int64_t rows, int64_t D, void* dy,
                          void* d_gamma, void* d_beta, void* d_bias, void* workspace,
                          size_t workspace_size, void* stream) {
  SPARTON_TRY(check_dtype(dtype));
  if (rows < 0 || D < 1 || rows > (1ll << 31) - 1 || D > (1 << 16) || rows * D > (1ll << 40))
    return fail(SPARTON_ERR_UNSUPPORTED, "sizes out of range (rows=%lld D=%lld)",
                (long long)rows, (long long)D);
  const bool cols = d_gamma != nullptr || d_beta != nullptr || d_bias != nullptr;
  // the column sums take one CTA row per 256 rows, 65535 at most
  if (cols && rows > 65535ll * 256)
    return fail(SPARTON_ERR_UNSUPPORTED, "rows=%lld above %lld for the parameter gradients",
                (long long)rows, 65535ll * 256);
  if (cols) SPARTON_TRY(check_workspace(workspace, workspace_size, transform_workspace_bytes(rows, D)));
  if (rows == 0) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t es = dtype == SPARTON_DTYPE_F32 ? 4 : 2;
    for (void* p : {d_gamma, d_beta, d_bias})
      if (p != nullptr) {
        const cudaError_t e = cudaMemsetAsync(p, 0, static_cast<size_t>(D) * es, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
      }
    return SPARTON_OK;
  }
  if (dh == nullptr || y == nullptr || gamma == nullptr || mean == nullptr || rstd == nullptr ||
      dy == nullptr)
    return fail(SPARTON_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  SPARTON_TRY(check_device());
  return launch_transform_bwd(dtype, dh, y, gamma, mean, rstd, static_cast<int>(rows),
                              static_cast<int>(D), dy, d_gamma, d_beta, d_bias, workspace,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
