/*
 * sparton_b200.h — C ABI of the B200-native SPLADE projection head.
 *
 * The head computes, for hidden states H[B,S,D], decoder weight W[V,D],
 * optional bias b[V] and attention mask M[B,S]:
 *
 *     logits[b,s,v] = H[b,s,:] . W[v,:] + b[v]
 *     reps[b,v]     = max_s log1p(relu(logits[b,s,v] * M[b,s]))
 *     idx[b,v]      = smallest s attaining that max (0 when the max is <= 0)
 *
 * and its backward (g = dLoss/dreps):
 *
 *     g'[b,v]            = reps[b,v] > 0 ? g[b,v] * exp(-reps[b,v]) : 0
 *     dH[b,idx[b,v],:]  += g'[b,v] * W[v,:]
 *     dW[v,:]            = sum_b g'[b,v] * H[b,idx[b,v],:]
 *     db[v]              = sum_b g'[b,v]
 *
 * Upstream, the same operator is the pair of torch custom ops
 * `sparton::fused_sparton_fwd` / `sparton::fused_sparton_bwd`
 * (hhkbble/sparton src/sparton/sparton_kernel.py:643-707), whose host drivers
 * are fused_sparton_fwd_with_indices (:226-253) and
 * fused_sparton_bwd_with_bias (:567-597). Those are Python functions bound
 * to torch tensors; this header is the language-neutral boundary that replaces
 * them: plain device pointers, sizes and a CUDA stream.
 *
 * Conventions for every entry point:
 *  - All tensors are dense, row-major (C-contiguous) device memory.
 *  - The library never allocates, frees or synchronises. The caller owns all
 *    buffers, including the scratch `workspace`, whose size is given by the
 *    matching *_workspace_size() function. Workspace pointers must be 256-byte
 *    aligned (any cudaMalloc / torch allocation is).
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Kernels are
 *    enqueued on it; the call returns before they finish.
 *  - Return value: SPARTON_OK (0) or a sparton_status code; on error nothing
 *    was launched and sparton_last_error() describes the problem. The message
 *    is thread-local.
 *  - Device-side waits are bounded. A kernel that gives up records a nonzero
 *    code in the workspace; sparton_read_device_status() returns it.
 */
#ifndef SPARTON_B200_H_
#define SPARTON_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPARTON_ABI_VERSION 1

typedef enum {
  SPARTON_OK = 0,
  SPARTON_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer, misaligned buffer */
  SPARTON_ERR_UNSUPPORTED = 2,      /* dtype / size outside what the kernels cover */
  SPARTON_ERR_WORKSPACE = 3,        /* workspace too small */
  SPARTON_ERR_CUDA = 4,             /* a CUDA runtime / driver call failed */
  SPARTON_ERR_DEVICE = 5            /* no sm_100 device current */
} sparton_status;

/* Element type of hidden / weight / bias / reps (and of gradients unless F32
 * is requested for them). */
typedef enum {
  SPARTON_DTYPE_F32 = 0,
  SPARTON_DTYPE_F16 = 1,
  SPARTON_DTYPE_BF16 = 2
} sparton_dtype;

/* Element type of the attention mask [B,S]. Any nonzero entry marks a valid
 * token. The upstream kernel multiplies logits by the mask value
 * (sparton_kernel.py:147); for 0/1 masks (every HF tokenizer mask) the two
 * are identical. */
typedef enum {
  SPARTON_MASK_U8 = 0, /* bool / uint8 */
  SPARTON_MASK_I32 = 1,
  SPARTON_MASK_I64 = 2,
  SPARTON_MASK_F32 = 3,
  SPARTON_MASK_F16 = 4,
  SPARTON_MASK_BF16 = 5
} sparton_mask_dtype;

/* Device status codes written by kernels into the workspace header. */
#define SPARTON_DEV_OK 0u
#define SPARTON_DEV_TIMEOUT_PRODUCER 0x101u
#define SPARTON_DEV_TIMEOUT_MMA 0x102u
#define SPARTON_DEV_TIMEOUT_EPILOGUE 0x103u
#define SPARTON_DEV_TIMEOUT_DRAIN 0x104u
#define SPARTON_DEV_TIMEOUT_SELFTEST 0x1F0u /* sparton_selftest_wait_timeout only */
#define SPARTON_DEV_TIMEOUT_PEER 0x105u     /* sparton_hidden_allreduce: a peer never signalled */
#define SPARTON_DEV_TIMEOUT_SCAN 0x106u     /* sparton_reps_csr: a chunk count never arrived */

int sparton_abi_version(void);

/* Human-readable description of the last error returned on this thread. */
const char* sparton_last_error(void);

/* ---------------------------------------------------------------- forward */

/* Bytes of workspace sparton_fwd / sparton_mask_prepare need. */
size_t sparton_fwd_workspace_size(int64_t B, int64_t S, int64_t D, int64_t V);

/* Full forward. Replaces fused_sparton_fwd_with_indices
 * (sparton_kernel.py:226-253) and the custom op sparton::fused_sparton_fwd
 * (:643-652).
 *   hidden [B,S,D], weight [V,D], bias [V] (NULL = no bias), all `dtype`
 *   mask   [B,S] of `mask_dtype`
 *   reps   [B,V] `dtype` (out), idx [B,V] int32 (out; upstream uses int64)
 * idx may be NULL: the inference forward, which keeps the max alone and
 * stores reps only. It replaces upstream's no-argmax forward fused_sparton_fwd
 * (sparton_kernel.py:372-394, reduce kernel :257-334), whose consumer is an
 * encode under no_grad (training/model.py:141-144); reps are identical to
 * those of the call with idx.
 * bf16 / f16 run on tcgen05 tensor cores with fp32 accumulation; f32 runs an
 * exact fp32 FMA path. Launches sparton_mask_prepare + sparton_fwd_prepared. */
int sparton_fwd(const void* hidden, const void* weight, const void* bias,
                const void* mask, int mask_dtype, int dtype,
                int64_t B, int64_t S, int64_t D, int64_t V,
                void* reps, int32_t* idx,
                void* workspace, size_t workspace_size, void* stream);

/* First half of sparton_fwd: reduce the mask to per-row bit words and
 * per-row extents (last valid position + 1) in the workspace, and reset the
 * device status and tile counter. Upstream re-reads the mask inside its
 * reduce kernel (sparton_kernel.py:140-147). */
int sparton_mask_prepare(const void* mask, int mask_dtype, int64_t B, int64_t S,
                         void* workspace, size_t workspace_size, void* stream);

/* Second half of sparton_fwd: the fused GEMM + masked max/argmax + log1p
 * kernel, given a workspace filled by sparton_mask_prepare for the same B, S.
 * Replaces the per-chunk matmul_bias + reduce loop of
 * fused_sparton_fwd_with_indices (sparton_kernel.py:240-251). */
int sparton_fwd_prepared(const void* hidden, const void* weight, const void* bias,
                         int dtype, int64_t B, int64_t S, int64_t D, int64_t V,
                         void* reps, int32_t* idx,
                         void* workspace, size_t workspace_size, void* stream);

/* Size of the scratch array compiled into the library for
 * sparton_fwd_noalloc (1 MiB). It covers sparton_fwd_workspace_size(B,S,..)
 * <= 1 MiB, i.e. roughly B * (3*S/8 + 24) bytes <= 1,048,576 (e.g. B=1024
 * rows at S=2048, or B=4096 at S=512). */
#define SPARTON_FWD_NOALLOC_SCRATCH_BYTES (1u << 20)

/* sparton_fwd without a caller-provided workspace. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they run the head (a cgo / JNI host with no CUDA allocator of its own, a
 * process whose framework already reserved the device memory for its pool, a
 * loop that must not call cudaMalloc because it can synchronise the device).
 * The scratch lives in a fixed __device__ array inside the library, one copy
 * per GPU that loads it, held until the process exits; nothing is allocated.
 * Arguments and results are those of sparton_fwd. Limits and caveats:
 *  - sizes whose scratch exceeds SPARTON_FWD_NOALLOC_SCRATCH_BYTES are rejected
 *    with SPARTON_ERR_UNSUPPORTED (use sparton_fwd then);
 *  - every call on a device shares the one array: calls that overlap on the
 *    GPU (e.g. on two streams without ordering between them) race and corrupt
 *    each other; serialise them;
 *  - every call looks up the array's device address (cudaGetSymbolAddress)
 *    with the calling device current; the address is not cached, so it stays
 *    right after a cudaDeviceReset, which reloads the module and may move the
 *    array. The first call on a device loads the module there: make it before
 *    any stream capture begins;
 *  - a kernel that gave up on a bounded device wait leaves partial reps / idx
 *    and records a nonzero code in the array's status word, which only
 *    sparton_fwd_noalloc_status can read. */
int sparton_fwd_noalloc(const void* hidden, const void* weight, const void* bias,
                        const void* mask, int mask_dtype, int dtype,
                        int64_t B, int64_t S, int64_t D, int64_t V,
                        void* reps, int32_t* idx, void* stream);

/* Device status word (SPARTON_DEV_*) that the last sparton_fwd_noalloc call on
 * the current device left in the library's scratch array; synchronises
 * `stream` (pass the stream of that call). 0 = no device-side timeout. The
 * counterpart of sparton_read_device_status for the allocation-free forward,
 * whose scratch the caller has no pointer to. */
int sparton_fwd_noalloc_status(void* stream, uint32_t* code);

/* --------------------------------------------------------------- backward */

/* Bytes of workspace sparton_bwd needs. */
size_t sparton_bwd_workspace_size(int64_t B, int64_t S, int64_t D, int64_t V);

/* Backward. Replaces fused_sparton_bwd_with_bias (sparton_kernel.py:567-597)
 * and the custom op sparton::fused_sparton_bwd (:663-685).
 *   grad_reps [B,V], reps [B,V] (`dtype`), idx [B,V] int32 from sparton_fwd
 *   hidden [B,S,D], weight [V,D] (`dtype`)
 *   d_hidden [B,S,D] (out, `d_hidden_dtype`), d_weight [V,D] and d_bias [V]
 *   (out, `d_param_dtype`); each dtype is `dtype` or SPARTON_DTYPE_F32. Any of
 *   the three outputs may be NULL to skip it.
 * Every output element is written (no pre-zeroing needed); the result is
 * deterministic (no atomics). Upstream accumulates with fp32 atomics into
 * zero-initialised fp32 buffers.
 * A call with only d_hidden and a call with only d_weight / d_bias may run
 * concurrently on two streams with the same workspace (they write disjoint
 * parts of it); running them so overlaps the two gathers. */
int sparton_bwd(const void* grad_reps, const void* reps, const int32_t* idx,
                const void* hidden, const void* weight, int dtype,
                int64_t B, int64_t S, int64_t D, int64_t V,
                void* d_hidden, void* d_weight, void* d_bias,
                int d_hidden_dtype, int d_param_dtype,
                void* workspace, size_t workspace_size, void* stream);

/* ---------------------------------------------------------- regularisers */

/* The sparsity regularisers that SPLADE training adds to its loss, on the
 * head's output reps [B, V] (or one vocabulary shard of it), in one pass:
 *   l1    = mean_b sum_v |reps[b, v]|       (training/train.py:80-82)
 *   flops = mean_v (sum_b reps[b, v])^2     (training/train.py:85-87)
 * Upstream computes them with separate torch reductions; there is no
 * counterpart entry point upstream (these replace those two functions). */

/* Bytes of workspace sparton_reg_fwd needs. The workspace must be zero-filled
 * before its first use (e.g. one cudaMemsetAsync after allocating it); every
 * call that runs to completion leaves it zero-filled again, so it is reused
 * as is. One workspace per stream: calls that overlap on the GPU must not
 * share it. */
size_t sparton_reg_workspace_size(int64_t B, int64_t V);

/* colsum[v] = sum_b reps[b, v] (fp32, [V], kept for the backward);
 * out[0] = scale_l1 * sum |reps|, out[1] = scale_flops * sum_v colsum[v]^2
 * (fp32, device). With scale_l1 = 1/B and scale_flops = 1/V_total these are
 * the two losses; over vocabulary shards the outputs simply add up.
 * Deterministic. */
int sparton_reg_fwd(const void* reps, int dtype, int64_t B, int64_t V, float scale_l1,
                    float scale_flops, float* colsum, float* out, void* workspace,
                    size_t workspace_size, void* stream);

/* grad[b, v] = (*g_l1) * scale_l1 * sign(reps[b, v])
 *            + (*g_flops) * scale_flops * colsum[v], in reps' dtype. g_l1 and
 * g_flops point to one fp32 each in device memory (the upstream gradients of
 * the two losses; NULL counts as 0); for the losses scale_l1 = 1/B and
 * scale_flops = 2/V_total. No value crosses to the host. */
int sparton_reg_bwd(const void* reps, const float* colsum, const float* g_l1,
                    const float* g_flops, float scale_l1, float scale_flops, int dtype, int64_t B,
                    int64_t V, void* grad, void* stream);

/* ----------------------------------------------------------- sparse reps */
/* Sparse forms of the head's output for indexing. Upstream has no counterpart:
 * its encode (training/model.py:141-144) returns the dense reps, and
 * training/train.py:205-210 logs the fraction of entries > 0. */

/* Workspace bytes of sparton_reps_csr for reps [B, V]. Zero-fill it once after
 * allocating it; it needs no clearing between calls (each call tags the words
 * it writes). Word 0 is the device status (sparton_read_device_status). One
 * workspace per stream: calls that overlap on the GPU must not share it. */
size_t sparton_sparse_workspace_size(int64_t B, int64_t V);

/* CSR of the entries reps[b, v] > threshold, rows in order, columns ascending
 * inside each row (torch.Tensor.to_sparse_csr of the thresholded reps):
 * crow [B + 1] int64 row starts (crow[B] = nnz); cols [capacity] int32 vocab
 * ids and vals [capacity] (reps' dtype) hold the first `capacity` entries. With
 * capacity 0 (cols / vals may be NULL) only crow is written: the caller reads
 * nnz, allocates, and calls again; capacity = B * V always suffices. */
int sparton_reps_csr(const void* reps, int dtype, int64_t B, int64_t V, float threshold,
                     int64_t* crow, int32_t* cols, void* vals, int64_t capacity, void* workspace,
                     size_t workspace_size, void* stream);

/* The k largest entries of every row of reps [B, V], by value descending and,
 * among equal values, vocab id ascending (NaN above +inf, as torch.topk
 * orders it): vals [B, k] (reps' dtype), idx [B, k] int32. 0 <= k <= V and
 * k <= 4096. No workspace. */
int sparton_reps_topk(const void* reps, int dtype, int64_t B, int64_t V, int64_t k, void* vals,
                      int32_t* idx, void* stream);

/* --------------------------------------------------------- MLM transform */
/* The GELU + LayerNorm part of the MLM transform in front of the head
 * (training/model.py:25-35, BERT's predictions.transform): with y = x @ Wd^T
 * + bd from the dense layer (a plain GEMM: sparton_gemm below, or the caller's BLAS),
 *   h = LayerNorm(gelu(y)) * gamma + beta   (exact erf gelu, its output
 *   rounded to `dtype`; biased variance; eps as torch.nn.LayerNorm)
 * for y, h [rows, D] in `dtype` and gamma, beta [D]; mean / rstd [rows] fp32
 * are saved for the backward. h is the head's hidden_states. */
int sparton_transform_fwd(const void* y, const void* gamma, const void* beta, float eps, int dtype,
                          int64_t rows, int64_t D, void* h, float* mean, float* rstd,
                          void* stream);

/* Workspace bytes of sparton_transform_bwd (column partials). */
size_t sparton_transform_workspace_size(int64_t rows, int64_t D);

/* Backward of sparton_transform_fwd from dh [rows, D] (the head's d_hidden):
 * dy [rows, D] = d(gelu + LayerNorm)/dy (sparton_gemm or the caller's BLAS then
 * forms dx = dy @ Wd and dWd = dy^T @ x), and, each optional (NULL skips it),
 * d_gamma, d_beta [D] and d_bias [D] = sum over rows of dy (the dense bias),
 * in `dtype`, summed in a fixed order (rows <= 65535 * 256 when any of them
 * is requested). */
int sparton_transform_bwd(const void* dh, const void* y, const void* gamma, const float* mean,
                          const float* rstd, int dtype, int64_t rows, int64_t D, void* dy,
                          void* d_gamma, void* d_beta, void* d_bias, void* workspace,
                          size_t workspace_size, void* stream);

/* ------------------------------------------------------------------ GEMM */
/* The contractions around the head on the same tcgen05 tensor-core machinery
 * as the forward: the dense layer of the MLM transform and its two backward
 * products (training/model.py:25-35, used at :82-85), and the InfoNCE scores
 * q_reps @ d_reps.T and their backward (training/train.py:73-77). Upstream
 * runs them as torch matmuls (cuBLAS); this entry point replaces those calls.
 *
 *   C[m, n] = sum_k A[m, k] * B[n, k]  (+ bias[n])      fp32 sums
 *
 * Operand layouts (dense, row-major in memory):
 *   SPARTON_LAYOUT_ROWS: A stored [M][K], B stored [N][K] (contraction index
 *                        contiguous; y = x @ W.T has A = x, B = W);
 *   SPARTON_LAYOUT_COLS: A stored [K][M], B stored [K][N] (output index
 *                        contiguous; dx = dy @ W has B = W stored [K][N],
 *                        dW = dy.T @ x has A = dy, B = x stored [K][*]).
 * A, B and bias [N] are `dtype` (bf16 or f16); C [M][ldc] is `c_dtype` (dtype
 * or F32). lda / ldb: elements per stored row of A / B (0 = dense: K for ROWS,
 * M / N for COLS); they must be multiples of 8 (16-byte rows for the TMA
 * loads), so a caller pads an odd extent (the vocabulary, 30522) and passes the
 * padded row length; padding in the contraction dimension must be zero. 0 < K.
 * Long contractions over few output tiles are split over the K range and the
 * splits added in a fixed order (deterministic); the workspace (256-byte
 * aligned) holds those partials. */
#define SPARTON_LAYOUT_ROWS 0
#define SPARTON_LAYOUT_COLS 1

size_t sparton_gemm_workspace_size(int64_t M, int64_t N, int64_t K);

/* Copies src [rows][cols] into dst [rows][ld] with zeros in columns cols..ld-1
 * (bf16 / f16; ld a multiple of 8, dst 16-byte aligned): the padded operand
 * sparton_gemm needs when a contiguous extent is not a multiple of 8 (reps
 * [B, 30522] for the InfoNCE scores). */
int sparton_pad_rows(const void* src, int dtype, int64_t rows, int64_t cols, void* dst,
                     int64_t ld, void* stream);

int sparton_gemm(const void* A, int a_layout, int64_t lda, const void* B, int b_layout,
                 int64_t ldb, const void* bias, int dtype, int64_t M, int64_t N, int64_t K, void* C,
                 int c_dtype, int64_t ldc, void* workspace, size_t workspace_size, void* stream);

/* ----------------------------------------------------- vocabulary shards */
/* Sum over the ranks of a vocabulary-sharded group (one process per GPU of one
 * node) of every rank's partial d_hidden, over NVLink peer memory; no
 * counterpart in the reference, which is single-GPU (north_star: "the partial
 * dH is all-reduced ... over NVLink"). Only positions before each batch row's
 * extent can carry gradient; the forward's workspace lays them out as T packed
 * rows (the same on every rank), and the sum reads T on the device, so only
 * those rows cross NVLink (a library collective would need T on the host).
 * Rank q reduces packed rows [T q / N, T (q+1) / N) of every rank's partial in
 * fp32, in rank order (deterministic), rounds once to `out_dtype` into its
 * reduced buffer; every rank then copies each row from its owner into its own
 * d_hidden [B,S,D] (`out_dtype`), zeros past the packed rows.
 *   parts[r]  rank r's partial d_hidden, [B*S][D] fp32 (sparton_bwd with
 *             d_hidden_dtype F32), complete in stream order before this call;
 *   reds[r]   rank r's reduced-row buffer, [B*S][D] of out_dtype;
 *   flags[r]  rank r's flag words, 2 x 8 uint32, zero before the first call;
 *   host arrays of `world` (<= 8) device pointers, mapped into this process
 *   (sparton_ipc_open) for r != rank;
 *   epoch     1, 2, 3, ... : one more on every call with these buffers;
 *   fwd_workspace  the workspace of the forward whose d_hidden this is.
 * Every rank makes the same sequence of calls. Waits on peers are bounded
 * (10 s); a wait that gives up records SPARTON_DEV_TIMEOUT_PEER in *status
 * (device memory) and the result is not valid. */
int sparton_hidden_allreduce(void* const* parts, void* const* reds, uint32_t* const* flags,
                             int rank, int world, uint32_t epoch, const void* fwd_workspace,
                             int64_t B, int64_t S, int64_t D, void* d_hidden, int out_dtype,
                             uint32_t* status, void* stream);

/* CUDA IPC for those buffers: export a device pointer of this process as a
 * 64-byte handle plus its offset inside its allocation; open it in another
 * process of the node (current device; peer access is enabled as needed);
 * close it (the pointer sparton_ipc_open returned and the same offset). */
int sparton_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int sparton_ipc_open(const void* handle, uint64_t offset, void** ptr);
int sparton_ipc_close(void* ptr, uint64_t offset);

/* --------------------------------------------------------------- status */

/* Copies the device status word of a workspace used by sparton_fwd /
 * sparton_bwd to *code (synchronises `stream`). 0 = no device-side timeout. */
int sparton_read_device_status(const void* workspace, void* stream, uint32_t* code);

/* Self-test of the bounded device waits; no counterpart in the reference (its
 * kernels never wait on one another). Launches one small kernel whose waits
 * nobody completes, through the same bounded-wait routine the forward uses:
 * one wait gives up after `limit_us` microseconds (1 .. 1e6) and records
 * SPARTON_DEV_TIMEOUT_SELFTEST in word 0 of `workspace` (>= 256 bytes, 256-byte
 * aligned); a second wait, with the production limit, leaves early through the
 * abort flag the first one raised. Word 1 = microseconds the first wait
 * waited, word 2 = 1 when the second left through the abort flag. Nothing
 * faults and the kernel ends by itself; the context stays usable. Read the
 * words (or sparton_read_device_status) after the stream has run it. */
int sparton_selftest_wait_timeout(uint32_t limit_us, void* workspace, size_t workspace_size,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARTON_B200_H_ */
