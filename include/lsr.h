/*
 * liblsr — C ABI of the B200 (sm_100a) optimizer hot path of cuda-lsr.
 *
 * Conventions shared by every entry point:
 *   - pointers are device pointers unless a comment says "host";
 *   - matrices are row-major with the given shape; batches are contiguous;
 *   - all work is enqueued on `stream`; nothing synchronizes the host;
 *   - nothing allocates: scratch memory comes from the caller's workspace
 *     (`ws`, `ws_bytes`), sized by the matching *_workspace_bytes() query;
 *   - the return value is LSR_OK or a negative LSR_ERR_* code; device-side
 *     failures (a bounded wait that timed out: codes 101-107; an event index
 *     out of range: 110) are recorded in the library's device status word,
 *     read with lsr_device_status();
 *   - calls are thread-safe as long as concurrent calls use distinct
 *     workspaces.
 *
 * Each declaration names the reference interface it replaces (paths are
 * relative to the cuda-lsr repository root).
 */
#ifndef LSR_H_
#define LSR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LSR_API __attribute__((visibility("default")))
#else
#define LSR_API
#endif

typedef struct CUstream_st* lsr_stream_t; /* == cudaStream_t */

#define LSR_OK 0
#define LSR_ERR_ARG (-1)       /* null pointer, bad count or flag            */
#define LSR_ERR_SHAPE (-2)     /* unsupported shape / batch / group count    */
#define LSR_ERR_WORKSPACE (-3) /* workspace missing or too small             */
#define LSR_ERR_LAUNCH (-4)    /* kernel launch failed (cudaGetLastError)    */
#define LSR_ERR_DRIVER (-5)    /* TMA tensor-map encoding failed             */
#define LSR_ERR_DEVICE (-6)    /* current device is not sm_100               */
#define LSR_ERR_TOO_LARGE (-7) /* problem exceeds the fixed scratch capacity */
#define LSR_ERR_PEER (-8)      /* CUDA IPC / peer memory call failed         */

/* Element types of lsr_blocks_apply_any's update operand. */
#define LSR_DTYPE_F32 0
#define LSR_DTYPE_BF16 1
#define LSR_DTYPE_F16 2

/* Library version string, e.g. "lsr-b200 0.1.0 (sm_100a)". */
LSR_API const char* lsr_version(void);

/* Human-readable message for an LSR_ERR_* code. */
LSR_API const char* lsr_strerror(int code);

/* Reads the device status word of the current device into *code (0 = no
 * failure recorded) and clears it when `clear` is non-zero. Synchronizes the
 * device. New: the reference has no device-side failure reporting. */
LSR_API int lsr_device_status(int* code, int clear);

/* Number of kernels this library has launched in this process. New: no
 * counterpart in the reference (used to report launches per step). */
LSR_API long long lsr_launch_count(void);

/* Per-launch timing. While enabled, every kernel launch of the library is
 * bracketed by two CUDA events recorded on its stream. lsr_profile_read
 * waits for the recorded events and returns, per launch kind (0 = NS X X^T,
 * 1 = NS b A + c A^2, 2 = NS a X + B X, 3 = momentum/orientation,
 * 4 = normalisation, 5 = parameter update, 6 = other GEMMs, 7 = other
 * elementwise), the summed milliseconds and launch counts, and clears the
 * records when `reset` is non-zero. New: the reference times phases with
 * torch CUDA events in its driver scripts (muon_lm_ddp.py:1309-1409). */
LSR_API int lsr_profile_enable(int on);
LSR_API int lsr_profile_read(double* ms, long long* launches, int nkinds, int reset);

/* ------------------------------------------------------------------------
 * Newton–Schulz quintic orthogonalisation (Muon).
 *
 * Replaces zeropower_serial(G, ns_steps, eps)           muon_lm_ddp.py:331-370
 *      and zeropower_batched_oriented(X, ns_steps, eps) muon_lm_ddp.py:373-426
 *
 * in/out: bf16 [batch, rows, cols]. With orient=1 a tall input (rows > cols)
 * is transposed before the iteration and the result transposed back
 * (zeropower_serial); with orient=0 the polynomial runs on the input as
 * given (zeropower_batched_oriented). Each matrix is divided by its bf16
 * Frobenius norm clamped at eps, then `steps` times
 *     A = X X^T ; B = b A + c A^2 ; X = a X + B X
 * with bf16 storage between products and fp32 accumulation inside them,
 * rounding at the same points as the reference's torch ops.
 * `in` and `out` may not overlap the workspace; `out` may equal `in`.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_ns_workspace_bytes(int batch, int rows, int cols, int orient);
LSR_API int lsr_ns_bf16(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a, float b,
                float c, float eps, void* ws, size_t ws_bytes, lsr_stream_t stream);

/* Allocation-free variant of lsr_ns_bf16 (same arguments minus the
 * workspace; same kernels and results). No counterpart in the reference: it
 * serves callers that cannot allocate device memory themselves (a host
 * program whose device memory belongs to another allocator, or one that
 * cannot afford the device synchronisation cudaMalloc/cudaFree may cause).
 * Its scratch is a fixed 24 MiB device array inside the library, held by
 * every GPU that loads the library until exit; problems whose
 * lsr_ns_workspace_bytes() exceeds lsr_ns_noalloc_capacity() are rejected
 * with LSR_ERR_TOO_LARGE. All calls share that array: calls that overlap on
 * the GPU race and must be ordered by the caller. The first call on a device
 * looks up the array's device address; make it before any stream capture. */
LSR_API size_t lsr_ns_noalloc_capacity(void);
LSR_API int lsr_ns_bf16_noalloc(const void* in, void* out, int batch, int rows, int cols, int orient, int steps,
                                float a, float b, float c, float eps, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Muon step over groups of equally shaped parameter matrices.
 *
 * Replaces MuonAdamW._momentum_update   muon_lm_ddp.py:554-568
 *          MuonAdamW._apply_update      muon_lm_ddp.py:571-593
 *          MuonAdamW.muon_step_batched  muon_lm_ddp.py:615-683
 *
 * A group holds `count` bf16 matrices of shape rows x cols (unoriented
 * parameter shape). grad_ptrs / mom_ptrs / param_ptrs are DEVICE arrays of
 * `count` device addresses (uint64) of the gradients, momentum buffers and
 * parameters. `lr` is the group's adjusted learning rate (adjusted_muon_lr).
 * ---------------------------------------------------------------------- */
typedef struct lsr_muon_group {
  int rows;
  int cols;
  int count;
  const uint64_t* grad_ptrs;
  const uint64_t* mom_ptrs;
  const uint64_t* param_ptrs;
  float lr;
} lsr_muon_group;

/* Workspace for lsr_muon_step_bf16 / lsr_muon_orthogonalize_bf16 (host array
 * of `ngroups` group descriptors). */
LSR_API size_t lsr_muon_workspace_bytes(const lsr_muon_group* groups, int ngroups);

/* Full step: momentum (and Nesterov) update, Newton–Schulz on every matrix,
 * decoupled weight decay p *= 1 - base_lr*wd, then p -= lr * update. */
LSR_API int lsr_muon_step_bf16(const lsr_muon_group* groups, int ngroups, float momentum, int nesterov,
                       float weight_decay, float base_lr, int ns_steps, float a, float b, float c, float eps,
                       void* ws, size_t ws_bytes, lsr_stream_t stream);

/* Sharded step, part 1: momentum update and Newton–Schulz for the matrices of
 * `groups`; group g's orthogonalised updates are written, oriented
 * (min(rows,cols) x max(rows,cols)), into the bf16 buffer updates[g]
 * [count, m, n] (host array of device pointers). */
LSR_API int lsr_muon_orthogonalize_bf16(const lsr_muon_group* groups, int ngroups, float momentum, int nesterov,
                                int ns_steps, float a, float b, float c, float eps, void* const* updates,
                                void* ws, size_t ws_bytes, lsr_stream_t stream);

/* The same in two calls that share `ws` (same groups, same ws pointer):
 * phase 1 runs the momentum update, orientation and Frobenius normalisation
 * into the workspace; phase 2 the Newton–Schulz iterations from there into
 * updates[g]; phase 3 both (= lsr_muon_orthogonalize_bf16). Lets a sharded
 * step run every group's memory-bound prologue before the parameter exchange
 * of the first group starts. */
LSR_API int lsr_muon_orthogonalize_phase_bf16(const lsr_muon_group* groups, int ngroups, float momentum,
                                              int nesterov, int ns_steps, float a, float b, float c, float eps,
                                              void* const* updates, int phase, void* ws, size_t ws_bytes,
                                              lsr_stream_t stream);

/* Sharded step, part 2: apply oriented updates (e.g. after an all-gather) to
 * the parameters of `groups` (grad/mom pointers are not read). */
LSR_API int lsr_muon_apply_bf16(const lsr_muon_group* groups, int ngroups, const void* const* updates,
                        float weight_decay, float base_lr, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Batched GEMM on the tcgen05 engine: D[b] = alpha * opA(A[b]) * opB(B[b]).
 *
 * Replaces the torch matmuls of the optimizer path (muon_lm_ddp.py:406-424,
 * hft.py:127-138, shampoo.py:331-339).
 *
 * A is M x K stored [M][K] (a_trans=0) or [K][M] (a_trans=1); B is K x N
 * stored [K][N] (b_trans=0) or [N][K] (b_trans=1); D is [M][N], bf16
 * (out_f32=0) or fp32 (out_f32=1). Inputs bf16, fp32 accumulation. Every
 * stored row length must be a multiple of 8 elements (16-byte TMA strides).
 * ---------------------------------------------------------------------- */
LSR_API int lsr_gemm_bf16(const void* A, const void* B, void* D, int batch, int M, int N, int K, int a_trans,
                          int b_trans, int out_f32, float alpha, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Shampoo statistics update (symmetric Gram matrix, fp32, EMA):
 *   side 0:  S[b] = beta * S[b] + alpha * G[b] G[b]^T    (S is rows x rows)
 *   side 1:  S[b] = beta * S[b] + alpha * G[b]^T G[b]    (S is cols x cols)
 *
 * Replaces the L/R statistics update of DistributedShampoo (third-party
 * distributed_shampoo, called from shampoo_soap_lm_ddp_zero1.py:609);
 * config 3's  L = G_s G_s^T  is side 0 with beta = 0, alpha = 1.
 * G is bf16 [batch, rows, cols] (cols a multiple of 8). Only the upper
 * triangle is computed; the lower triangle is written as its mirror.
 * ---------------------------------------------------------------------- */
LSR_API int lsr_gram_update_f32(const void* G, void* S, int batch, int rows, int cols, int side, float beta,
                                float alpha, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * fp32 batched GEMM on the tensor cores: C[b] = alpha A[b] B[b] with A [M][K],
 * B [K][N], C [M][N] row-major fp32, evaluated as 3xTF32 (hi*hi + hi*lo +
 * lo*hi of the tf32 splits, corrections in a second accumulator): fp32-level
 * accuracy. Replaces the reference's fp32 torch.matmul / bmm products of its
 * preconditioner code (the coupled-Newton products, shampoo.py:408-542; the
 * two-sided apply, hft.py:108-140). K and N multiples of 4.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_gemm_f32_workspace_bytes(int batch, int M, int N, int K);
LSR_API int lsr_gemm_f32(const float* A, const float* B, float* C, int batch, int M, int N, int K, float alpha,
                         void* ws, size_t ws_bytes, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Batched Householder QR of square fp32 matrices, n <= 1024:
 *   W[b] = Q[b] R[b], Q written to Q (W is overwritten by R and the
 *   Householder vectors), column signs chosen so that diag(R) >= 0.
 * SOAP eigenbasis refresh (the periodic, amortized eigenbasis computation of
 * DefaultSOAPConfig in the third-party distributed_shampoo, whose periodic
 * steps shampoo_soap_lm_ddp_zero1.py:622-653 times): `iterations` steps of
 * power iteration on each factor S[b] (n x n, fp32, symmetric):
 *   W = (S + eps I) Qf  (from_identity: W = S + eps I on the first step),
 *   Qf = qr(W).Q;
 * Qf [b][n][n] fp32 is the basis in and out; Qb, if not null, receives its
 * bf16 copy (the operand of lsr_soap_direction_bf16). Because diag(R) >= 0
 * a converged basis comes back unchanged, without column sign flips.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_qr_workspace_bytes(int batch, int n);
LSR_API int lsr_householder_qr_f32(float* W, float* Q, int batch, int n, void* ws, size_t ws_bytes,
                                   lsr_stream_t stream);
LSR_API size_t lsr_eigenbasis_refresh_workspace_bytes(int batch, int n);
LSR_API int lsr_eigenbasis_refresh_f32(const float* S, float* Qf, void* Qb, int batch, int n, float eps,
                                       int from_identity, int iterations, void* ws, size_t ws_bytes,
                                       lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Kronecker sum  (A ⊕ B) vec(X) = vec(A X + X B^T), row-major vec, batched
 * over X [batch][m][n]; A (m x m) and B (n x n) shared by the batch; Y is
 * fp32 [batch][m][n]. One fused kernel: both products accumulate in the same
 * tensor-memory tile; A ⊗ I and I ⊗ B are never formed.
 *
 * Replaces the S = 2 case {(A, I), (I, B)} of kron_sum_64x8_kernel /
 * kron_sum_out (hft_fused.py:89-319) and of kron_apply_shared_2d
 * (hft.py:108-140), generalised to any m, n with m % 8 == 0 and n % 8 == 0.
 *   _bf16: bf16 operands, fp32 accumulation.
 *   _f32 : fp32 operands via a 3xTF32 split on tensor cores (workspace from
 *          lsr_kron_sum_workspace_bytes(batch, m, n, 1)); m, n % 4 == 0.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_kron_sum_workspace_bytes(int batch, int m, int n, int f32);
LSR_API int lsr_kron_sum_bf16(const void* A, const void* X, const void* B, float* Y, int batch, int m, int n,
                              lsr_stream_t stream);
LSR_API int lsr_kron_sum_f32(const float* A, const float* X, const float* B, float* Y, int batch, int m, int n,
                             void* ws, size_t ws_bytes, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Kronecker apply  Y[i] = sum_s A_s X[i] B_s^T  (= (sum_s A_s ⊗ B_s) vec(X)).
 *
 * Replaces kron_sum_out(x, at, b, out) / kron_sum_64x8_kernel<S>
 * (hft_fused.py:89-319, there fixed to m = 64, n = 8, S in {1,2,4,8}) and
 * kron_apply_shared_2d (hft.py:108-140, hft_fused.py:463-509); with S = 1 it
 * is the Shampoo preconditioner apply L^{-1/4} G R^{-1/4}.
 * A: [nterms][m][m] (a_trans = 1: the array holds A_s^T, as kron_sum_out's
 * `at`), B: [nterms][n][n], X: [batch][m][n], Y: fp32 [batch][m][n].
 * Each term is two chained GEMMs (the cheaper association first); the
 * intermediate is kept as a hi + lo pair so the second product stays at fp32
 * accuracy.  _bf16: bf16 operands.  _f32: fp32 operands (3xTF32).
 * Small fp32 problems (m <= 64, n in {1, 2, 4, 8, 16}) run as one fp32 FFMA
 * launch instead when a cost model fitted on B200 predicts it faster than the
 * tensor-core path (the reference's x [M, 64, 8] sweep: M <= 256 up to S = 8,
 * M = 1024 up to S = 4, M = 4096 at S = 1): the workspace size is then 0 and ws
 * may be NULL.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_kron_apply_workspace_bytes(int batch, int m, int n, int nterms, int f32);
/* Small-factor Kronecker apply split in two, for callers that apply the same
 * factors to many right-hand-side batches (m n <= 1024, m n % 4 == 0):
 *   lsr_kron_dense_operator_f32: W = sum_s A_s (x) B_s as a tf32 pair, Wh and Wl
 *     fp32 [m n][m n] (A_s given transposed when a_trans, like kron_sum_out's
 *     prepacked at = A^T, hft_fused.py:247-252);
 *   lsr_kron_dense_apply_f32: Y [batch][m n] = X [batch][m n] W^T, one 3xTF32 GEMM.
 * lsr_kron_apply_f32 does both per call. */
LSR_API int lsr_kron_dense_operator_f32(const float* A, int a_trans, const float* B, int m, int n, int nterms,
                                        float* Wh, float* Wl, lsr_stream_t stream);
LSR_API size_t lsr_kron_dense_apply_workspace_bytes(int batch, int mn);
LSR_API int lsr_kron_dense_apply_f32(const float* Wh, const float* Wl, const float* X, float* Y, int batch, int mn,
                                     void* ws, size_t ws_bytes, lsr_stream_t stream);
LSR_API int lsr_kron_apply_bf16(const void* A, int a_trans, const void* X, const void* B, float* Y, int batch,
                                int m, int n, int nterms, void* ws, size_t ws_bytes, lsr_stream_t stream);
LSR_API int lsr_kron_apply_f32(const float* A, int a_trans, const float* X, const float* B, float* Y, int batch,
                               int m, int n, int nterms, void* ws, size_t ws_bytes, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Tiny-factor Kronecker reconstruction
 *   W = sum_{s < S} F_0[s] ⊗ F_1[s] ⊗ ... ⊗ F_{K-1}[s]   (fp32, 1 <= K <= 8)
 * factors / rows / cols: HOST arrays of K entries; factor k is a DEVICE array
 * [S][rows[k]][cols[k]]; W is [prod rows][prod cols], row-major, with factor
 * K-1 the fastest-varying mode (torch.kron order).
 * Replaces native_reconstruct / direct_k{3,4,5}_kernel (kron_cuda.py:242-583),
 * generalised from the fixed 16 x 768 K = 3/4/5 layouts to any K <= 8.
 * ---------------------------------------------------------------------- */
LSR_API int lsr_kron_reconstruct_f32(const float* const* factors, const int* rows, const int* cols, int K, int S,
                                     float* W, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Multivariate Hawkes event update, fp32, state [n][D] row-major:
 *   dense: out[i][j] = decay[i] state[i][j] + kcol[event[i]][j]
 *          (kcol = K^T, [D][D], so the selected column is contiguous);
 *   kron : out[i][j] = decay[i] state[i][j] + ka[j / ne][event_asset[i]] ke[j % ne][event_type[i]]
 *          (K = ka ⊗ ke, D = na ne, never formed).
 * Events are int32. An event index out of range is not read: that stream's row
 * is written as NaN and status 110 is recorded in the device status word.
 * out may alias state (in-place update).
 * Replaces hawkes_dense / hawkes_kron and their Triton kernels (hft.py:412-611).
 * ---------------------------------------------------------------------- */
LSR_API int lsr_hawkes_dense_f32(const float* state, const int* event, const float* decay, const float* kcol,
                                 float* out, int n, int d, lsr_stream_t stream);
LSR_API int lsr_hawkes_kron_f32(const float* state, const int* event_asset, const int* event_type,
                                const float* decay, const float* ka, const float* ke, float* out, int n, int na,
                                int ne, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Pauli-string Hamiltonian applied to a state vector of N = 2^K amplitudes,
 * without forming H:
 *   out[r] = sum_s coeff[s] i^{ny[s]} (-1)^{popcount((r ^ flip[s]) & sign[s])} psi[r ^ flip[s]]
 * psi / out: complex amplitudes as separate fp32 real and imaginary arrays of
 * N entries (out must not overlap psi); flip / sign / ny: int32 [S] (flip: X or
 * Y on qubit k sets bit k, sign: Y or Z, ny: number of Y factors, used mod 4),
 * coeff: fp32 [S]. Bits of flip at or above K are ignored. 0 <= K <= 30.
 * Replaces native_apply / pauli_partial_kernel / pauli_reduce_kernel
 * (pauli.py:296-578) in one launch with no partial arrays.
 * ---------------------------------------------------------------------- */
LSR_API int lsr_pauli_apply_f32(const float* psi_r, const float* psi_i, const int* flip, const int* sign,
                                const int* ny, const float* coeff, float* out_r, float* out_i, int K, int S,
                                lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Shampoo / SOAP on stacks of equally shaped parameter blocks
 * ([batch][rows][cols], blocks of at most max_preconditioner_dim per side).
 *
 * Replaces the preconditioner math of DistributedShampoo (third-party
 * distributed_shampoo; constructed in shampoo_soap_lm_ddp_zero1.py:312-400,
 * stepped at :609) for the "shampoo" (Adam grafting) and "soap"
 * (DefaultSOAPConfig) modes. bf16 operands, fp32 accumulation and state.
 *
 * lsr_soap_direction_bf16: with update_stats, first
 *     L = beta2 L + (1-beta2) G G^T,  R = beta2 R + (1-beta2) G^T G;
 *   then G' = Q_L^T G Q_R and Adam in that basis (fused into the rotation):
 *     m = beta1 m + (1-beta1) G',  v = beta2 v + (1-beta2) G'^2,
 *     U' = (m / (1-beta1^step)) / (sqrt(v / (1-beta2^step)) + eps),
 *   and the update direction U = Q_L U' Q_R^T (fp32). G, Q_L and Q_R are the
 *   bf16 operands; every value computed from them that feeds a further GEMM
 *   (the intermediate of each two-sided product, G Q_R or Q_L^T G and then
 *   U' Q_R^T or Q_L U', the cheaper association first, and U' itself) is kept
 *   as a bf16 hi + lo pair, so the result has fp32-level accuracy.
 *   L fp32 [b][r][r], R fp32 [b][c][c], Q_L bf16 [b][r][r], Q_R bf16 [b][c][c],
 *   m, v fp32 [b][r][c]; rows, cols multiples of 8.
 * lsr_shampoo_direction_bf16: optional statistics update as above, then
 *   P = Lroot G Rroot with precomputed bf16 inverse roots Lroot = L^{-1/4},
 *   Rroot = R^{-1/4} (symmetric), one pair per block; P fp32.
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_soap_workspace_bytes(int batch, int rows, int cols);
LSR_API int lsr_soap_direction_bf16(const void* G, float* L, float* R, const void* QL, const void* QR, float* m,
                                    float* v, float* U, int batch, int rows, int cols, float beta1, float beta2,
                                    float eps, int step, int update_stats, void* ws, size_t ws_bytes,
                                    lsr_stream_t stream);
LSR_API size_t lsr_shampoo_workspace_bytes(int batch, int rows, int cols);
LSR_API int lsr_shampoo_direction_bf16(const void* G, float* L, float* R, const void* Lroot, const void* Rroot,
                                       float* P, int batch, int rows, int cols, float beta2, int update_stats,
                                       void* ws, size_t ws_bytes, lsr_stream_t stream);

/* Parameter blocks: ptrs / lds are DEVICE arrays of `nblocks` bf16 block
 * addresses (element (0,0) of the block inside its parameter) and parameter
 * row strides. Gather copies the blocks into stack [nblocks][rows][cols];
 * apply performs the decoupled update p = p (1 - lr wd) - lr U per block
 * (WeightDecayType.DECOUPLED, shampoo_soap_lm_ddp_zero1.py:340). */
LSR_API int lsr_blocks_gather_bf16(const uint64_t* ptrs, const int* lds, int nblocks, int rows, int cols,
                                   void* stack, lsr_stream_t stream);
LSR_API int lsr_blocks_apply_bf16(const uint64_t* ptrs, const int* lds, int nblocks, int rows, int cols,
                                  const float* U, float lr, float weight_decay, lsr_stream_t stream);
/* As lsr_blocks_apply_bf16 with U of element type u_dtype (LSR_DTYPE_*; the
 * ZeRO-1 exchange's communication dtype, shampoo_soap_lm_ddp_zero1.py:341-345,
 * :429-434) and an optional DEVICE index array: block b reads U entry
 * u_index[b] (b when u_index is null), so an all-gathered buffer with padding
 * slots is applied in place. */
LSR_API int lsr_blocks_apply_any(const uint64_t* ptrs, const int* lds, int nblocks, int rows, int cols,
                                 const void* U, int u_dtype, const int* u_index, float lr, float weight_decay,
                                 lsr_stream_t stream);

/* Adam grafting of the Shampoo direction (the reference's "shampoo" mode,
 * grafting_config=AdamPreconditionerConfig(beta2=betas[1], epsilon=1e-8),
 * shampoo_soap_lm_ddp_zero1.py:347-352), on a gradient stack G [b][r][c] bf16:
 * lsr_shampoo_graft_prepare_bf16, per element:
 *     v = gbeta2 v + (1-gbeta2) g^2;
 *     beta1 > 0: m = beta1 m + (1-beta1) g, gf = m / (1-beta1^step); else gf = g;
 *     adam = gf / (sqrt(v / (1-gbeta2^step)) + geps);
 *   Gf = bf16(gf) (the operand of the Shampoo apply), U = adam when U is not
 *   null (steps before the first inverse roots), and per block the partial sums
 *   of adam^2, adam_sq [b][lsr_graft_tiles(r, c)].
 * lsr_shampoo_graft_scale_f32: U[b] *= ||adam_b||_F / max(||U_b||_F, 1e-30),
 *   the grafted Shampoo direction; u_sq is scratch of the same shape as
 *   adam_sq. Both norms are summed in a fixed order per block, so a block's
 *   scale does not depend on which blocks share its stack. m, v fp32 [b][r][c]. */
LSR_API int lsr_graft_tiles(int rows, int cols);
LSR_API int lsr_shampoo_graft_prepare_bf16(const void* G, float* m, float* v, void* Gf, float* U, float* adam_sq,
                                           int batch, int rows, int cols, float beta1, float gbeta2, float geps,
                                           int step, lsr_stream_t stream);
LSR_API int lsr_shampoo_graft_scale_f32(float* U, const float* adam_sq, float* u_sq, int batch, int rows, int cols,
                                        lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Batched coupled Newton inverse roots  X[b] = (A[b] + eps I)^{-1/root}
 *
 * Replaces batched_coupled_newton (shampoo.py:408-542; the recurrence of
 * coupled_newton_one, shampoo.py:277-347): fp32 SPD factors A [batch][n][n],
 * root 2 or 4, per-factor convergence mask (a factor stops when
 * max|M - I| <= tolerance or after max_iterations). Outputs X fp32
 * [batch][n][n], iters int32 [batch] (iterations each factor ran), err fp32
 * [batch] (its final max|M - I|). n a multiple of 4; A, X 16-byte aligned.
 * use_tf32 = 0 (the reference runs with TF32 off): the recurrence in fp32
 * FFMA on the CUDA cores, the reference's numerics (symmetric products
 * computed as upper triangles and mirrored). use_tf32 = 1: the products run
 * as 3xTF32 on the tensor cores until max|M - I| <= 1e-4, then in fp32
 * FFMA to the tolerance (X then within ~1e-4 of the fp32 result on
 * well-conditioned factors); factors that needed more than
 * 14 (root 2) / 13 (root 4) iterations (ill-conditioned ones, where the
 * tensor cores' truncating accumulation costs accuracy) are then recomputed
 * from scratch in fp32 FFMA, as the reference's hybrid path recomputes its
 * hard factors (shampoo.py:545-595), and redo (int32 [batch], may be NULL)
 * receives 1 for them. iters counts the recurrence's iterations, err is the
 * final max|M - I|.
 * check_every = k > 0: every k iterations
 * the host reads the number of active factors (a stream synchronization) and
 * stops when it is 0; check_every = 0: no host synchronization, always
 * max_iterations rounds of launches (converged factors skip all work).
 * ---------------------------------------------------------------------- */
LSR_API size_t lsr_coupled_newton_workspace_bytes(int batch, int n);
LSR_API int lsr_coupled_newton_f32(const float* A, float* X, int* iters, float* err, int* redo, int batch, int n,
                                   int root, float epsilon, float tolerance, int max_iterations, int check_every,
                                   int use_tf32, void* ws, size_t ws_bytes, lsr_stream_t stream);

/* ------------------------------------------------------------------------
 * Peer-memory exchange of finished parameter shards (sharded Muon step).
 *
 * Replaces the exchange step of the distributed paths: the DDP all-reduce
 * that keeps replicated Muon parameters equal (muon_lm_ddp.py:1270-1278) and
 * the ZeRO-1 all-gather of DDPDistributedConfig
 * (shampoo_soap_lm_ddp_zero1.py:341-345). Each rank keeps a replica of every
 * flat, rank-major parameter buffer in memory the other ranks open through
 * CUDA IPC; after applying its own updates it stores its shard into every
 * peer's replica at the same byte offset (lsr_peer_push), then the ranks meet
 * at a barrier. No counterpart function exists in the reference.
 *
 * lsr_ipc_alloc: cudaMalloc `bytes` and export them; `handle` (host) receives
 *   LSR_IPC_HANDLE_BYTES bytes to send to the other ranks.
 * lsr_ipc_open / lsr_ipc_close: map / unmap another process's buffer.
 * lsr_ipc_free: release a buffer made by lsr_ipc_alloc.
 * lsr_peer_push: for q < npeers store bytes [src, src + bytes) at
 *   src + peer_deltas[q] (host array; the byte distance from the local buffer
 *   to peer q's mapped replica, a multiple of 16). `bytes` even; up to
 *   `max_ctas` CTAs (<= 0: one per SM). The CTAs use no shared memory, so they
 *   run beside the library's GEMM kernels.
 * The ipc functions allocate or map memory by design; the push allocates
 * nothing.
 * ---------------------------------------------------------------------- */
#define LSR_IPC_HANDLE_BYTES 64
#define LSR_MAX_PEERS 15
LSR_API int lsr_ipc_alloc(size_t bytes, void** ptr, void* handle);
LSR_API int lsr_ipc_open(const void* handle, void** ptr);
LSR_API int lsr_ipc_close(void* ptr);
LSR_API int lsr_ipc_free(void* ptr);
LSR_API int lsr_peer_push(const void* src, size_t bytes, const long long* peer_deltas, int npeers, int max_ctas,
                          lsr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LSR_H_ */
