// Batched Householder QR of square fp32 matrices (n <= 1024) and the SOAP
// eigenbasis refresh built on it.
//
// The SOAP refresh is one step (or a few) of power iteration per
// preconditioner factor S (the statistics L or R of a block):
//     W = (S + eps I) Q_prev,   Q_new R = W   (Householder QR),
// with the signs of Q_new's columns chosen so that diag(R) > 0, so a basis
// that has converged comes back unchanged (Q_new = Q_prev, no sign flips) and
// the Adam moments kept in the rotated basis stay aligned with it. Starting
// from Q_prev = I this converges to the eigenvectors of S; run every
// precondition_frequency steps it tracks them as S drifts. This replaces an
// eigendecomposition per refresh (torch.linalg.eigh) with GEMMs on the tcgen05
// engine (3xTF32, fp32-level accuracy) and one QR kernel.
//
// QR: blocked Householder with panels of 32 columns (the compact WY form
// H_1 ... H_32 = I - V T V^T), one CTA per matrix:
//   * qr_factor_kernel: for each panel, the panel (<= 1024 x 32) is factored
//     in shared memory, column by column (each column one norm reduction and
//     one 32-wide reduction that yields both the trailing-column dot products
//     and the column of T); V and R are written back in place, then the rest
//     of the matrix is updated, A2 -= V T^T (V^T A2), one thread per column;
//   * qr_form_q_kernel: Q = H_0 ... H_{P-1} accumulated backwards from I,
//     Q2 -= V T (V^T Q2), then column signs so that diag(R) > 0.
// FP32 FMA throughout (the factorization is O(n^3) SIMT work per matrix,
// matrices run side by side, one per SM).
#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int QR_NB = 32;
constexpr int QR_THREADS = 256;
constexpr int QR_WARPS = QR_THREADS / 32;
constexpr int QR_MAXN = 1024;
constexpr int QR_LDP = 33;  // panel row stride in shared memory (conflict-free column reads)

constexpr size_t qr_smem_bytes() {
  return ((size_t)QR_MAXN * QR_LDP + QR_NB * QR_LDP + QR_WARPS * 32 + 64) * sizeof(float);
}

// Sum over the block; every thread gets the total.
__device__ __forceinline__ float qr_block_sum(float v, float* red, float* out) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < QR_WARPS ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) *out = t;
  }
  __syncthreads();
  return *out;
}

// 32 per-thread partial sums -> out[c] = sum over the block of acc[c]
// (warp reduce-scatter with 31 shuffles, then across warps).
__device__ __forceinline__ void qr_block_sum32(float (&acc)[32], float* red, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      const float keep = hi ? acc[o + k] : acc[k];
      const float send = hi ? acc[k] : acc[o + k];
      acc[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  red[warp * 32 + lane] = acc[0];  // lane l holds the warp's sum for value l
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
    for (int w = 0; w < QR_WARPS; ++w) t += red[w * 32 + lane];
    out[lane] = t;
  }
  __syncthreads();
}

// Block-reflector update of column pairs of a trailing matrix C (m rows, row
// stride n): C -= V X (V^T C), X = T^T (factorization: H_1 ... H_w applied
// transposed) or X = T (forming Q). V [m][32] is in shared memory with rows of
// 32 floats (16-byte aligned) and its unit lower-trapezoidal form written out
// (ones on the diagonal, zeros above), so every row is read as eight 16-byte
// broadcasts and no row needs a select. Each thread owns columns c and
// c + QR_THREADS, so every V value read feeds two FMA chains; rows go in
// batches of QR_ROWB, their loads issued together (the matrix streams from L2 /
// DRAM: one load in flight per thread would leave the kernel latency-bound).
constexpr int QR_ROWB = 8;
constexpr int QR_VLD = 32;  // row stride of the compacted V

__device__ __forceinline__ void v_row(const float* V, int i, float (&v)[32]) {
  const float4* r4 = reinterpret_cast<const float4*>(V + i * QR_VLD);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 t = r4[q];
    v[4 * q] = t.x;
    v[4 * q + 1] = t.y;
    v[4 * q + 2] = t.z;
    v[4 * q + 3] = t.w;
  }
}

template <bool TRANS_T>
__device__ __forceinline__ void wy_update_cols(float* C, int n, int m, int ncols, int w, const float* V,
                                               const float* Ts) {
  for (int c0 = threadIdx.x; c0 < ncols; c0 += 2 * QR_THREADS) {
    const int c1 = c0 + QR_THREADS;
    const bool has1 = c1 < ncols;
    float* col0 = C + c0;
    float* col1 = C + (has1 ? c1 : c0);
    float a0[32], a1[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) a0[k] = a1[k] = 0.f;
    int i = 0;
    for (; i + QR_ROWB <= m; i += QR_ROWB) {
      float x0[QR_ROWB], x1[QR_ROWB];
#pragma unroll
      for (int u = 0; u < QR_ROWB; ++u) {
        x0[u] = col0[(size_t)(i + u) * n];
        x1[u] = col1[(size_t)(i + u) * n];
      }
#pragma unroll
      for (int u = 0; u < QR_ROWB; ++u) {
        float v[32];
        v_row(V, i + u, v);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          a0[k] = fmaf(v[k], x0[u], a0[k]);
          a1[k] = fmaf(v[k], x1[u], a1[k]);
        }
      }
    }
    for (; i < m; ++i) {
      const float x0 = col0[(size_t)i * n], x1 = col1[(size_t)i * n];
      float v[32];
      v_row(V, i, v);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        a0[k] = fmaf(v[k], x0, a0[k]);
        a1[k] = fmaf(v[k], x1, a1[k]);
      }
    }
    // y = X a in place (T upper triangular): T^T a needs a[0..k] for y[k], so
    // k runs downwards; T a needs a[k..31], so k runs upwards
    if (TRANS_T) {
#pragma unroll
      for (int k = 31; k >= 0; --k) {
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int r = 0; r <= k; ++r) {
          t0 = fmaf(Ts[r * QR_LDP + k], a0[r], t0);
          t1 = fmaf(Ts[r * QR_LDP + k], a1[r], t1);
        }
        a0[k] = k < w ? t0 : 0.f;
        a1[k] = k < w ? t1 : 0.f;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int r = k; r < 32; ++r) {
          t0 = fmaf(Ts[k * QR_LDP + r], a0[r], t0);
          t1 = fmaf(Ts[k * QR_LDP + r], a1[r], t1);
        }
        a0[k] = k < w ? t0 : 0.f;
        a1[k] = k < w ? t1 : 0.f;
      }
    }
    // C[i] -= sum_k V[i][k] y[k]
    int r = 0;
    for (; r + QR_ROWB <= m; r += QR_ROWB) {
      float x0[QR_ROWB], x1[QR_ROWB];
#pragma unroll
      for (int u = 0; u < QR_ROWB; ++u) {
        x0[u] = col0[(size_t)(r + u) * n];
        x1[u] = col1[(size_t)(r + u) * n];
      }
#pragma unroll
      for (int u = 0; u < QR_ROWB; ++u) {
        float v[32];
        v_row(V, r + u, v);
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          d0 = fmaf(v[k], a0[k], d0);
          d1 = fmaf(v[k], a1[k], d1);
        }
        col0[(size_t)(r + u) * n] = x0[u] - d0;
        if (has1) col1[(size_t)(r + u) * n] = x1[u] - d1;
      }
    }
    for (; r < m; ++r) {
      float v[32];
      v_row(V, r, v);
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        d0 = fmaf(v[k], a0[k], d0);
        d1 = fmaf(v[k], a1[k], d1);
      }
      col0[(size_t)r * n] -= d0;
      if (has1) col1[(size_t)r * n] -= d1;
    }
  }
}

// Rewrites the factored panel P ([m][QR_LDP]: V below the diagonal) in place as
// the compacted V [m][QR_VLD] with its unit lower-trapezoidal form written out.
// Chunks of 32 rows go in order, each read completely before it is written:
// chunk c's destination ends below chunk c+1's source (1024 (c+1) <= 1056 (c+1)).
__device__ __forceinline__ void compact_panel(float* P, int m, int w) {
  for (int c0 = 0; c0 < m; c0 += 32) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = threadIdx.x + q * QR_THREADS, i = c0 + idx / 32, k = idx % 32;
      v[q] = 0.f;
      if (i < m && k < w) v[q] = k < i ? P[i * QR_LDP + k] : (k == i ? 1.f : 0.f);
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = threadIdx.x + q * QR_THREADS, i = c0 + idx / 32, k = idx % 32;
      if (i < m) P[i * QR_VLD + k] = v[q];
    }
    __syncthreads();
  }
}

// A [b][n][n] (row-major) is factored in place: R on and above the diagonal,
// the Householder vectors (unit leading entry implied) below it; tau [b][n];
// T [b][P][32][32] the upper-triangular WY factor of each panel.
__global__ void __launch_bounds__(QR_THREADS, 1) qr_factor_kernel(float* A, float* tau, float* T, int n) {
  extern __shared__ float qsm[];
  float* P = qsm;                          // [m][QR_LDP] panel
  float* Ts = P + QR_MAXN * QR_LDP;        // [32][QR_LDP]
  float* red = Ts + QR_NB * QR_LDP;        // [QR_WARPS * 32]
  float* sh = red + QR_WARPS * 32;         // [64] reduction results
  const int b = blockIdx.x, tid = threadIdx.x;
  float* Ab = A + (size_t)b * n * n;
  const int npan = (n + QR_NB - 1) / QR_NB;
  for (int p = 0; p < npan; ++p) {
    const int c0 = p * QR_NB, w = min(QR_NB, n - c0), m = n - c0;
    for (int idx = tid; idx < m * QR_NB; idx += QR_THREADS) {
      const int i = idx / QR_NB, j = idx % QR_NB;
      P[i * QR_LDP + j] = j < w ? Ab[(size_t)(c0 + i) * n + c0 + j] : 0.f;
    }
    for (int idx = tid; idx < QR_NB * QR_LDP; idx += QR_THREADS) Ts[idx] = 0.f;
    __syncthreads();
    for (int j = 0; j < w; ++j) {
      float s = 0.f;
      for (int i = j + 1 + tid; i < m; i += QR_THREADS) {
        const float x = P[i * QR_LDP + j];
        s = fmaf(x, x, s);
      }
      const float sigma = qr_block_sum(s, red, sh + 32);
      const float alpha = P[j * QR_LDP + j];
      float tj = 0.f, beta = alpha, scale = 0.f;
      if (sigma > 0.f) {
        const float nrm = sqrtf(fmaf(alpha, alpha, sigma));
        beta = alpha >= 0.f ? -nrm : nrm;
        tj = (beta - alpha) / beta;
        scale = 1.f / (alpha - beta);
      }
      for (int i = j + 1 + tid; i < m; i += QR_THREADS) P[i * QR_LDP + j] *= scale;
      __syncthreads();
      if (tid == 0) P[j * QR_LDP + j] = beta;
      // d[c] = sum_{i >= j} v_i P[i][c] (v_j = 1): for c > j the trailing
      // columns' dot products, for c < j the products V[:, c]^T v that build T
      float acc[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) acc[c] = 0.f;
      for (int i = j + tid; i < m; i += QR_THREADS) {
        const float vi = i == j ? 1.f : P[i * QR_LDP + j];
        const float* row = P + i * QR_LDP;
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = fmaf(vi, (i == j && c == j) ? 0.f : row[c], acc[c]);
      }
      qr_block_sum32(acc, red, sh);
      // trailing panel columns: P[i][c] -= tau_j d[c] v_i   (i >= j, c > j)
      for (int i = j + tid; i < m; i += QR_THREADS) {
        const float vi = i == j ? 1.f : P[i * QR_LDP + j];
        for (int c = j + 1; c < w; ++c) P[i * QR_LDP + c] = fmaf(-tj * sh[c], vi, P[i * QR_LDP + c]);
      }
      // T column j: T[r][j] = -tau_j sum_{r <= k < j} T[r][k] d[k], T[j][j] = tau_j
      if (tid < j) {
        float t = 0.f;
        for (int k = tid; k < j; ++k) t = fmaf(Ts[tid * QR_LDP + k], sh[k], t);
        Ts[tid * QR_LDP + j] = -tj * t;
      }
      if (tid == j) {
        Ts[j * QR_LDP + j] = tj;
        tau[(size_t)b * n + c0 + j] = tj;
      }
      __syncthreads();
    }
    // panel back to A (R and V), T to global
    for (int idx = tid; idx < m * QR_NB; idx += QR_THREADS) {
      const int i = idx / QR_NB, j = idx % QR_NB;
      if (j < w) Ab[(size_t)(c0 + i) * n + c0 + j] = P[i * QR_LDP + j];
    }
    for (int idx = tid; idx < QR_NB * QR_NB; idx += QR_THREADS)
      T[((size_t)b * npan + p) * QR_NB * QR_NB + idx] = Ts[(idx / QR_NB) * QR_LDP + idx % QR_NB];
    // trailing matrix: A2 (rows c0.., cols c0+w..) -= V T^T (V^T A2)
    if (n - c0 - w > 0) {
      compact_panel(P, m, w);
      wy_update_cols<true>(Ab + (size_t)c0 * n + c0 + w, n, m, n - c0 - w, w, P, Ts);
    }
    __syncthreads();
  }
}

// Q [b][n][n] = H_0 ... H_{P-1} (from the factored A, tau, T), then column j
// multiplied by sign(R[j][j]) so that the triangular factor has a positive diagonal.
__global__ void __launch_bounds__(QR_THREADS, 1) qr_form_q_kernel(const float* A, const float* T, float* Q, int n) {
  extern __shared__ float qsm[];
  float* P = qsm;
  float* Ts = P + QR_MAXN * QR_LDP;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* Ab = A + (size_t)b * n * n;
  float* Qb = Q + (size_t)b * n * n;
  const int npan = (n + QR_NB - 1) / QR_NB;
  for (int idx = tid; idx < n * n; idx += QR_THREADS) Qb[idx] = (idx / n == idx % n) ? 1.f : 0.f;
  __syncthreads();
  for (int p = npan - 1; p >= 0; --p) {
    const int c0 = p * QR_NB, w = min(QR_NB, n - c0), m = n - c0;
    for (int idx = tid; idx < m * QR_NB; idx += QR_THREADS) {
      const int i = idx / QR_NB, j = idx % QR_NB;
      P[i * QR_VLD + j] = j < w ? (i > j ? Ab[(size_t)(c0 + i) * n + c0 + j] : (i == j ? 1.f : 0.f)) : 0.f;
    }
    for (int idx = tid; idx < QR_NB * QR_NB; idx += QR_THREADS)
      Ts[(idx / QR_NB) * QR_LDP + idx % QR_NB] = T[((size_t)b * npan + p) * QR_NB * QR_NB + idx];
    __syncthreads();
    // Q2 (rows c0.., cols c0..) -= V T (V^T Q2)
    wy_update_cols<false>(Qb + (size_t)c0 * n + c0, n, m, m, w, P, Ts);
    __syncthreads();
  }
  for (int c = tid; c < n; c += QR_THREADS) {
    if (Ab[(size_t)c * n + c] < 0.f) {
      for (int i = 0; i < n; ++i) Qb[(size_t)i * n + c] = -Qb[(size_t)i * n + c];
    }
  }
}

// W = S + eps I (the first power-iteration step from the identity basis).
__global__ void add_diag_kernel(const float* S, float* W, int n, float eps, long long total) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const long long in_mat = e % ((long long)n * n);
    W[e] = S[e] + ((in_mat / n == in_mat % n) ? eps : 0.f);
  }
}

// y += a x
__global__ void axpy_kernel(const float* x, float* y, long long total, float a) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x)
    y[e] = fmaf(a, x[e], y[e]);
}

__global__ void to_bf16_kernel(const float* x, __nv_bfloat16* y, long long total) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x)
    y[e] = __float2bfloat16_rn(x[e]);
}

int ew_blocks(long long total) { return (int)std::max<long long>(1, std::min<long long>((total + 255) / 256, 148LL * 32)); }

size_t a256q(size_t x) { return align_up(x, 256); }

}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

size_t lsr_qr_workspace_bytes(int batch, int n) {
  if (batch < 0 || n <= 0 || n > QR_MAXN) return 0;
  const size_t b = (size_t)std::max(batch, 1);
  const size_t npan = (size_t)(n + QR_NB - 1) / QR_NB;
  return a256q(b * n * 4) + a256q(b * npan * QR_NB * QR_NB * 4) + 256;  // tau, T
}

int lsr_householder_qr_f32(float* W, float* Q, int batch, int n, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (batch < 0 || batch > 65535 || n <= 0) return LSR_ERR_ARG;
  if (n > QR_MAXN) return LSR_ERR_SHAPE;
  if (batch == 0) return LSR_OK;
  if (!W || !Q || W == Q) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_qr_workspace_bytes(batch, n)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  float* tau = reinterpret_cast<float*>(w);
  float* T = reinterpret_cast<float*>(w + a256q((size_t)batch * n * 4));
  const int smem = (int)qr_smem_bytes();
  if (cudaFuncSetAttribute(qr_factor_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(qr_form_q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return LSR_ERR_LAUNCH;
  {
    ProfScope prof(PK_EW_OTHER, st);
    qr_factor_kernel<<<batch, QR_THREADS, smem, st>>>(W, tau, T, n);
  }
  if (cudaGetLastError() != cudaSuccess) return LSR_ERR_LAUNCH;
  ProfScope prof(PK_EW_OTHER, st);
  qr_form_q_kernel<<<batch, QR_THREADS, smem, st>>>(W, T, Q, n);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

size_t lsr_eigenbasis_refresh_workspace_bytes(int batch, int n) {
  const size_t q = lsr_qr_workspace_bytes(batch, n);
  if (!q) return 0;
  const size_t mat = a256q((size_t)std::max(batch, 1) * n * n * 4);
  return q + mat + lsr_gemm_f32_workspace_bytes(batch, n, n, n) + 256;  // + W + the fp32 GEMM's tf32 pairs
}

int lsr_eigenbasis_refresh_f32(const float* S, float* Qf, void* Qb, int batch, int n, float eps, int from_identity,
                               int iterations, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (batch < 0 || batch > 65535 || n <= 0 || iterations < 1) return LSR_ERR_ARG;
  if (n > QR_MAXN) return LSR_ERR_SHAPE;
  if (batch == 0) return LSR_OK;
  if (!S || !Qf) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_eigenbasis_refresh_workspace_bytes(batch, n)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  const long long total = (long long)batch * n * n;
  float* W = reinterpret_cast<float*>(w);
  uint8_t* qws = w + a256q((size_t)total * 4);
  const size_t qbytes = lsr_qr_workspace_bytes(batch, n);
  uint8_t* gws = qws + qbytes;
  const size_t gbytes = lsr_gemm_f32_workspace_bytes(batch, n, n, n);
  for (int it = 0; it < iterations; ++it) {
    if (it == 0 && from_identity) {
      ProfScope prof(PK_EW_OTHER, st);
      add_diag_kernel<<<ew_blocks(total), 256, 0, st>>>(S, W, n, eps, total);
      if (cudaGetLastError() != cudaSuccess) return LSR_ERR_LAUNCH;
    } else {
      // W = S Q (fp32 via 3xTF32) + eps Q
      rc = lsr_gemm_f32(S, Qf, W, batch, n, n, n, 1.f, gws, gbytes, stream);
      if (rc) return rc;
      if (eps != 0.f) {
        ProfScope prof(PK_EW_OTHER, st);
        axpy_kernel<<<ew_blocks(total), 256, 0, st>>>(Qf, W, total, eps);
        if (cudaGetLastError() != cudaSuccess) return LSR_ERR_LAUNCH;
      }
    }
    rc = lsr_householder_qr_f32(W, Qf, batch, n, qws, qbytes, stream);
    if (rc) return rc;
  }
  if (Qb) {
    ProfScope prof(PK_EW_OTHER, st);
    to_bf16_kernel<<<ew_blocks(total), 256, 0, st>>>(Qf, static_cast<__nv_bfloat16*>(Qb), total);
    if (cudaGetLastError() != cudaSuccess) return LSR_ERR_LAUNCH;
  }
  return LSR_OK;
}

}  // extern "C"
