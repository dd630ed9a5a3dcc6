// Kronecker operators on the tcgen05 engine (gemm_sm100.cuh).
//
//   Kronecker sum    (A ⊕ B) vec(X) = vec(A X + X B^T)          one kernel, one
//                    accumulator: the two products are two K segments of the
//                    same tile, so A ⊗ I and I ⊗ B are never formed.
//   Kronecker apply  Y = Σ_s A_s X B_s^T  (row-major vec: (A ⊗ B) vec(X))
//                    two chained GEMMs per term; the intermediate is written as
//                    a hi + lo pair by the first GEMM's epilogue so that the
//                    second product keeps fp32-level accuracy.
//
// Reference: hft_fused.py:89-319 (kron_sum_64x8_kernel, S-term apply, SIMT fp32)
// and hft.py:108-140 / hft_fused.py:463-509 (kron_apply_shared_2d, torch).
//
// bf16 variants: bf16 operands, fp32 accumulation, fp32 output.
// fp32 variants: every fp32 operand x is split as hi = tf32(x), lo = x - hi and
// each product a*b is evaluated as hi*hi + hi*lo + lo*hi on kind::tf32 tensor
// cores (the "3xTF32" emulation of fp32 GEMM); the neglected lo*lo term and
// the tf32 truncation of lo are below 2^-21 relative. tf32 operands are always
// given to the tensor core K-major (MN-major tf32 operands read as zero on this
// part): the split pass writes a transposed copy where a product needs one, and
// the intermediate of a right-first apply is stored transposed by its epilogue.
#include <atomic>

#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int K_BN = 256;
constexpr int SPLIT_THREADS = 256;

// hi = tf32(x), lo = x - hi over n elements.
__global__ void __launch_bounds__(SPLIT_THREADS) split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                                                   float* __restrict__ lo, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float h = tf32_hi(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// Transposing split: for each of `batch` R x C matrices, hi[b][c][r] = tf32(x[b][r][c]),
// lo = x - hi. One block per 32x32 tile (blockIdx.z = matrix).
__global__ void __launch_bounds__(SPLIT_THREADS) split_tf32_t_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                                                     float* __restrict__ lo, int R, int C) {
  __shared__ float tile[32][33];
  const long long base = (long long)blockIdx.z * R * C;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows per pass
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < R && c < C) ? x[base + (long long)r * C + c] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + tx;  // output row c, column r
    if (c < C && r < R) {
      const float v = tile[tx][i];
      const float h = tf32_hi(v);
      hi[base + (long long)c * R + r] = h;
      lo[base + (long long)c * R + r] = v - h;
    }
  }
}

int launch_ok() { return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH; }

int split_tf32(const float* x, float* hi, float* lo, long long n, cudaStream_t st) {
  if (n <= 0) return LSR_OK;
  const int blocks = (int)std::min<long long>((n + SPLIT_THREADS - 1) / SPLIT_THREADS, 148LL * 16);
  ProfScope prof(PK_EW_OTHER, st);
  split_tf32_kernel<<<blocks, SPLIT_THREADS, 0, st>>>(x, hi, lo, n);
  return launch_ok();
}

// Split `batch` R x C matrices into transposed hi/lo copies ([batch][C][R]).
int split_tf32_t(const float* x, float* hi, float* lo, int batch, int R, int C, cudaStream_t st) {
  if (batch <= 0) return LSR_OK;
  ProfScope prof(PK_EW_OTHER, st);
  split_tf32_t_kernel<<<dim3(cdiv(C, 32), cdiv(R, 32), batch), SPLIT_THREADS, 0, st>>>(x, hi, lo, R, C);
  return launch_ok();
}

size_t a256(size_t x) { return align_up(x, 256); }

bool kron_dims_ok(int batch, int m, int n, int nterms) {
  return batch >= 0 && batch <= 65535 && m > 0 && n > 0 && nterms > 0 && nterms <= 65535;
}

// Small factors (m n <= 1024, m n % 4 == 0): the fp32 apply forms the dense
// operator W = sum_s A_s (x) B_s once ((m n)^2 entries, at most 4 MB) and runs
// Y_flat = X_flat W^T as ONE tensor-core GEMM over every right-hand side
// (rows = batch, K = N = m n), instead of 2 S chained GEMMs of m x n tiles that
// would fill a fraction of a 128 x 256 tile each. This is the shape of
// hft_fused.py's own kron_sum_64x8_kernel workload (x [M, 64, 8], S terms).
constexpr int kDenseMaxMN = 1024;
bool kron_use_dense(int m, int n) {
  const long long mn = (long long)m * n;
  return mn <= kDenseMaxMN && mn % 4 == 0;
}

// Small fp32 problems (m <= 64, n in {1, 2, 4, 8, 16}): one FFMA launch with no
// workspace (kron_small_kernel) when a cost model says it beats the dense
// operator's tensor-core GEMM. The model was fitted on B200 to the reference's
// x [M, 64, 8] sweep (M 256..16384, S 1..8; microseconds per call):
//   small ≈ 4 + (X + Y bytes) / 2.2 TB/s + S (1.2 + term flops / 26 TFLOP/s)
//   dense ≈ max(31, 18.6 + 3xTF32 flops / 452 TFLOP/s)
// The FFMA kernel pays a latency per term; the dense GEMM has a launch floor and
// a handful of 128 x 256 tiles whose K loop runs 3 (m n / 32) blocks in series.
constexpr int KS_THREADS = 256;

bool kron_use_small(int batch, int m, int n, int nterms) {
  if (m > 64 || n > 16 || 32 % n) return false;
  const double mn = (double)m * n;
  const double small_us = 4.0 + 8.0 * batch * mn / 2.2e6 +
                          nterms * (1.2 + 2.0 * batch * mn * (m + n) / 26.0e6);
  if (mn > kDenseMaxMN || (m * n) % 4) return true;  // no dense path for these factors
  const double dense_us = std::max(31.0, 18.6 + 6.0 * batch * mn * mn / 452.0e6);
  return small_us < dense_us;
}

// W[(i n + j)][(k n + l)] = sum_s A_s[i][k] B_s[j][l]  (A_s[i][k] = at[s][k][i] when a_trans),
// written as a tf32 hi / lo pair.
__global__ void __launch_bounds__(SPLIT_THREADS) kron_dense_w_kernel(const float* __restrict__ A, int a_trans,
                                                                     const float* __restrict__ B, int m, int n, int S,
                                                                     float* __restrict__ Wh, float* __restrict__ Wl) {
  const int mn = m * n;
  const long long total = (long long)mn * mn;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(e / mn), col = (int)(e % mn);
    const int i = row / n, j = row % n, k = col / n, l = col % n;
    float acc = 0.f;
    for (int s = 0; s < S; ++s) {
      const float a = a_trans ? A[((long long)s * m + k) * m + i] : A[((long long)s * m + i) * m + k];
      acc = fmaf(a, B[((long long)s * n + j) * n + l], acc);
    }
    const float h = tf32_hi(acc);
    Wh[e] = h;
    Wl[e] = acc - h;
  }
}

// Operand helpers (all matrices row-major).
//   mat(base, rows, cols, batch, mn, f32): `batch` matrices rows x cols, ld = cols.
Operand mat(const void* base, int rows, int cols, int batch, int mn, int f32) {
  Operand o{base, rows, cols, cols, (long long)rows * cols, batch, mn};
  o.f32 = f32;
  return o;
}

}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

// ---------------------------------------------------------------------------
// Kronecker sum
// ---------------------------------------------------------------------------

size_t lsr_kron_sum_workspace_bytes(int batch, int m, int n, int f32) {
  if (!kron_dims_ok(batch, m, n, 1)) return 0;
  if (!f32) return 0;
  // hi/lo copies of A, B, X and X^T
  return 2 * (a256((size_t)m * m * 4) + a256((size_t)n * n * 4) + 2 * a256((size_t)batch * m * n * 4)) + 256;
}

int lsr_kron_sum_bf16(const void* A, const void* X, const void* B, float* Y, int batch, int m, int n,
                      lsr_stream_t stream) {
  if (!kron_dims_ok(batch, m, n, 1)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !X || !B || !Y) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  G.batch = batch;
  G.M = m;
  G.N = n;
  G.nseg = 2;
  // segment 0: A (K-major, shared) x X (MN-major): sum_k A[r][k] X[k][c]
  G.seg[0] = SegDesc{cdiv(m, BK), 0, 1, 1, 0};
  G.seg[1] = SegDesc{cdiv(n, BK), 0, 0, 0, 1};
  rc = make_operand_map(&p.mapA[0][0], mat(A, m, m, 1, 0, 0), false, K_BN);
  if (!rc) rc = make_operand_map(&p.mapB[0][0], mat(X, m, n, batch, 1, 0), true, K_BN, &G.seg[0].b_mn);
  // segment 1: X (K-major) x B (K-major, shared): sum_k X[r][k] B[c][k]
  if (!rc) rc = make_operand_map(&p.mapA[0][1], mat(X, m, n, batch, 0, 0), false, K_BN);
  if (!rc) rc = make_operand_map(&p.mapB[0][1], mat(B, n, n, 1, 0, 0), true, K_BN);
  if (rc) return rc;
  G.out = Y;
  G.out_bs = (long long)m * n;
  G.ldo = n;
  G.alpha = 1.f;
  return launch_gemm<K_BN, EPI_STORE_F32>(p, reinterpret_cast<cudaStream_t>(stream));
}

int lsr_kron_sum_f32(const float* A, const float* X, const float* B, float* Y, int batch, int m, int n, void* ws,
                     size_t ws_bytes, lsr_stream_t stream) {
  if (!kron_dims_ok(batch, m, n, 1)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !X || !B || !Y) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_kron_sum_workspace_bytes(batch, m, n, 1)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  float* Ah = reinterpret_cast<float*>(w);
  float* Al = reinterpret_cast<float*>(w += a256((size_t)m * m * 4));
  float* Bh = reinterpret_cast<float*>(w += a256((size_t)m * m * 4));
  float* Bl = reinterpret_cast<float*>(w += a256((size_t)n * n * 4));
  float* Xh = reinterpret_cast<float*>(w += a256((size_t)n * n * 4));
  float* Xl = reinterpret_cast<float*>(w += a256((size_t)batch * m * n * 4));
  float* Xth = reinterpret_cast<float*>(w += a256((size_t)batch * m * n * 4));
  float* Xtl = reinterpret_cast<float*>(w += a256((size_t)batch * m * n * 4));
  rc = split_tf32(A, Ah, Al, (long long)m * m, st);
  if (!rc) rc = split_tf32(B, Bh, Bl, (long long)n * n, st);
  if (!rc) rc = split_tf32(X, Xh, Xl, (long long)batch * m * n, st);
  if (!rc) rc = split_tf32_t(X, Xth, Xtl, batch, m, n, st);
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  G.batch = batch;
  G.M = m;
  G.N = n;
  G.nseg = 6;
  const float* left[3][2] = {{Ah, Xth}, {Ah, Xtl}, {Al, Xth}};  // A X   : hi*hi + hi*lo + lo*hi
  const float* right[3][2] = {{Xh, Bh}, {Xh, Bl}, {Xl, Bh}};     // X B^T : hi*hi + hi*lo + lo*hi
  for (int t = 0; t < 3 && !rc; ++t) {
    // A X: B operand element (c, k) = X[k][c] = X^T[c][k], K-major in the transposed copy
    rc = make_operand_map(&p.mapA[0][t], mat(left[t][0], m, m, 1, 0, 1), false, K_BN);
    if (!rc) rc = make_operand_map(&p.mapB[0][t], mat(left[t][1], n, m, batch, 0, 1), true, K_BN);
    if (!rc) rc = make_operand_map(&p.mapA[0][3 + t], mat(right[t][0], m, n, batch, 0, 1), false, K_BN);
    if (!rc) rc = make_operand_map(&p.mapB[0][3 + t], mat(right[t][1], n, n, 1, 0, 1), true, K_BN);
    G.seg[t] = SegDesc{cdiv(m, BK_TF32), 0, 0, 1, 0, t > 0};
    G.seg[3 + t] = SegDesc{cdiv(n, BK_TF32), 0, 0, 0, 1, t > 0};
  }
  if (rc) return rc;
  G.out = Y;
  G.out_bs = (long long)m * n;
  G.ldo = n;
  G.alpha = 1.f;
  return launch_gemm<K_BN, EPI_STORE_F32, default_stages<EPI_STORE_F32>(), 1, 1>(p, st);
}

// ---------------------------------------------------------------------------
// Kronecker apply  Y[i] = sum_s A_s X[i] B_s^T
// ---------------------------------------------------------------------------

size_t lsr_kron_apply_workspace_bytes(int batch, int m, int n, int nterms, int f32) {
  if (!kron_dims_ok(batch, m, n, nterms)) return 0;
  const size_t mn = (size_t)batch * m * n;
  if (!f32) return 2 * a256(mn * 2) + 256;  // bf16 hi/lo intermediate
  if (kron_use_small(batch, m, n, nterms)) return 0;  // one FFMA launch, no workspace
  if (kron_use_dense(m, n)) {
    const size_t w = (size_t)m * n * m * n * 4;
    return 2 * a256(w) + 2 * a256(mn * 4) + 256;  // W hi/lo, X hi/lo
  }
  // fp32: hi/lo of A (K-major), B, X (one orientation) and of the fp32 intermediate
  return 2 * (a256((size_t)nterms * m * m * 4) + a256((size_t)nterms * n * n * 4) + a256(mn * 4) + a256(mn * 4)) +
         256;
}

}  // extern "C"

namespace lsr {
namespace {

// Fill one GEMM group from a list of (A operand, B operand) pairs.
int set_segments(GemmParams& p, const Operand (*pairs)[2], const SegDesc* segs, int nseg) {
  int rc = 0;
  for (int t = 0; t < nseg && !rc; ++t) {
    p.g[0].seg[t] = segs[t];
    rc = make_operand_map(&p.mapA[0][t], pairs[t][0], false, K_BN, &p.g[0].seg[t].a_mn);
    if (!rc) rc = make_operand_map(&p.mapB[0][t], pairs[t][1], true, K_BN, &p.g[0].seg[t].b_mn);
  }
  p.g[0].nseg = nseg;
  return rc;
}

void set_out(GroupDesc& G, int batch, int m, int n, void* out, void* out2, int out_trans) {
  G.batch = batch;
  G.M = m;
  G.N = n;
  G.out = out;
  G.out2 = out2;
  G.out_bs = (long long)m * n;
  G.ldo = out_trans ? m : n;
  G.out_trans = out_trans;
  G.alpha = 1.f;
}

}  // namespace

// One term, bf16 operands: Y (+)= A X B^T with the cheaper association first;
// the intermediate is a bf16 hi + lo pair (two K segments in the second GEMM).
//   right-first (n > m): U = X B^T -> Y = A U   (U read MN-major)
//   left-first          : T = A X  -> Y = T B^T (X read MN-major)
// fac_batched = 1: A and B hold one factor per batch entry ([batch][m][m], [batch][n][n]).
int kron_term_bf16(const void* A, int a_trans, const void* X, const void* B, float* Y, void* Th, void* Tl, int batch,
                   int m, int n, int accumulate, cudaStream_t st, int fac_batched) {
  const bool right_first = n > m;
  const int fb = fac_batched ? batch : 1;
  const int bc = fac_batched ? 0 : 1;  // broadcast flag of the factors
  const Operand Aop = mat(A, m, m, fb, a_trans ? 1 : 0, 0);  // A[r][k], or A^T stored [k][r]
  const int am = a_trans ? 1 : 0;
  {
    GemmParams p{};
    p.ngroups = 1;
    set_out(p.g[0], batch, m, n, Th, Tl, 0);
    int rc;
    if (right_first) {
      const Operand pr[1][2] = {{mat(X, m, n, batch, 0, 0), mat(B, n, n, fb, 0, 0)}};
      const SegDesc sg[1] = {SegDesc{cdiv(n, BK), 0, 0, 0, bc}};
      rc = set_segments(p, pr, sg, 1);
    } else {
      const Operand pr[1][2] = {{Aop, mat(X, m, n, batch, 1, 0)}};
      const SegDesc sg[1] = {SegDesc{cdiv(m, BK), am, 1, bc, 0}};
      rc = set_segments(p, pr, sg, 1);
    }
    if (!rc) rc = launch_gemm<K_BN, EPI_SPLIT_BF16X2>(p, st);
    if (rc) return rc;
  }
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  set_out(G, batch, m, n, Y, nullptr, 0);
  G.aux = Y;
  G.aux_bs = (long long)m * n;
  G.ld_aux = n;
  G.beta = accumulate ? 1.f : 0.f;
  int rc;
  if (right_first) {
    const Operand pr[2][2] = {{Aop, mat(Th, m, n, batch, 1, 0)}, {Aop, mat(Tl, m, n, batch, 1, 0)}};
    const SegDesc sg[2] = {SegDesc{cdiv(m, BK), am, 1, bc, 0}, SegDesc{cdiv(m, BK), am, 1, bc, 0}};
    rc = set_segments(p, pr, sg, 2);
  } else {
    const Operand pr[2][2] = {{mat(Th, m, n, batch, 0, 0), mat(B, n, n, fb, 0, 0)},
                              {mat(Tl, m, n, batch, 0, 0), mat(B, n, n, fb, 0, 0)}};
    const SegDesc sg[2] = {SegDesc{cdiv(n, BK), 0, 0, 0, bc}, SegDesc{cdiv(n, BK), 0, 0, 0, bc}};
    rc = set_segments(p, pr, sg, 2);
  }
  return rc ? rc : launch_gemm<K_BN, EPI_F32_EMA>(p, st);
}

namespace {

// One term, fp32 operands as tf32 hi/lo pairs (3xTF32), every operand K-major:
//   right-first: U = X B^T, stored transposed (U^T, [n][m]) as a tf32 pair -> Y = A U
//   left-first : T = A X with X^T given -> T stored as a tf32 pair -> Y = T B^T
// Ah/Al: K-major A; Bh/Bl: B; Xh/Xl: X (right-first) or X^T (left-first).
int kron_term_f32(const float* Ah, const float* Al, const float* Xh, const float* Xl, const float* Bh, const float* Bl,
                  float* Y, float* Th, float* Tl, int batch, int m, int n, int accumulate, cudaStream_t st) {
  const bool right_first = n > m;
  {
    GemmParams p{};
    p.ngroups = 1;
    int rc;
    if (right_first) {
      set_out(p.g[0], batch, m, n, Th, Tl, 1);
      const Operand pr[3][2] = {{mat(Xh, m, n, batch, 0, 1), mat(Bh, n, n, 1, 0, 1)},
                                {mat(Xh, m, n, batch, 0, 1), mat(Bl, n, n, 1, 0, 1)},
                                {mat(Xl, m, n, batch, 0, 1), mat(Bh, n, n, 1, 0, 1)}};
      const SegDesc sd{cdiv(n, BK_TF32), 0, 0, 0, 1, 0}, sc{cdiv(n, BK_TF32), 0, 0, 0, 1, 1};
      const SegDesc sg[3] = {sd, sc, sc};
      rc = set_segments(p, pr, sg, 3);
    } else {
      set_out(p.g[0], batch, m, n, Th, Tl, 0);
      const Operand pr[3][2] = {{mat(Ah, m, m, 1, 0, 1), mat(Xh, n, m, batch, 0, 1)},
                                {mat(Ah, m, m, 1, 0, 1), mat(Xl, n, m, batch, 0, 1)},
                                {mat(Al, m, m, 1, 0, 1), mat(Xh, n, m, batch, 0, 1)}};
      const SegDesc sd{cdiv(m, BK_TF32), 0, 0, 1, 0, 0}, sc{cdiv(m, BK_TF32), 0, 0, 1, 0, 1};
      const SegDesc sg[3] = {sd, sc, sc};
      rc = set_segments(p, pr, sg, 3);
    }
    if (!rc) rc = launch_gemm<K_BN, EPI_SPLIT_TF32, default_stages<EPI_SPLIT_TF32>(), 1, 1>(p, st);
    if (rc) return rc;
  }
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  set_out(G, batch, m, n, Y, nullptr, 0);
  G.aux = Y;
  G.aux_bs = (long long)m * n;
  G.ld_aux = n;
  G.beta = accumulate ? 1.f : 0.f;
  int rc;
  if (right_first) {
    // Y = A U: B operand element (c, k) = U[k][c] = U^T[c][k] (rows n, cols m)
    const Operand pr[3][2] = {{mat(Ah, m, m, 1, 0, 1), mat(Th, n, m, batch, 0, 1)},
                              {mat(Ah, m, m, 1, 0, 1), mat(Tl, n, m, batch, 0, 1)},
                              {mat(Al, m, m, 1, 0, 1), mat(Th, n, m, batch, 0, 1)}};
    const SegDesc sd{cdiv(m, BK_TF32), 0, 0, 1, 0, 0}, sc{cdiv(m, BK_TF32), 0, 0, 1, 0, 1};
    const SegDesc sg[3] = {sd, sc, sc};
    rc = set_segments(p, pr, sg, 3);
  } else {
    const Operand pr[3][2] = {{mat(Th, m, n, batch, 0, 1), mat(Bh, n, n, 1, 0, 1)},
                              {mat(Th, m, n, batch, 0, 1), mat(Bl, n, n, 1, 0, 1)},
                              {mat(Tl, m, n, batch, 0, 1), mat(Bh, n, n, 1, 0, 1)}};
    const SegDesc sd{cdiv(n, BK_TF32), 0, 0, 0, 1, 0}, sc{cdiv(n, BK_TF32), 0, 0, 0, 1, 1};
    const SegDesc sg[3] = {sd, sc, sc};
    rc = set_segments(p, pr, sg, 3);
  }
  return rc ? rc : launch_gemm<K_BN, EPI_F32_EMA, default_stages<EPI_F32_EMA>(), 1, 1>(p, st);
}

// Dense small-factor path (see kron_use_dense): the operator's tf32 pair W = Wh + Wl ...
int dense_operator(const float* A, int a_trans, const float* B, int m, int n, int nterms, float* Wh, float* Wl,
                   cudaStream_t st) {
  const long long mn = (long long)m * n, total = mn * mn;
  const int blocks = (int)std::min<long long>((total + SPLIT_THREADS - 1) / SPLIT_THREADS, 148LL * 16);
  ProfScope prof(PK_EW_OTHER, st);
  kron_dense_w_kernel<<<blocks, SPLIT_THREADS, 0, st>>>(A, a_trans, B, m, n, nterms, Wh, Wl);
  return launch_ok();
}

// ... and Y_flat = X_flat W^T: the X pair, one 3xTF32 GEMM (rows = batch, K = N = mn).
int dense_apply(const float* Wh, const float* Wl, const float* X, float* Y, int batch, int mn, float* Xh, float* Xl,
                cudaStream_t st) {
  int rc = split_tf32(X, Xh, Xl, (long long)batch * mn, st);
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  set_out(G, 1, batch, mn, Y, nullptr, 0);
  // Y[r][c] = sum_k X[r][k] W[c][k]: both operands K-major; hi*hi in slot 0, the corrections in slot 1
  const Operand pr[3][2] = {{mat(Xh, batch, mn, 1, 0, 1), mat(Wh, mn, mn, 1, 0, 1)},
                            {mat(Xh, batch, mn, 1, 0, 1), mat(Wl, mn, mn, 1, 0, 1)},
                            {mat(Xl, batch, mn, 1, 0, 1), mat(Wh, mn, mn, 1, 0, 1)}};
  const SegDesc sd{cdiv(mn, BK_TF32), 0, 0, 0, 0, 0}, sc{cdiv(mn, BK_TF32), 0, 0, 0, 0, 1};
  const SegDesc sg[3] = {sd, sc, sc};
  rc = set_segments(p, pr, sg, 3);
  return rc ? rc : launch_gemm<K_BN, EPI_STORE_F32, default_stages<EPI_STORE_F32>(), 1, 1>(p, st);
}

int kron_apply_dense_f32(const void* A, int a_trans, const void* X, const void* B, float* Y, int batch, int m, int n,
                         int nterms, uint8_t* w, cudaStream_t st) {
  const int mn = m * n;
  const size_t wbytes = (size_t)mn * mn * 4, xbytes = (size_t)batch * mn * 4;
  float* Wh = reinterpret_cast<float*>(w);
  float* Wl = reinterpret_cast<float*>(w + a256(wbytes));
  float* Xh = reinterpret_cast<float*>(w + 2 * a256(wbytes));
  float* Xl = reinterpret_cast<float*>(w + 2 * a256(wbytes) + a256(xbytes));
  int rc = dense_operator(static_cast<const float*>(A), a_trans, static_cast<const float*>(B), m, n, nterms, Wh, Wl, st);
  return rc ? rc : dense_apply(Wh, Wl, static_cast<const float*>(X), Y, batch, mn, Xh, Xl, st);
}

// Small Kronecker apply, fp32 FFMA: Y[b] = sum_s A_s X[b] B_s^T for X [batch][m][n].
// A block takes NW / n right-hand sides (their X staged in shared memory once)
// and all m <= 64 rows. Per term s it forms T = [X_0 B_s^T | ... ] (m x NW) in
// shared memory and adds A_s T into a register tile (RI rows x CPT columns per
// thread, NW = 16 CPT), so the sum over s stays in registers and Y is written
// once. A_{s+1} and B_{s+1} are loaded into registers while term s computes
// and stored into the other half of a double buffer, so no term waits for a
// global load. Lanes 0-15 / 16-31 of a warp take adjacent column groups of two
// row groups: every read of T is one wavefront and the A reads are broadcasts.
constexpr int KS_MAXM = 64, KS_PRE = KS_MAXM * KS_MAXM / KS_THREADS;  // A_s elements per thread

// Per-snapshot stride of the staged X: m n + 1 (the snapshots of a block start in
// distinct banks), or m n + 4 for n = 8, where rows are read as 16-byte vectors
// (the four snapshots of a 32-column block then start 4 banks apart).
__host__ __device__ __forceinline__ int ks_xstride(int m, int n) { return m * n + (n == 8 ? 4 : 1); }

template <int RI, int CPT>
__global__ void __launch_bounds__(KS_THREADS) kron_small_kernel(const float* __restrict__ A, int a_trans,
                                                                const float* __restrict__ X,
                                                                const float* __restrict__ B, float* __restrict__ Y,
                                                                int batch, int m, int n, int S) {
  extern __shared__ __align__(16) float ksm[];
  constexpr int NW = 16 * CPT;
  const int P = NW / n, xs = ks_xstride(m, n);
  const int mm = m * m, nn = n * n;
  float* Xs = ksm;                       // [P][xs]
  float* T = Xs + ((P * xs + 3) & ~3);   // [m][NW]
  float* As = T + m * NW;                // [2][m (k)][m (i)]: As[k][i] = A_s[i][k]
  float* Bs = As + 2 * mm;               // [2][n][n]
  const int m0 = blockIdx.x * P;
  const int np = min(P, batch - m0);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int cg = lane & 15;              // column group: columns CPT cg ..
  const int ig = (lane >> 4) + 2 * w;    // row group: rows RI ig ..
  // T[k][c] = sum_l X_p[k][l] B_s[j][l]: NW divides the block, so this thread's
  // column tc (snapshot tp, B row tj) is the same for every k it forms
  const int tc = tid % NW, tp = tc / n, tj = tc - tp * n;
  const long long xo = (long long)m0 * m * n;
  for (int e = tid; e < P * m * n; e += KS_THREADS) {
    const int p = e / (m * n), q = e - p * (m * n);
    Xs[p * xs + q] = p < np ? X[xo + e] : 0.f;
  }
  // element e of As (k = e / m, i = e % m) from term s
  auto a_elem = [&](int s, int e) -> float {
    const int k = e / m, i = e - k * m;
    const float* src = A + (size_t)s * mm;
    return a_trans ? __ldg(src + e) : __ldg(src + (size_t)i * m + k);
  };
  for (int e = tid; e < mm; e += KS_THREADS) As[e] = a_elem(0, e);
  for (int e = tid; e < nn; e += KS_THREADS) Bs[e] = __ldg(B + e);
  float acc[RI][CPT];
#pragma unroll
  for (int r = 0; r < RI; ++r)
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[r][c] = 0.f;
  __syncthreads();
  for (int s = 0; s < S; ++s) {
    const int cur = s & 1;
    const float* Ac = As + cur * mm;
    const float* Bc = Bs + cur * nn;
    float pre[KS_PRE], preb = 0.f;
    const bool more = s + 1 < S;
    if (more) {
#pragma unroll
      for (int q = 0; q < KS_PRE; ++q) {
        const int e = tid + q * KS_THREADS;
        pre[q] = e < mm ? a_elem(s + 1, e) : 0.f;
      }
      if (tid < nn) preb = __ldg(B + (size_t)(s + 1) * nn + tid);
    }
    {
      float br[16];  // row tj of B_s (n <= 16), read once per term
#pragma unroll
      for (int l = 0; l < 16; ++l) br[l] = l < n ? Bc[tj * n + l] : 0.f;
      const float* xp = Xs + tp * xs;
      for (int k = tid / NW; k < m; k += KS_THREADS / NW) {
        const float* xr = xp + k * n;
        float t = 0.f;
        if (n == 8) {  // xs and k n are multiples of 4: two aligned 16-byte reads
          const float4 x0 = *reinterpret_cast<const float4*>(xr);
          const float4 x1 = *reinterpret_cast<const float4*>(xr + 4);
          t = fmaf(x0.x, br[0], fmaf(x0.y, br[1], fmaf(x0.z, br[2], x0.w * br[3])));
          t += fmaf(x1.x, br[4], fmaf(x1.y, br[5], fmaf(x1.z, br[6], x1.w * br[7])));
        } else {
#pragma unroll
          for (int l = 0; l < 16; ++l)
            if (l < n) t = fmaf(xr[l], br[l], t);
        }
        T[k * NW + tc] = t;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < m; ++k) {
      float tv[CPT];
      if constexpr (CPT == 2) {
        const float2 t2 = *reinterpret_cast<const float2*>(T + k * NW + 2 * cg);
        tv[0] = t2.x;
        tv[1] = t2.y;
      } else {
        tv[0] = T[k * NW + cg];
      }
      float av[RI];
      bool done = false;
      if constexpr (RI == 4) {
        if (m == 64) {  // the thread's four rows are one aligned 16-byte vector
          const float4 a4 = *reinterpret_cast<const float4*>(Ac + k * 64 + ig * 4);
          av[0] = a4.x;
          av[1] = a4.y;
          av[2] = a4.z;
          av[3] = a4.w;
          done = true;
        }
      }
      if (!done) {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
          const int i = ig * RI + r;
          av[r] = i < m ? Ac[k * m + i] : 0.f;
        }
      }
#pragma unroll
      for (int r = 0; r < RI; ++r)
#pragma unroll
        for (int c = 0; c < CPT; ++c) acc[r][c] = fmaf(av[r], tv[c], acc[r][c]);
    }
    if (more) {
      float* An = As + (cur ^ 1) * mm;
#pragma unroll
      for (int q = 0; q < KS_PRE; ++q) {
        const int e = tid + q * KS_THREADS;
        if (e < mm) An[e] = pre[q];
      }
      if (tid < nn) Bs[(cur ^ 1) * nn + tid] = preb;
    }
    __syncthreads();  // T read by every thread; the next term's A / B stored
  }
#pragma unroll
  for (int r = 0; r < RI; ++r) {
    const int i = ig * RI + r;
    if (i >= m) continue;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int col = CPT * cg + c, p = col / n, j = col - p * n;
      if (p < np) Y[((long long)(m0 + p) * m + i) * n + j] = acc[r][c];
    }
  }
}

template <int RI, int CPT>
int launch_small(const float* A, int a_trans, const float* X, const float* B, float* Y, int batch, int m, int n,
                 int S, cudaStream_t st) {
  static std::atomic<int> attr_set{0};
  constexpr int NW = 16 * CPT;
  const int P = NW / n;
  const size_t smem =
      ((size_t)((P * ks_xstride(m, n) + 3) & ~3) + (size_t)m * NW + 2 * (size_t)m * m + 2 * (size_t)n * n) * 4;
  constexpr int kMaxSmem = 64 * 1024;  // m <= 64, n <= 16: at most 32 (64 + 1) + 64 x 32 + 2 (4096 + 256) floats
  if (smem > (size_t)kMaxSmem) return LSR_ERR_SHAPE;
  if (!attr_set.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kron_small_kernel<RI, CPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return LSR_ERR_LAUNCH;
    attr_set.store(1, std::memory_order_relaxed);
  }
  ProfScope prof(PK_GEMM_OTHER, st);
  kron_small_kernel<RI, CPT><<<cdiv(batch, P), KS_THREADS, smem, st>>>(A, a_trans, X, B, Y, batch, m, n, S);
  return launch_ok();
}

// 32-column blocks (two columns per thread) once there are enough right-hand sides
// to give every SM two blocks; 16-column blocks below that, so small batches
// still spread over the GPU. RI = rows per thread = m / 16, rounded up.
template <int CPT>
int small_rows(const float* A, int a_trans, const float* X, const float* B, float* Y, int batch, int m, int n, int S,
               cudaStream_t st) {
  switch (cdiv(m, 16)) {
    case 1: return launch_small<1, CPT>(A, a_trans, X, B, Y, batch, m, n, S, st);
    case 2: return launch_small<2, CPT>(A, a_trans, X, B, Y, batch, m, n, S, st);
    case 3: return launch_small<3, CPT>(A, a_trans, X, B, Y, batch, m, n, S, st);
    default: return launch_small<4, CPT>(A, a_trans, X, B, Y, batch, m, n, S, st);
  }
}

int kron_apply_small_f32(const float* A, int a_trans, const float* X, const float* B, float* Y, int batch, int m,
                         int n, int S, cudaStream_t st) {
  if (n <= 16 && 16 % n == 0 && cdiv(batch, 16 / n) < 2 * device_sm_count())
    return small_rows<1>(A, a_trans, X, B, Y, batch, m, n, S, st);
  return small_rows<2>(A, a_trans, X, B, Y, batch, m, n, S, st);
}

int kron_apply(const void* A, int a_trans, const void* X, const void* B, float* Y, int batch, int m, int n,
               int nterms, int f32, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!kron_dims_ok(batch, m, n, nterms)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !X || !B || !Y) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (f32 && kron_use_small(batch, m, n, nterms))
    return kron_apply_small_f32(static_cast<const float*>(A), a_trans, static_cast<const float*>(X),
                                static_cast<const float*>(B), Y, batch, m, n, nterms, st);
  if (!ws || ws_bytes < lsr_kron_apply_workspace_bytes(batch, m, n, nterms, f32)) return LSR_ERR_WORKSPACE;
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  const size_t mn = (size_t)batch * m * n;
  if (!f32) {
    void* Th = w;
    void* Tl = w + a256(mn * 2);
    for (int s = 0; s < nterms && !rc; ++s) {
      const void* As = static_cast<const uint8_t*>(A) + (size_t)s * m * m * 2;
      const void* Bs = static_cast<const uint8_t*>(B) + (size_t)s * n * n * 2;
      rc = kron_term_bf16(As, a_trans, X, Bs, Y, Th, Tl, batch, m, n, s > 0, st, 0);
    }
    return rc;
  }
  if (kron_use_dense(m, n)) return kron_apply_dense_f32(A, a_trans, X, B, Y, batch, m, n, nterms, w, st);
  float* Ah = reinterpret_cast<float*>(w);
  float* Al = reinterpret_cast<float*>(w += a256((size_t)nterms * m * m * 4));
  float* Bh = reinterpret_cast<float*>(w += a256((size_t)nterms * m * m * 4));
  float* Bl = reinterpret_cast<float*>(w += a256((size_t)nterms * n * n * 4));
  float* Xh = reinterpret_cast<float*>(w += a256((size_t)nterms * n * n * 4));
  float* Xl = reinterpret_cast<float*>(w += a256(mn * 4));
  float* Th = reinterpret_cast<float*>(w += a256(mn * 4));
  float* Tl = reinterpret_cast<float*>(w += a256(mn * 4));
  const float* Af = static_cast<const float*>(A);
  // A as K-major tf32 pairs (the caller may hold A^T); B as pairs; X in the orientation the association needs
  rc = a_trans ? split_tf32_t(Af, Ah, Al, nterms, m, m, st) : split_tf32(Af, Ah, Al, (long long)nterms * m * m, st);
  if (!rc) rc = split_tf32(static_cast<const float*>(B), Bh, Bl, (long long)nterms * n * n, st);
  if (!rc)
    rc = (n > m) ? split_tf32(static_cast<const float*>(X), Xh, Xl, (long long)mn, st)
                 : split_tf32_t(static_cast<const float*>(X), Xh, Xl, batch, m, n, st);
  for (int s = 0; s < nterms && !rc; ++s) {
    const size_t ao = (size_t)s * m * m, bo = (size_t)s * n * n;
    rc = kron_term_f32(Ah + ao, Al + ao, Xh, Xl, Bh + bo, Bl + bo, Y, Th, Tl, batch, m, n, s > 0, st);
  }
  return rc;
}

}  // namespace
}  // namespace lsr

extern "C" {

size_t lsr_gemm_f32_workspace_bytes(int batch, int M, int N, int K) {
  if (batch < 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  const size_t b = (size_t)std::max(batch, 1);
  return 2 * a256(b * M * K * 4) + 2 * a256(b * N * K * 4) + 256;  // tf32 pairs of A and of B^T
}

int lsr_gemm_f32(const float* A, const float* B, float* C, int batch, int M, int N, int K, float alpha, void* ws,
                 size_t ws_bytes, lsr_stream_t stream) {
  if (batch < 0 || batch > 65535 || M <= 0 || N <= 0 || K <= 0) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !B || !C) return LSR_ERR_ARG;
  if (K % 4 || N % 4) return LSR_ERR_SHAPE;  // 16-byte rows for the tensor maps
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_gemm_f32_workspace_bytes(batch, M, N, K)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  const size_t ab = a256((size_t)batch * M * K * 4), bb = a256((size_t)batch * N * K * 4);
  float* Ah = reinterpret_cast<float*>(w);
  float* Al = reinterpret_cast<float*>(w + ab);
  float* Bh = reinterpret_cast<float*>(w + 2 * ab);
  float* Bl = reinterpret_cast<float*>(w + 2 * ab + bb);
  rc = split_tf32(A, Ah, Al, (long long)batch * M * K, st);
  if (!rc) rc = split_tf32_t(B, Bh, Bl, batch, K, N, st);  // B^T pair, [batch][N][K]
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  GroupDesc& G = p.g[0];
  set_out(G, batch, M, N, C, nullptr, 0);
  G.alpha = alpha;
  const Operand pr[3][2] = {{mat(Ah, M, K, batch, 0, 1), mat(Bh, N, K, batch, 0, 1)},
                            {mat(Ah, M, K, batch, 0, 1), mat(Bl, N, K, batch, 0, 1)},
                            {mat(Al, M, K, batch, 0, 1), mat(Bh, N, K, batch, 0, 1)}};
  const SegDesc sd{cdiv(K, BK_TF32), 0, 0, 0, 0, 0}, sc{cdiv(K, BK_TF32), 0, 0, 0, 0, 1};
  const SegDesc sg[3] = {sd, sc, sc};
  rc = set_segments(p, pr, sg, 3);
  return rc ? rc : launch_gemm<K_BN, EPI_STORE_F32, default_stages<EPI_STORE_F32>(), 1, 1>(p, st);
}

int lsr_kron_dense_operator_f32(const float* A, int a_trans, const float* B, int m, int n, int nterms, float* Wh,
                                float* Wl, lsr_stream_t stream) {
  if (!kron_dims_ok(1, m, n, nterms) || (long long)m * n > kDenseMaxMN) return LSR_ERR_ARG;
  if (!A || !B || !Wh || !Wl) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  return dense_operator(A, a_trans, B, m, n, nterms, Wh, Wl, reinterpret_cast<cudaStream_t>(stream));
}

size_t lsr_kron_dense_apply_workspace_bytes(int batch, int mn) {
  if (batch < 0 || mn <= 0) return 0;
  return 2 * a256((size_t)std::max(batch, 1) * mn * 4) + 256;
}

int lsr_kron_dense_apply_f32(const float* Wh, const float* Wl, const float* X, float* Y, int batch, int mn, void* ws,
                             size_t ws_bytes, lsr_stream_t stream) {
  if (batch < 0 || mn <= 0 || mn > kDenseMaxMN || mn % 4) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!Wh || !Wl || !X || !Y) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_kron_dense_apply_workspace_bytes(batch, mn)) return LSR_ERR_WORKSPACE;
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  float* Xh = reinterpret_cast<float*>(w);
  float* Xl = reinterpret_cast<float*>(w + a256((size_t)batch * mn * 4));
  return dense_apply(Wh, Wl, X, Y, batch, mn, Xh, Xl, reinterpret_cast<cudaStream_t>(stream));
}

int lsr_kron_apply_bf16(const void* A, int a_trans, const void* X, const void* B, float* Y, int batch, int m, int n,
                        int nterms, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  return kron_apply(A, a_trans, X, B, Y, batch, m, n, nterms, 0, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int lsr_kron_apply_f32(const float* A, int a_trans, const float* X, const float* B, float* Y, int batch, int m, int n,
                       int nterms, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  return kron_apply(A, a_trans, X, B, Y, batch, m, n, nterms, 1, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Tiny-factor Kronecker reconstruction  W = sum_s F_0[s] ⊗ F_1[s] ⊗ ... ⊗ F_{K-1}[s]
//
// Replaces direct_k{3,4,5}_kernel / native_reconstruct (kron_cuda.py:242-583):
// each output entry W[i][j] is decoded into mixed-radix mode digits once, one
// scalar is read from every factor per term and the K scalars multiplied; no
// partial Kronecker product is materialised. The kernel is specialised on K
// (unrolled factor loop, factor pointers and extents in registers). A block
// covers 64 consecutive entries and splits the S terms into 4 contiguous
// slices, one per 64-thread group, summed in a fixed order at the end (the
// result does not depend on scheduling): 16 x 768 outputs make 192 blocks, so
// every SM works even at S = 256. Factors are read through the read-only
// cache; the reference's largest factor set (K = 3, S = 256) is 213 KB.
// ---------------------------------------------------------------------------

namespace lsr {
namespace {

constexpr int kMaxFactors = 8;
constexpr int REC_OUTS = 64, REC_SPLIT = 4;

struct RecParams {
  const float* f[kMaxFactors];
  int r[kMaxFactors], c[kMaxFactors];
  int S;
  long long R, C;
};

template <int K>
__global__ void __launch_bounds__(REC_OUTS * REC_SPLIT) kron_reconstruct_kernel(const __grid_constant__ RecParams p,
                                                                               float* __restrict__ W) {
  __shared__ float part[REC_SPLIT][REC_OUTS];
  const int o = threadIdx.x % REC_OUTS, q = threadIdx.x / REC_OUTS;
  const long long total = p.R * p.C;
  const float* f[K];
  int sz[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    f[k] = p.f[k];
    sz[k] = p.r[k] * p.c[k];
  }
  const int s0 = (int)((long long)p.S * q / REC_SPLIT), s1 = (int)((long long)p.S * (q + 1) / REC_SPLIT);
  for (long long base = (long long)blockIdx.x * REC_OUTS; base < total; base += (long long)gridDim.x * REC_OUTS) {
    const long long e = base + o;
    float acc = 0.f;
    if (e < total) {
      long long i = e / p.C, j = e - (e / p.C) * p.C;
      const float* ptr[K];
#pragma unroll
      for (int k = K - 1; k >= 0; --k) {  // the last factor is the fastest-varying mode
        const int ik = (int)(i % p.r[k]), jk = (int)(j % p.c[k]);
        i /= p.r[k];
        j /= p.c[k];
        ptr[k] = f[k] + (long long)s0 * sz[k] + ik * p.c[k] + jk;
      }
#pragma unroll 4
      for (int s = s0; s < s1; ++s) {
        float prod = __ldg(ptr[0]);
        ptr[0] += sz[0];
#pragma unroll
        for (int k = 1; k < K; ++k) {
          prod *= __ldg(ptr[k]);
          ptr[k] += sz[k];
        }
        acc += prod;
      }
    }
    part[q][o] = acc;
    __syncthreads();
    if (q == 0 && e < total) {
      float w = part[0][o];
#pragma unroll
      for (int k = 1; k < REC_SPLIT; ++k) w += part[k][o];
      W[e] = w;
    }
    __syncthreads();
  }
}

template <int K>
int launch_reconstruct(const RecParams& p, float* W, cudaStream_t st) {
  const long long total = p.R * p.C;
  const int blocks = (int)std::max<long long>(
      1, std::min<long long>((total + REC_OUTS - 1) / REC_OUTS, 8LL * lsr::device_sm_count()));
  kron_reconstruct_kernel<K><<<blocks, REC_OUTS * REC_SPLIT, 0, st>>>(p, W);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

}  // namespace
}  // namespace lsr

extern "C" {

int lsr_kron_reconstruct_f32(const float* const* factors, const int* rows, const int* cols, int K, int S, float* W,
                             lsr_stream_t stream) {
  if (!factors || !rows || !cols || !W || K < 1 || K > lsr::kMaxFactors || S < 0) return LSR_ERR_ARG;
  lsr::RecParams p{};
  p.S = S;
  p.R = 1;
  p.C = 1;
  for (int k = 0; k < K; ++k) {
    if (!factors[k] || rows[k] <= 0 || cols[k] <= 0) return LSR_ERR_ARG;
    p.f[k] = factors[k];
    p.r[k] = rows[k];
    p.c[k] = cols[k];
    p.R *= rows[k];
    p.C *= cols[k];
    if (p.R > (1LL << 31) || p.C > (1LL << 31) || (long long)rows[k] * cols[k] > (1LL << 31)) return LSR_ERR_SHAPE;
  }
  int rc = lsr::check_device();
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  lsr::ProfScope prof(lsr::PK_EW_OTHER, st);
  switch (K) {
    case 1: return lsr::launch_reconstruct<1>(p, W, st);
    case 2: return lsr::launch_reconstruct<2>(p, W, st);
    case 3: return lsr::launch_reconstruct<3>(p, W, st);
    case 4: return lsr::launch_reconstruct<4>(p, W, st);
    case 5: return lsr::launch_reconstruct<5>(p, W, st);
    case 6: return lsr::launch_reconstruct<6>(p, W, st);
    case 7: return lsr::launch_reconstruct<7>(p, W, st);
    default: return lsr::launch_reconstruct<8>(p, W, st);
  }
}

}  // extern "C"
