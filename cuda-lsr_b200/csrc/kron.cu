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

int kron_apply(const void* A, int a_trans, const void* X, const void* B, float* Y, int batch, int m, int n,
               int nterms, int f32, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!kron_dims_ok(batch, m, n, nterms)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !X || !B || !Y) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
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
// one thread per entry W[i][j]; (i, j) are decoded into mixed-radix mode
// digits, one scalar is read from every factor and the K scalars multiplied,
// accumulated over s in order; no partial Kronecker product is materialised.
// Every factor (a few KB for the reference's 16 x 768 cases) is staged once
// per block in shared memory. The work is a single wave of a few dozen
// blocks: latency-bound, not bandwidth- or compute-bound.
// ---------------------------------------------------------------------------

namespace lsr {
namespace {

constexpr int kMaxFactors = 8;

struct RecParams {
  const float* f[kMaxFactors];
  int r[kMaxFactors], c[kMaxFactors];
  int off[kMaxFactors];  // offset of factor k in the staged buffer (floats)
  int K, S;
  long long R, C;
  int staged;  // factors fit in shared memory
};

__global__ void __launch_bounds__(256) kron_reconstruct_kernel(RecParams p, float* __restrict__ W) {
  extern __shared__ float sf[];
  if (p.staged) {
    for (int k = 0; k < p.K; ++k) {
      const int n = p.S * p.r[k] * p.c[k];
      for (int i = threadIdx.x; i < n; i += blockDim.x) sf[p.off[k] + i] = p.f[k][i];
    }
    __syncthreads();
  }
  const long long total = p.R * p.C;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    long long i = e / p.C, j = e - (e / p.C) * p.C;
    int idx[kMaxFactors];
    for (int k = p.K - 1; k >= 0; --k) {  // last factor is the fastest-varying mode
      const int ik = (int)(i % p.r[k]), jk = (int)(j % p.c[k]);
      i /= p.r[k];
      j /= p.c[k];
      idx[k] = ik * p.c[k] + jk;
    }
    float acc = 0.f;
    for (int s = 0; s < p.S; ++s) {
      float prod = 1.f;
      for (int k = 0; k < p.K; ++k) {
        const int sz = p.r[k] * p.c[k];
        const float v = p.staged ? sf[p.off[k] + s * sz + idx[k]] : __ldg(p.f[k] + (long long)s * sz + idx[k]);
        prod = (k == 0) ? v : prod * v;
      }
      acc += prod;
    }
    W[e] = acc;
  }
}

}  // namespace
}  // namespace lsr

extern "C" {

int lsr_kron_reconstruct_f32(const float* const* factors, const int* rows, const int* cols, int K, int S, float* W,
                             lsr_stream_t stream) {
  if (!factors || !rows || !cols || !W || K < 1 || K > lsr::kMaxFactors || S < 0) return LSR_ERR_ARG;
  lsr::RecParams p{};
  p.K = K;
  p.S = S;
  p.R = 1;
  p.C = 1;
  long long staged_floats = 0;
  for (int k = 0; k < K; ++k) {
    if (!factors[k] || rows[k] <= 0 || cols[k] <= 0) return LSR_ERR_ARG;
    p.f[k] = factors[k];
    p.r[k] = rows[k];
    p.c[k] = cols[k];
    p.off[k] = (int)staged_floats;
    staged_floats += (long long)S * rows[k] * cols[k];
    p.R *= rows[k];
    p.C *= cols[k];
    if (p.R > (1LL << 31) || p.C > (1LL << 31)) return LSR_ERR_SHAPE;
  }
  int rc = lsr::check_device();
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)staged_floats * 4;
  p.staged = smem <= 160 * 1024;
  auto kfn = lsr::kron_reconstruct_kernel;
  if (p.staged && smem > 48 * 1024 &&
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return LSR_ERR_LAUNCH;
  const long long total = p.R * p.C;
  const int blocks = (int)std::max<long long>(1, std::min<long long>((total + 255) / 256, 4LL * lsr::device_sm_count()));
  lsr::ProfScope prof(lsr::PK_EW_OTHER, st);
  kfn<<<blocks, 256, p.staged ? smem : 0, st>>>(p, W);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

}  // extern "C"
