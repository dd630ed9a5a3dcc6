// Batched coupled Newton iteration for inverse p-th roots A^{-1/p} (p = 2, 4)
// of symmetric positive definite factors, fp32 (shampoo.py:277-347 for one
// factor, :408-542 batched with a per-factor convergence mask).
//
// The reference recurrence, per factor:
//   z = (p + 1) / (2 ||A + eps I||_F),  X = z^{1/p} I,  M = z (A + eps I)
//   while max|M - I| > tol and it < max_it:
//     Mp = alpha M + (1 - alpha) I      (alpha = -1/p)
//     X  = X Mp ;  M = Mp^p M
//
// use_tf32 = 0 (the reference's setting: it turns TF32 off, shampoo.py:73-75):
// the recurrence in fp32 FFMA on the CUDA cores (round-to-nearest, the
// reference's numerics): one pass, pass 2 below started from the beginning.
//
// use_tf32 = 1: three passes, all in this direct form:
//
// 1. Tensor cores, until max|M - I| <= 1e-4 (or the tolerance, if looser).
//    Every GEMM is 3xTF32 (hi*hi + hi*lo + lo*hi into two TMEM accumulators).
//    X and M are carried as tf32 hi / lo pairs that the GEMM epilogue writes
//    directly, so the operands of the next products need no extra pass. Every
//    matrix of the recurrence is a polynomial in A, hence symmetric: each
//    product computes the upper-triangle tiles and mirrors them, and operand B
//    is read as its own transpose (K-major).
// 2. fp32 FFMA (CUDA cores, round-to-nearest) from that state to the
//    tolerance: one or two steps, as Newton converges quadratically. The
//    tensor cores add each group of products into the fp32 accumulator with
//    truncation; that bias puts a floor near max|M - I| ~ 1e-6 under the
//    tensor-core pass, which this pass removes.
// 3. Ill-conditioned factors (more than 14 iterations for p = 2, 13 for p = 4
//    in passes 1 + 2; well-conditioned factors finish within those counts) are
//    recomputed from scratch in fp32 FFMA: there the truncation bias of pass 1
//    is a sizeable fraction of the smallest eigenvalues (a 1e-5 ridge: X ~1e-2
//    off instead of the reference's ~4e-4). The reference's hybrid path does
//    the same for its hard factors (shampoo.py:545-595).
//
// Convergence is tracked on the device (per-factor error, active flag,
// iteration count). The GEMMs skip the tiles of inactive factors and the
// elementwise kernels return at once for them; the host reads the number of
// active factors only every `check_every` iterations (0: never; each pass then
// runs max_iterations rounds of launches).
#include <cmath>

#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int CN_THREADS = 256;
constexpr int CN_BN = 256;
constexpr float kSwitchTol = 1e-4f;  // tensor-core pass -> fp32 pass
constexpr int kCnMats = 14;          // n x n fp32 buffers per factor in the workspace

int launch_status() { return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH; }

size_t a256(size_t x) { return align_up(x, 256); }

__device__ __forceinline__ void split4(const float4& v, float4& h, float4& l) {
  h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
  l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
}

__device__ __forceinline__ float4 add4(const float4& a, const float4& b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ float amax4(const float4& v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// Diagonal value d placed in the lanes of a 4-vector that starts at element i of an n x n matrix.
__device__ __forceinline__ float4 diag4(long long i, int n, float d) {
  const int r = (int)(i / n), c = (int)(i % n);
  return make_float4(r == c ? d : 0.f, r == c + 1 ? d : 0.f, r == c + 2 ? d : 0.f, r == c + 3 ? d : 0.f);
}

// max |M - I| over a 4-vector of M starting at element i.
__device__ __forceinline__ float dev4(const float4& m, long long i, int n) {
  const float4 one = diag4(i, n, 1.f);
  return amax4(make_float4(m.x - one.x, m.y - one.y, m.z - one.z, m.w - one.w));
}

// alpha m + (1 - alpha) on the diagonal, each operation rounded (no FMA contraction).
__device__ __forceinline__ float4 mp4(const float4& m, long long i, int n, float alpha) {
  const float4 d = diag4(i, n, 1.f - alpha);
  return make_float4(__fadd_rn(__fmul_rn(alpha, m.x), d.x), __fadd_rn(__fmul_rn(alpha, m.y), d.y),
                     __fadd_rn(__fmul_rn(alpha, m.z), d.z), __fadd_rn(__fmul_rn(alpha, m.w), d.w));
}

// Block-wide max of non-negative values, then one atomicMax per block.
__device__ __forceinline__ void block_max_to(float v, unsigned int* dst) {
  __shared__ float red[CN_THREADS / 32];
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < CN_THREADS / 32 ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) atomicMax(dst, __float_as_uint(v));
  }
}

// Grid-stride loop over the float4 vectors of one factor (blockIdx.y = factor).
#define CN_FOR_ELEMS(k) \
  for (long long k = (long long)blockIdx.x * CN_THREADS + threadIdx.x; k < n4; k += (long long)gridDim.x * CN_THREADS)

// z = (p + 1) / (2 ||A + eps I||_F) per factor (one block per factor, fp64 sum).
__global__ void __launch_bounds__(CN_THREADS) cn_norm_kernel(const float* __restrict__ A, int n, float eps, int root,
                                                            float* __restrict__ z) {
  const int b = blockIdx.x;
  const float4* a = reinterpret_cast<const float4*>(A + (long long)b * n * n);
  const long long n4 = (long long)n * n / 4;
  double s = 0.0;
  for (long long k = threadIdx.x; k < n4; k += CN_THREADS) {
    float4 v = a[k];
    if (eps != 0.f) v = add4(v, diag4(4 * k, n, eps));
    s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  __shared__ double red[CN_THREADS / 32];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < CN_THREADS / 32; ++w) t += red[w];
    const float nrm = (float)sqrt(t);
    z[b] = (float)(root + 1) / (2.f * nrm);
  }
}

// Start of the recurrence for every factor with sel[b] (all when sel is null):
// X = z^{1/p} I, M = z (sym(A) + eps I), as fp32 into X / M, or as tf32 pairs into
// Xh / Xl, Mh / Ml when Xh is given; errb = max |M - I|.
__global__ void __launch_bounds__(CN_THREADS) cn_init_kernel(const float* __restrict__ A, int n, float eps, int root,
                                                            const float* __restrict__ z, const int* __restrict__ sel,
                                                            float* X, float* M, float* Xh, float* Xl, float* Mh,
                                                            float* Ml, unsigned int* __restrict__ errb) {
  const int b = blockIdx.y;
  if (sel && !sel[b]) return;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  const float zb = z[b];
  const float xd = powf(zb, 1.f / (float)root);
  float m = 0.f;
  CN_FOR_ELEMS(k) {
    // the symmetric part of A (A itself when A is exactly symmetric): every
    // product of the recurrence then has symmetric operands
    float4 a = reinterpret_cast<const float4*>(A)[base + k];
    {
      const long long e = 4 * k;
      const int r = (int)(e / n), c = (int)(e % n);
      const float* At = A + (long long)b * n * n;
      a = make_float4(0.5f * (a.x + At[(long long)c * n + r]), 0.5f * (a.y + At[(long long)(c + 1) * n + r]),
                      0.5f * (a.z + At[(long long)(c + 2) * n + r]), 0.5f * (a.w + At[(long long)(c + 3) * n + r]));
    }
    if (eps != 0.f) a = add4(a, diag4(4 * k, n, eps));
    const float4 mm = make_float4(__fmul_rn(zb, a.x), __fmul_rn(zb, a.y), __fmul_rn(zb, a.z), __fmul_rn(zb, a.w));
    const float4 x = diag4(4 * k, n, xd);
    const long long i = base + k;
    if (Xh) {
      float4 h, l;
      split4(x, h, l);
      reinterpret_cast<float4*>(Xh)[i] = h;
      reinterpret_cast<float4*>(Xl)[i] = l;
      split4(mm, h, l);
      reinterpret_cast<float4*>(Mh)[i] = h;
      reinterpret_cast<float4*>(Ml)[i] = l;
    } else {
      reinterpret_cast<float4*>(X)[i] = x;
      reinterpret_cast<float4*>(M)[i] = mm;
    }
    m = fmaxf(m, dev4(mm, 4 * k, n));
  }
  block_max_to(m, errb + b);
}

// Pass bookkeeping, one block. For every participating factor (sel[b], or all):
//   mode 0 (after an iteration): if active: iters += 1, err, active = err > tol
//   mode 1 (a pass starts, count restarts): iters = 0, err, active = err > tol
//   mode 2 (a pass starts, count continues): err, active = err > tol
// Other factors become inactive. The error accumulator is cleared for the
// next iteration and the number of active factors written to *nactive.
__global__ void __launch_bounds__(1024) cn_finalize_kernel(unsigned int* __restrict__ errb, float* __restrict__ err,
                                                          int* __restrict__ active, int* __restrict__ iters,
                                                          int* __restrict__ nactive, int batch, float tol, int mode,
                                                          const int* __restrict__ sel) {
  int cnt = 0;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    if (sel && !sel[b]) {
      active[b] = 0;
    } else if (mode != 0 || active[b]) {
      const float e = __uint_as_float(errb[b]);
      err[b] = e;
      if (mode == 0) iters[b] += 1;
      if (mode == 1) iters[b] = 0;
      active[b] = e > tol ? 1 : 0;
    }
    errb[b] = 0u;
    cnt += active[b];
  }
  __shared__ int red[32];
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    *nactive = t;
  }
}

// ---------------------------------------------------------------------------
// Pass 1: tensor cores
// ---------------------------------------------------------------------------

// Mp = alpha M + (1 - alpha) I from M = Mh + Ml, as a tf32 pair.
__global__ void __launch_bounds__(CN_THREADS) cn_tc_mp_kernel(const float* __restrict__ Mh, const float* __restrict__ Ml,
                                                             float* __restrict__ Mph, float* __restrict__ Mpl, int n,
                                                             float alpha, const int* __restrict__ active) {
  const int b = blockIdx.y;
  if (!active[b]) return;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  CN_FOR_ELEMS(k) {
    const float4 m = add4(reinterpret_cast<const float4*>(Mh)[base + k], reinterpret_cast<const float4*>(Ml)[base + k]);
    float4 h, l;
    split4(mp4(m, 4 * k, n, alpha), h, l);
    reinterpret_cast<float4*>(Mph)[base + k] = h;
    reinterpret_cast<float4*>(Mpl)[base + k] = l;
  }
}

// X = Xn, M = Mn (tf32 pairs) for active factors; errb = max |M - I|.
__global__ void __launch_bounds__(CN_THREADS) cn_tc_commit_kernel(float* Xh, float* Xl, float* Mh, float* Ml,
                                                                 const float* Xnh, const float* Xnl,
                                                                 const float* Mnh, const float* Mnl, int n,
                                                                 const int* __restrict__ active,
                                                                 unsigned int* __restrict__ errb) {
  const int b = blockIdx.y;
  if (!active[b]) return;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  float mx = 0.f;
  CN_FOR_ELEMS(k) {
    const long long i = base + k;
    const float4 mh = reinterpret_cast<const float4*>(Mnh)[i], ml = reinterpret_cast<const float4*>(Mnl)[i];
    reinterpret_cast<float4*>(Mh)[i] = mh;
    reinterpret_cast<float4*>(Ml)[i] = ml;
    reinterpret_cast<float4*>(Xh)[i] = reinterpret_cast<const float4*>(Xnh)[i];
    reinterpret_cast<float4*>(Xl)[i] = reinterpret_cast<const float4*>(Xnl)[i];
    mx = fmaxf(mx, dev4(add4(mh, ml), 4 * k, n));
  }
  block_max_to(mx, errb + b);
}

// End of pass 1 for every factor: X = Xh + Xl, M = Mh + Ml (fp32), errb = max |M - I|.
__global__ void __launch_bounds__(CN_THREADS) cn_tc_unpack_kernel(const float* Xh, const float* Xl, const float* Mh,
                                                                 const float* Ml, float* X, float* M, int n,
                                                                 unsigned int* __restrict__ errb) {
  const int b = blockIdx.y;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  float mx = 0.f;
  CN_FOR_ELEMS(k) {
    const long long i = base + k;
    const float4 m = add4(reinterpret_cast<const float4*>(Mh)[i], reinterpret_cast<const float4*>(Ml)[i]);
    reinterpret_cast<float4*>(M)[i] = m;
    reinterpret_cast<float4*>(X)[i] =
        add4(reinterpret_cast<const float4*>(Xh)[i], reinterpret_cast<const float4*>(Xl)[i]);
    mx = fmaxf(mx, dev4(m, 4 * k, n));
  }
  block_max_to(mx, errb + b);
}

Operand tf32_mat(const float* base, int n, int batch) {
  Operand o{base, n, n, n, (long long)n * n, batch, 0};
  o.f32 = 1;
  return o;
}

// (outh, outl)_g = tf32 pair of A_g B_g for ng (<= 2) symmetric products per
// factor, 3xTF32, upper-triangle tiles mirrored; inactive factors skipped.
int cn_tc_products(int ng, float* const* outh, float* const* outl, const float* const* Ah, const float* const* Al,
                   const float* const* Bh, const float* const* Bl, int batch, int n, const int* active,
                   cudaStream_t st) {
  GemmParams p{};
  p.ngroups = ng;
  p.masked = 1;
  const int kb = cdiv(n, BK_TF32);
  for (int g = 0; g < ng; ++g) {
    const float* pa[3] = {Ah[g], Ah[g], Al[g]};
    const float* pb[3] = {Bh[g], Bl[g], Bh[g]};
    for (int t = 0; t < 3; ++t) {
      int rc = make_operand_map(&p.mapA[g][t], tf32_mat(pa[t], n, batch), false, CN_BN);
      if (!rc) rc = make_operand_map(&p.mapB[g][t], tf32_mat(pb[t], n, batch), true, CN_BN);
      if (rc) return rc;
    }
    GroupDesc& G = p.g[g];
    G.batch = batch;
    G.M = G.N = n;
    G.tri = 1;
    G.nseg = 3;
    G.seg[0] = SegDesc{kb, 0, 0, 0, 0, 0};
    G.seg[1] = SegDesc{kb, 0, 0, 0, 0, 1};
    G.seg[2] = SegDesc{kb, 0, 0, 0, 0, 1};
    G.out = outh[g];
    G.out2 = outl[g];
    G.out_bs = (long long)n * n;
    G.ldo = n;
    G.alpha = 1.f;
    G.active = active;
  }
  return launch_gemm<CN_BN, EPI_SPLIT_TF32, default_stages<EPI_SPLIT_TF32>(), 1, 1>(p, st, PK_GEMM_OTHER);
}

// ---------------------------------------------------------------------------
// Passes 2 and 3: fp32 FFMA on the CUDA cores
// ---------------------------------------------------------------------------

constexpr int SG_T = 128;    // output tile (SG_T x SG_T per block)
constexpr int SG_K = 16;     // K rows per pipeline stage
constexpr int SG_STAGES = 3;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = smem_u32(smem);
  const int n = pred ? 16 : 0;  // 0: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// C[b] = A[b] B[b] for every factor with active[b] (n x n row-major fp32,
// n % 4 == 0), for a symmetric A and a symmetric product (every product of the
// recurrence: its operands are polynomials in the same factor). A symmetric
// means the A tile's K-major copy is A's own rows, so both tiles are plain
// 16-byte cp.async copies into a 3-stage shared-memory ring. Only tiles on or
// above the diagonal run, and mirror their elements. 256 threads = 8 warps of
// 32 x 64 outputs (4 x 2 warps per tile); a lane owns 8 x 8 outputs, two 4-row
// strips 16 apart by two 4-column strips 32 apart. fp32 FFMA in K order,
// summed per 8-wide K step before it enters the running sum (n / 8 roundings
// of the running sum instead of n).
__global__ void __launch_bounds__(256) cn_sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                      float* __restrict__ C, int n, const int* __restrict__ active) {
  const int b = blockIdx.z;
  if (!active[b] || blockIdx.x < blockIdx.y) return;
  const long long off = (long long)b * n * n;
  A += off;
  B += off;
  C += off;
  __shared__ __align__(16) float As[SG_STAGES][SG_K][SG_T];  // As[k][r] = A[k0 + k][r0 + r] = A[r0 + r][k0 + k]
  __shared__ __align__(16) float Bs[SG_STAGES][SG_K][SG_T];  // Bs[k][c] = B[k0 + k][c0 + c]
  const int r0 = blockIdx.y * SG_T, c0 = blockIdx.x * SG_T;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int rbase = (warp >> 1) * 32 + (lane >> 3) * 4;  // first of the lane's rows (then +16)
  const int cbase = (warp & 1) * 64 + (lane & 7) * 4;    // first of the lane's columns (then +32)
  // copy K rows [k0, k0 + 16) of both tiles into stage s: 512 16-byte vectors each, 2 per thread
  auto issue = [&](int s, int k0) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int v = tid + t * 256;
      const int kr = v >> 5, cv = (v & 31) * 4;
      const int gk = k0 + kr;
      const bool ka = gk < n;
      cp_async16(&As[s][kr][cv], A + (long long)(ka ? gk : 0) * n + (r0 + cv < n ? r0 + cv : 0), ka && r0 + cv < n);
      cp_async16(&Bs[s][kr][cv], B + (long long)(ka ? gk : 0) * n + (c0 + cv < n ? c0 + cv : 0), ka && c0 + cv < n);
    }
  };
  const int ksteps = (n + SG_K - 1) / SG_K;
  issue(0, 0);
  cp_async_commit();
  if (ksteps > 1) issue(1, SG_K);
  cp_async_commit();
  float acc[8][8] = {};
  for (int ks = 0; ks < ksteps; ++ks) {
    cp_async_wait<1>();  // stage ks has landed (this thread's copies)
    __syncthreads();     // ... and every thread's; stage ks - 1 is no longer read
    if (ks + 2 < ksteps) issue((ks + 2) % SG_STAGES, (ks + 2) * SG_K);
    cp_async_commit();
    const int s = ks % SG_STAGES;
#pragma unroll
    for (int h = 0; h < SG_K; h += 8) {
      float part[8][8];
#pragma unroll
      for (int k = h; k < h + 8; ++k) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[s][k][rbase]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[s][k][rbase + 16]);
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[s][k][cbase]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[s][k][cbase + 32]);
        const float a8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float b8[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) part[i][j] = k == h ? a8[i] * b8[j] : fmaf(a8[i], b8[j], part[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += part[i][j];
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + rbase + (i & 3) + (i >> 2) * 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + cbase + (j & 3) + (j >> 2) * 32;
      if (r >= n || c >= n || c < r) continue;
      C[(long long)r * n + c] = acc[i][j];
      if (c > r) C[(long long)c * n + r] = acc[i][j];
    }
  }
}

// Mp = alpha M + (1 - alpha) I for active factors.
__global__ void __launch_bounds__(CN_THREADS) cn_mp_kernel(const float* __restrict__ M, float* __restrict__ Mp, int n,
                                                          float alpha, const int* __restrict__ active) {
  const int b = blockIdx.y;
  if (!active[b]) return;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  CN_FOR_ELEMS(k) {
    reinterpret_cast<float4*>(Mp)[base + k] = mp4(reinterpret_cast<const float4*>(M)[base + k], 4 * k, n, alpha);
  }
}

// X = Xn, M = Mn for active factors; errb = max |M - I|.
__global__ void __launch_bounds__(CN_THREADS) cn_commit_kernel(float* __restrict__ X, float* __restrict__ M,
                                                              const float* __restrict__ Xn,
                                                              const float* __restrict__ Mn, int n,
                                                              const int* __restrict__ active,
                                                              unsigned int* __restrict__ errb) {
  const int b = blockIdx.y;
  if (!active[b]) return;
  const long long n4 = (long long)n * n / 4;
  const long long base = (long long)b * n * n / 4;
  float mx = 0.f;
  CN_FOR_ELEMS(k) {
    const float4 m = reinterpret_cast<const float4*>(Mn)[base + k];
    reinterpret_cast<float4*>(M)[base + k] = m;
    reinterpret_cast<float4*>(X)[base + k] = reinterpret_cast<const float4*>(Xn)[base + k];
    mx = fmaxf(mx, dev4(m, 4 * k, n));
  }
  block_max_to(mx, errb + b);
}

// redo[b] = iters[b] > threshold
__global__ void cn_select_kernel(const int* __restrict__ iters, int threshold, int* __restrict__ redo, int batch) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < batch; b += gridDim.x * blockDim.x)
    redo[b] = iters[b] > threshold ? 1 : 0;
}

bool cn_args_ok(int batch, int n, int root) {
  return batch >= 0 && batch <= 65535 && n > 0 && n % 4 == 0 && n <= 16384 && (root == 2 || root == 4);
}

}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

size_t lsr_coupled_newton_workspace_bytes(int batch, int n) {
  if (!cn_args_ok(batch, n, 2)) return 0;
  const size_t mat = a256((size_t)batch * n * n * 4);
  return kCnMats * mat + 5 * a256((size_t)batch * 4) + 256;
}

int lsr_coupled_newton_f32(const float* A, float* X, int* iters, float* err, int* redo_out, int batch, int n, int root,
                           float epsilon, float tolerance, int max_iterations, int check_every, int use_tf32,
                           void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (!cn_args_ok(batch, n, root) || max_iterations < 0 || check_every < 0) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !X || !iters || !err) return LSR_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(X)) & 15) return LSR_ERR_SHAPE;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_coupled_newton_workspace_bytes(batch, n)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  const size_t mat = a256((size_t)batch * n * n * 4);
  float* buf[kCnMats];
  for (int i = 0; i < kCnMats; ++i) buf[i] = reinterpret_cast<float*>(w + i * mat);
  w += kCnMats * mat;
  const size_t vec = a256((size_t)batch * 4);
  float* z = reinterpret_cast<float*>(w);
  unsigned int* errb = reinterpret_cast<unsigned int*>(w + vec);
  int* active = reinterpret_cast<int*>(w + 2 * vec);
  int* redo = reinterpret_cast<int*>(w + 3 * vec);
  int* nactive = reinterpret_cast<int*>(w + 4 * vec);
  // pass 1 (tf32 pairs)
  float *Xh = buf[0], *Xl = buf[1], *Mh = buf[2], *Ml = buf[3], *Mph = buf[4], *Mpl = buf[5];
  float *Xnh = buf[6], *Xnl = buf[7], *Ph = buf[8], *Pl = buf[9], *P2h = buf[10], *P2l = buf[11];
  float *Mnh = buf[12], *Mnl = buf[13];
  // passes 2 and 3 (fp32; X is the caller's buffer)
  float *M = buf[6], *Mp = buf[7], *P = buf[8], *P2 = buf[9], *Xn = buf[10], *Mn = buf[11];

  const float alpha = -1.f / (float)root;
  const float sw = std::max(tolerance, kSwitchTol);
  const long long n4 = (long long)n * n / 4;
  const dim3 eg((unsigned)std::min<long long>(64, (n4 + CN_THREADS - 1) / CN_THREADS), (unsigned)batch);
  const dim3 sg((unsigned)cdiv(n, SG_T), (unsigned)cdiv(n, SG_T), (unsigned)batch);

  // one accounted launch per kernel
#define CN_LAUNCH(...)                     \
  do {                                     \
    ProfScope prof(PK_EW_OTHER, st);       \
    __VA_ARGS__;                           \
    if ((rc = launch_status())) return rc; \
  } while (0)
  // host check, every check_every iterations: 1 = no factor active, -1 = error
  auto done = [&](int it) -> int {
    if (check_every <= 0 || it % check_every) return 0;
    int h = 0;
    if (cudaMemcpyAsync(&h, nactive, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return -1;
    return h == 0 ? 1 : 0;
  };
  // one fp32 FFMA iteration of the direct form for the active factors
  auto fp32_step = [&]() -> int {
    CN_LAUNCH(cn_mp_kernel<<<eg, CN_THREADS, 0, st>>>(M, Mp, n, alpha, active));
    CN_LAUNCH(cn_sgemm_kernel<<<sg, 256, 0, st>>>(X, Mp, Xn, n, active));
    CN_LAUNCH(cn_sgemm_kernel<<<sg, 256, 0, st>>>(Mp, Mp, P, n, active));
    if (root == 4) {
      CN_LAUNCH(cn_sgemm_kernel<<<sg, 256, 0, st>>>(P, P, P2, n, active));
      CN_LAUNCH(cn_sgemm_kernel<<<sg, 256, 0, st>>>(P2, M, Mn, n, active));
    } else {
      CN_LAUNCH(cn_sgemm_kernel<<<sg, 256, 0, st>>>(P, M, Mn, n, active));
    }
    CN_LAUNCH(cn_commit_kernel<<<eg, CN_THREADS, 0, st>>>(X, M, Xn, Mn, n, active, errb));
    return LSR_OK;
  };

  if (cudaMemsetAsync(errb, 0, (size_t)batch * 4, st) != cudaSuccess) return LSR_ERR_LAUNCH;
  if (cudaMemsetAsync(redo, 0, (size_t)batch * 4, st) != cudaSuccess) return LSR_ERR_LAUNCH;
  CN_LAUNCH(cn_norm_kernel<<<batch, CN_THREADS, 0, st>>>(A, n, epsilon, root, z));

  if (!use_tf32) {
    // ---- fp32 FFMA from the start, to the tolerance
    CN_LAUNCH(cn_init_kernel<<<eg, CN_THREADS, 0, st>>>(A, n, epsilon, root, z, nullptr, X, M, nullptr, nullptr,
                                                        nullptr, nullptr, errb));
    CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 1, nullptr));
    for (int it = 0; it < max_iterations; ++it) {
      const int d = done(it);
      if (d < 0) return LSR_ERR_LAUNCH;
      if (d) break;
      if ((rc = fp32_step())) return rc;
      CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 0,
                                                       nullptr));
    }
    if (redo_out && cudaMemsetAsync(redo_out, 0, (size_t)batch * sizeof(int), st) != cudaSuccess)
      return LSR_ERR_LAUNCH;
    return LSR_OK;
  }

  // ---- pass 1: tensor cores, to max|M - I| <= sw
  CN_LAUNCH(cn_init_kernel<<<eg, CN_THREADS, 0, st>>>(A, n, epsilon, root, z, nullptr, nullptr, nullptr, Xh, Xl, Mh,
                                                      Ml, errb));
  CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, sw, 1, nullptr));
  for (int it = 0; it < max_iterations; ++it) {
    const int d = done(it);
    if (d < 0) return LSR_ERR_LAUNCH;
    if (d) break;
    CN_LAUNCH(cn_tc_mp_kernel<<<eg, CN_THREADS, 0, st>>>(Mh, Ml, Mph, Mpl, n, alpha, active));
    {
      float* oh[2] = {Xnh, Ph};
      float* ol[2] = {Xnl, Pl};
      const float* ah[2] = {Xh, Mph};
      const float* al[2] = {Xl, Mpl};
      const float* bh[2] = {Mph, Mph};
      const float* bl[2] = {Mpl, Mpl};
      if ((rc = cn_tc_products(2, oh, ol, ah, al, bh, bl, batch, n, active, st))) return rc;
    }
    const float* Prh = Ph;
    const float* Prl = Pl;
    if (root == 4) {
      float* oh[1] = {P2h};
      float* ol[1] = {P2l};
      const float* ah[1] = {Ph};
      const float* al[1] = {Pl};
      if ((rc = cn_tc_products(1, oh, ol, ah, al, ah, al, batch, n, active, st))) return rc;
      Prh = P2h;
      Prl = P2l;
    }
    {
      float* oh[1] = {Mnh};
      float* ol[1] = {Mnl};
      const float* ah[1] = {Prh};
      const float* al[1] = {Prl};
      const float* bh[1] = {Mh};
      const float* bl[1] = {Ml};
      if ((rc = cn_tc_products(1, oh, ol, ah, al, bh, bl, batch, n, active, st))) return rc;
    }
    CN_LAUNCH(cn_tc_commit_kernel<<<eg, CN_THREADS, 0, st>>>(Xh, Xl, Mh, Ml, Xnh, Xnl, Mnh, Mnl, n, active, errb));
    CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, sw, 0, nullptr));
  }

  // ---- pass 2: fp32 FFMA from the tensor-core state to the tolerance
  CN_LAUNCH(cn_tc_unpack_kernel<<<eg, CN_THREADS, 0, st>>>(Xh, Xl, Mh, Ml, X, M, n, errb));
  CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 2, nullptr));
  for (int it = 0; it < max_iterations; ++it) {
    const int d = done(it);
    if (d < 0) return LSR_ERR_LAUNCH;
    if (d) break;
    if ((rc = fp32_step())) return rc;
    CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 0, nullptr));
  }

  // ---- pass 3: ill-conditioned factors from scratch in fp32 FFMA
  CN_LAUNCH(cn_select_kernel<<<cdiv(batch, 256), 256, 0, st>>>(iters, root == 2 ? 14 : 13, redo, batch));
  CN_LAUNCH(cn_init_kernel<<<eg, CN_THREADS, 0, st>>>(A, n, epsilon, root, z, redo, X, M, nullptr, nullptr, nullptr,
                                                      nullptr, errb));
  CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 1, redo));
  for (int it = 0; it < max_iterations; ++it) {
    const int d = done(it);
    if (d < 0) return LSR_ERR_LAUNCH;
    if (d) break;
    if ((rc = fp32_step())) return rc;
    CN_LAUNCH(cn_finalize_kernel<<<1, 1024, 0, st>>>(errb, err, active, iters, nactive, batch, tolerance, 0, redo));
  }
#undef CN_LAUNCH
  if (redo_out && cudaMemcpyAsync(redo_out, redo, (size_t)batch * sizeof(int), cudaMemcpyDeviceToDevice, st) !=
                      cudaSuccess)
    return LSR_ERR_LAUNCH;
  return LSR_OK;
}

}  // extern "C"
