// Newton–Schulz quintic orthogonalisation and the Muon step on sm_100a.
//
// Per shape group and per quintic step three tcgen05 GEMM launches:
//   1. A  = bf16(X X^T)                         upper-triangle tiles, mirrored
//   2. B  = bf16(bf16(b A) + bf16(c bf16(A A)))  upper-triangle tiles, mirrored
//   3. X' = bf16(bf16(a X) + bf16(B X))          X read MN-major by TMA
// The bf16 rounding points are those of the reference's torch ops
// (muon_lm_ddp.py:405-424: bmm -> bf16, scalar*tensor -> bf16, add -> bf16).
//
// Elementwise stages (HBM-bound) around the GEMMs:
//   orient  : momentum / Nesterov update (muon_lm_ddp.py:554-568), transpose of
//             tall matrices (muon_lm_ddp.py:647-650), per-tile sum of squares;
//   finalize: deterministic per-matrix norm -> bf16, clamp at eps
//             (muon_lm_ddp.py:388-401);
//   scale   : X /= norm (bf16 division, in place);
//   apply   : p = bf16(p * (1 - lr*wd)); p = bf16(p - lr_adj * update)
//             (muon_lm_ddp.py:571-593), transposing the update back.
#include <vector>

#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int TILE = 64;
constexpr int EW_THREADS = 256;
constexpr int NS_BN = 256;

typedef __nv_bfloat16 bf16;

// A batch of matrices given either as a device array of addresses or as a
// contiguous base with a batch stride (elements).
struct MatRef {
  const uint64_t* ptrs;
  const void* base;
  long long bstride;
};

__device__ __forceinline__ bf16* mat_at(const MatRef& r, int b) {
  if (r.ptrs) return reinterpret_cast<bf16*>(r.ptrs[b]);
  return const_cast<bf16*>(reinterpret_cast<const bf16*>(r.base)) + (long long)b * r.bstride;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  }
  return t;  // valid in thread 0
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
  return v;
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// 64x64 bf16 tile in shared memory as 64 rows of 32 32-bit words. The word
// index is XOR-swizzled by the row's 8-row group so that reading one column
// for 8 rows 8 apart (the transposed read) hits distinct banks, while each
// 16-byte vector (4 aligned words) of a row stays contiguous.
__device__ __forceinline__ int swz(int row, int word) { return row * 32 + (word ^ (((row >> 3) & 7) << 2)); }

__device__ __forceinline__ float tile_get(const uint32_t* t, int row, int col) {
  const uint32_t w = t[swz(row, col >> 1)];
  const uint16_t h = (col & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
  return __bfloat162float(__ushort_as_bfloat16(h));
}

// Momentum / Nesterov on 8 elements (muon_lm_ddp.py:554-568 rounding order).
template <bool MOMENTUM>
__device__ __forceinline__ void momentum8(const float (&g)[8], float (&buf)[8], float (&u)[8], float mu,
                                          int nesterov) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if constexpr (MOMENTUM) {
      buf[e] = bf16r(bf16r(mu * buf[e]) + g[e]);
      u[e] = nesterov ? bf16r(g[e] + bf16r(mu * buf[e])) : buf[e];
    } else {
      u[e] = g[e];
    }
  }
}

// One block per 64x64 tile of the source matrix (R x C row-major, ld = C).
//   MOMENTUM=false: u = src
//   MOMENTUM=true : buf = bf16(bf16(mu*buf) + g); u = nesterov ? bf16(g + bf16(mu*buf)) : buf
// u is written oriented into X (transposed when `trans`), and the tile's sum of
// u^2 into partials[b * gridDim.x + tile]. 16-byte vector path when the row
// lengths are multiples of 8 and the matrices 16-byte aligned; scalar path
// otherwise (ragged shapes).
template <bool MOMENTUM>
__global__ void __launch_bounds__(EW_THREADS) orient_kernel(MatRef src, MatRef mom, int R, int C, int trans, bf16* X,
                                                            long long x_bs, int ldx, float* partials, float mu,
                                                            int nesterov) {
  __shared__ __align__(16) float smem[TILE * (TILE + 1)];
  __shared__ float red[EW_THREADS / 32];
  const int b = blockIdx.y;
  const int tiles_c = (C + TILE - 1) / TILE;
  const int r0 = (blockIdx.x / tiles_c) * TILE;
  const int c0 = (blockIdx.x % tiles_c) * TILE;
  const bf16* g = mat_at(src, b);
  bf16* buf = MOMENTUM ? mat_at(mom, b) : nullptr;
  bf16* xd = X + (long long)b * x_bs;
  const int tid = threadIdx.x;
  float ss = 0.f;
  const bool vec = (C % 8 == 0) && (!trans || R % 8 == 0) && (ldx % 8 == 0) && aligned16(g) && aligned16(xd) &&
                   (!MOMENTUM || aligned16(buf));
  if (vec) {
    uint32_t* tile = reinterpret_cast<uint32_t*>(smem);
    // both rows' gradient and momentum vectors are loaded before anything is
    // stored (the stores could alias later loads, so the compiler would not
    // hoist them): twice the bytes in flight per thread
    uint4 gv[2], bv[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = r0 + (tid >> 3) + 32 * k, c = c0 + 8 * (tid & 7);
      gv[k] = bv[k] = make_uint4(0u, 0u, 0u, 0u);
      if (r < R && c < C) {
        const long long idx = (long long)r * C + c;
        gv[k] = *reinterpret_cast<const uint4*>(g + idx);
        if constexpr (MOMENTUM) bv[k] = *reinterpret_cast<const uint4*>(buf + idx);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = (tid >> 3) + 32 * k;
      const int v = tid & 7;
      const int r = r0 + i, c = c0 + 8 * v;
      float u[8];
      if (r < R && c < C) {
        const long long idx = (long long)r * C + c;
        float gf[8], bf[8];
        unpack8(gv[k], gf);
        if constexpr (MOMENTUM) unpack8(bv[k], bf);
        momentum8<MOMENTUM>(gf, bf, u, mu, nesterov);
        if constexpr (MOMENTUM) *reinterpret_cast<uint4*>(buf + idx) = pack8(bf);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(u[e], u[e], ss);
        if (!trans) *reinterpret_cast<uint4*>(xd + (long long)r * ldx + c) = pack8(u);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) u[e] = 0.f;
      }
      if (trans) *reinterpret_cast<uint4*>(&tile[swz(i, 4 * v)]) = pack8(u);
    }
    if (trans) {
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int cc = (tid >> 3) + 32 * k;  // source column offset = destination row offset
        const int v = tid & 7;               // destination columns = source rows r0 + 8v .. +7
        const int xr = c0 + cc, xc = r0 + 8 * v;
        if (xr < C && xc < R) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = tile_get(tile, 8 * v + e, cc);
          *reinterpret_cast<uint4*>(xd + (long long)xr * ldx + xc) = pack8(f);
        }
      }
    }
  } else {
    float(*tile)[TILE + 1] = reinterpret_cast<float(*)[TILE + 1]>(smem);
    const int tx = tid & 31, ty = tid >> 5;
#pragma unroll 2
    for (int k = 0; k < TILE / 8; ++k) {
      const int i = ty + 8 * k;
      const int r = r0 + i;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * tx + e;
        const int c = c0 + j;
        float u = 0.f;
        if (r < R && c < C) {
          const long long idx = (long long)r * C + c;
          const float gv = __bfloat162float(g[idx]);
          if constexpr (MOMENTUM) {
            float bv = __bfloat162float(buf[idx]);
            bv = bf16r(bf16r(mu * bv) + gv);
            buf[idx] = __float2bfloat16_rn(bv);
            u = nesterov ? bf16r(gv + bf16r(mu * bv)) : bv;
          } else {
            u = gv;
          }
          ss = fmaf(u, u, ss);
          if (!trans) xd[(long long)r * ldx + c] = __float2bfloat16_rn(u);
        }
        tile[i][j] = u;
      }
    }
    if (trans) {
      __syncthreads();
#pragma unroll 2
      for (int k = 0; k < TILE / 8; ++k) {
        const int jj = ty + 8 * k;
        const int dr = c0 + jj;
        if (dr >= C) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int ii = 2 * tx + e;
          if (r0 + ii < R) xd[(long long)dr * ldx + (r0 + ii)] = __float2bfloat16_rn(tile[ii][jj]);
        }
      }
    }
  }
  const float t = block_sum(ss, red);
  if (threadIdx.x == 0) partials[(long long)b * gridDim.x + blockIdx.x] = t;
}

// nrm[b] = max(bf16(sqrt(sum of partials)), bf16(eps)); fixed summation order.
__global__ void __launch_bounds__(EW_THREADS) norm_finalize_kernel(const float* partials, int nparts, float eps,
                                                                   float* nrm) {
  __shared__ float red[EW_THREADS / 32];
  const int b = blockIdx.x;
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += partials[(long long)b * nparts + i];
  const float t = block_sum(s, red);
  if (threadIdx.x == 0) {
    const float n = bf16r(sqrtf(t));
    const float e = bf16r(eps);
    nrm[b] = n < e ? e : n;
  }
}

// X[b] (m x n, row stride ldx) = bf16(X / nrm[b]); one block per row.
__global__ void __launch_bounds__(EW_THREADS) scale_kernel(bf16* X, long long x_bs, int ldx, int n, const float* nrm) {
  const int b = blockIdx.y;
  const float d = nrm[b];
  bf16* row = X + (long long)b * x_bs + (long long)blockIdx.x * ldx;
  if ((n % 8 == 0) && aligned16(row)) {
    for (int j = 8 * threadIdx.x; j < n; j += 8 * blockDim.x) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + j), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __fdiv_rn(f[e], d);
      *reinterpret_cast<uint4*>(row + j) = pack8(f);
    }
  } else {
    for (int j = threadIdx.x; j < n; j += blockDim.x)
      row[j] = __float2bfloat16_rn(__fdiv_rn(__bfloat162float(row[j]), d));
  }
}

// One block per 64x64 tile of the parameter matrix (R x C). U holds the
// oriented update (m x n, row stride ldu; U[j][i] = update[i][j] when trans).
//   p = bf16(p * wd_factor)   (if apply_wd)
//   p = bf16(p + neg_lr * u)
__global__ void __launch_bounds__(EW_THREADS) apply_kernel(MatRef param, int R, int C, int trans, const bf16* U,
                                                           long long u_bs, int ldu, float wd_factor, int apply_wd,
                                                           float neg_lr) {
  __shared__ __align__(16) float smem[TILE * (TILE + 1)];
  const int b = blockIdx.y;
  const int tiles_c = (C + TILE - 1) / TILE;
  const int r0 = (blockIdx.x / tiles_c) * TILE;
  const int c0 = (blockIdx.x % tiles_c) * TILE;
  bf16* p = mat_at(param, b);
  const bf16* u = U + (long long)b * u_bs;
  const int tid = threadIdx.x;
  const bool vec = (C % 8 == 0) && (!trans || R % 8 == 0) && (ldu % 8 == 0) && aligned16(p) && aligned16(u);
  if (vec) {
    uint32_t* tile = reinterpret_cast<uint32_t*>(smem);
    if (trans) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int uu = (tid >> 3) + 32 * k;  // U row offset = parameter column offset
        const int v = tid & 7;               // U columns = parameter rows r0 + 8v .. +7
        const int ur = c0 + uu, uc = r0 + 8 * v;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (ur < C && uc < R) val = *reinterpret_cast<const uint4*>(u + (long long)ur * ldu + uc);
        *reinterpret_cast<uint4*>(&tile[swz(uu, 4 * v)]) = val;
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = (tid >> 3) + 32 * k;
      const int v = tid & 7;
      const int r = r0 + i, c = c0 + 8 * v;
      if (r >= R || c >= C) continue;
      float uf[8], pf[8];
      if (trans) {
#pragma unroll
        for (int e = 0; e < 8; ++e) uf[e] = tile_get(tile, 8 * v + e, i);
      } else {
        unpack8(*reinterpret_cast<const uint4*>(u + (long long)r * ldu + c), uf);
      }
      const long long idx = (long long)r * C + c;
      unpack8(*reinterpret_cast<const uint4*>(p + idx), pf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float pv = pf[e];
        if (apply_wd) pv = bf16r(pv * wd_factor);
        pf[e] = fmaf(neg_lr, uf[e], pv);
      }
      *reinterpret_cast<uint4*>(p + idx) = pack8(pf);
    }
    return;
  }
  float(*tile)[TILE + 1] = reinterpret_cast<float(*)[TILE + 1]>(smem);
  const int tx = tid & 31, ty = tid >> 5;
  if (trans) {
#pragma unroll 2
    for (int k = 0; k < TILE / 8; ++k) {
      const int jj = ty + 8 * k;
      const int ur = c0 + jj;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ii = 2 * tx + e;
        tile[ii][jj] = (ur < C && r0 + ii < R) ? __bfloat162float(u[(long long)ur * ldu + r0 + ii]) : 0.f;
      }
    }
    __syncthreads();
  }
#pragma unroll 2
  for (int k = 0; k < TILE / 8; ++k) {
    const int i = ty + 8 * k;
    const int r = r0 + i;
    if (r >= R) continue;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 2 * tx + e;
      const int c = c0 + j;
      if (c >= C) continue;
      const float uv = trans ? tile[i][j] : __bfloat162float(u[(long long)r * ldu + c]);
      const long long idx = (long long)r * C + c;
      float pv = __bfloat162float(p[idx]);
      if (apply_wd) pv = bf16r(pv * wd_factor);
      p[idx] = __float2bfloat16_rn(fmaf(neg_lr, uv, pv));
    }
  }
}

// dst (R x C, contiguous per matrix) = oriented src (m x n, row stride lds),
// transposed back when `trans`. Used when no GEMM step writes the output.
__global__ void __launch_bounds__(EW_THREADS) copy_out_kernel(const bf16* S, long long s_bs, int lds, bf16* D,
                                                              int R, int C, int trans) {
  const int b = blockIdx.y;
  const long long total = (long long)R * C;
  const bf16* s = S + (long long)b * s_bs;
  bf16* d = D + (long long)b * total;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / C), c = (int)(idx % C);
    d[idx] = trans ? s[(long long)c * lds + r] : s[(long long)r * lds + c];
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct NsGroup {
  int batch = 0, m = 0, n = 0, ldn = 0, ldm = 0;
  bf16* X[2] = {nullptr, nullptr};
  bf16* A = nullptr;
  bf16* B = nullptr;
  float* partials = nullptr;
  float* nrm = nullptr;
  int nparts = 0;
  // destination of the last step (nullptr: stay in X[steps & 1])
  void* final_out = nullptr;
  int final_ld = 0;
  int final_trans = 0;
  long long final_bs = 0;
};

struct Carver {
  uint8_t* p;
  size_t used = 0;
  template <typename T>
  T* take(size_t bytes) {
    T* r = reinterpret_cast<T*>(p ? p + used : nullptr);
    used += align_up(bytes, 256);
    return r;
  }
};

// Partition workspace for one group (rows x cols source shape, already oriented m x n).
void carve_group(Carver& cv, NsGroup& G, int batch, int m, int n, int src_tiles) {
  G.batch = batch;
  G.m = m;
  G.n = n;
  G.ldn = (int)align_up(n, 8);
  G.ldm = (int)align_up(m, 8);
  G.X[0] = cv.take<bf16>((size_t)batch * m * G.ldn * 2);
  G.X[1] = cv.take<bf16>((size_t)batch * m * G.ldn * 2);
  G.A = cv.take<bf16>((size_t)batch * m * G.ldm * 2);
  G.B = cv.take<bf16>((size_t)batch * m * G.ldm * 2);
  G.nparts = src_tiles;
  G.partials = cv.take<float>((size_t)batch * src_tiles * 4);
  G.nrm = cv.take<float>((size_t)batch * 4);
}

inline int src_tiles(int R, int C) { return cdiv(R, TILE) * cdiv(C, TILE); }

int launch_ok() { return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH; }

// Norm finalize + in-place scale of X[0] for one group.
int normalize_group(NsGroup& G, float eps, cudaStream_t st) {
  {
    ProfScope prof(PK_EW_NORMALIZE, st);
    norm_finalize_kernel<<<G.batch, EW_THREADS, 0, st>>>(G.partials, G.nparts, eps, G.nrm);
  }
  if (launch_ok()) return LSR_ERR_LAUNCH;
  ProfScope prof(PK_EW_NORMALIZE, st);
  scale_kernel<<<dim3(G.m, G.batch), EW_THREADS, 0, st>>>(G.X[0], (long long)G.m * G.ldn, G.ldn, G.n, G.nrm);
  return launch_ok();
}

// `steps` quintic iterations over up to kMaxGroups groups.
template <int EPI>
int launch_ns(GemmParams& p, cudaStream_t st, int kind, bool pair) {
  if (pair) return launch_gemm<NS_BN, EPI, default_stages<EPI, 1>(), 0, 0, 1>(p, st, kind);
  return launch_gemm<NS_BN, EPI>(p, st, kind);
}

int ns_iterations(NsGroup* gs, int ng, int steps, float a, float b, float c, cudaStream_t st) {
  constexpr int BN = NS_BN;
  // Matrices taller than one 128-row tile run on CTA pairs: 256-row tiles, each
  // CTA loading half of operand B, so the tensor cores need a third less
  // operand bandwidth per flop.
  bool pair = false;
#ifndef LSR_NS_SINGLE_CTA
  for (int g = 0; g < ng; ++g) pair |= gs[g].m > BM;
#endif
  const int BB = pair ? BN / 2 : BN;  // operand-B box rows
  for (int it = 0; it < steps; ++it) {
    const int cur = it & 1, nxt = cur ^ 1;
    const bool last = it == steps - 1;
    GemmParams p1{}, p2{}, p3{};
    p1.ngroups = p2.ngroups = p3.ngroups = ng;
    for (int g = 0; g < ng; ++g) {
      NsGroup& S = gs[g];
      const long long xbs = (long long)S.m * S.ldn, abs_ = (long long)S.m * S.ldm;
      // phase 1: A = X X^T
      Operand xk{S.X[cur], S.m, S.n, S.ldn, xbs, S.batch, 0};
      int rc = make_operand_map(&p1.mapA[g][0], xk, false, BN);
      if (!rc) rc = make_operand_map(&p1.mapB[g][0], xk, true, BB);
      GroupDesc& G1 = p1.g[g];
      G1.batch = S.batch;
      G1.M = G1.N = S.m;
      G1.tri = 1;
      G1.nseg = 1;
      G1.seg[0] = SegDesc{cdiv(S.n, BK), 0, 0, 0, 0};
      G1.out = S.A;
      G1.out_bs = abs_;
      G1.ldo = S.ldm;
      G1.alpha = 1.f;
      // phase 2: B = b A + c A A
      Operand ak{S.A, S.m, S.m, S.ldm, abs_, S.batch, 0};
      if (!rc) rc = make_operand_map(&p2.mapA[g][0], ak, false, BN);
      if (!rc) rc = make_operand_map(&p2.mapB[g][0], ak, true, BB);
      GroupDesc& G2 = p2.g[g];
      G2.batch = S.batch;
      G2.M = G2.N = S.m;
      G2.tri = 1;
      G2.nseg = 1;
      G2.seg[0] = SegDesc{cdiv(S.m, BK), 0, 0, 0, 0};
      G2.out = S.B;
      G2.out_bs = abs_;
      G2.ldo = S.ldm;
      G2.aux = S.A;
      G2.aux_bs = abs_;
      G2.ld_aux = S.ldm;
      G2.alpha = b;
      G2.beta = c;
      // phase 3: X' = a X + B X   (X is the MN-major B operand)
      Operand bk{S.B, S.m, S.m, S.ldm, abs_, S.batch, 0};
      Operand xmn{S.X[cur], S.m, S.n, S.ldn, xbs, S.batch, 1};
      if (!rc) rc = make_operand_map(&p3.mapA[g][0], bk, false, BN);
      if (!rc) rc = make_operand_map(&p3.mapB[g][0], xmn, true, BB);
      if (rc) return rc;
      GroupDesc& G3 = p3.g[g];
      G3.batch = S.batch;
      G3.M = S.m;
      G3.N = S.n;
      G3.tri = 0;
      G3.nseg = 1;
      G3.seg[0] = SegDesc{cdiv(S.m, BK), 0, 1, 0, 0};
      G3.aux = S.X[cur];
      G3.aux_bs = xbs;
      G3.ld_aux = S.ldn;
      G3.alpha = a;
      if (last && S.final_out) {
        G3.out = S.final_out;
        G3.out_bs = S.final_bs;
        G3.ldo = S.final_ld;
        G3.out_trans = S.final_trans;
      } else {
        G3.out = S.X[nxt];
        G3.out_bs = xbs;
        G3.ldo = S.ldn;
      }
    }
    int rc = launch_ns<EPI_NS_GRAM>(p1, st, PK_GEMM_GRAM, pair);
    if (!rc) rc = launch_ns<EPI_NS_POLY>(p2, st, PK_GEMM_POLY, pair);
    if (!rc) rc = launch_ns<EPI_NS_UPDATE>(p3, st, PK_GEMM_UPDATE, pair);
    if (rc) return rc;
  }
  return LSR_OK;
}

int ns_iterations_all(std::vector<NsGroup>& gs, int steps, float a, float b, float c, cudaStream_t st) {
  for (size_t g0 = 0; g0 < gs.size(); g0 += kMaxGroups) {
    const int ng = (int)std::min<size_t>(kMaxGroups, gs.size() - g0);
    int rc = ns_iterations(gs.data() + g0, ng, steps, a, b, c, st);
    if (rc) return rc;
  }
  return LSR_OK;
}

// Copy the un-iterated normalised X (steps == 0) to its destination.
int copy_final(NsGroup& G, int R, int C, cudaStream_t st) {
  if (!G.final_out) return LSR_OK;
  const long long total = (long long)R * C;
  const int blocks = (int)std::min<long long>((total + EW_THREADS - 1) / EW_THREADS, 4096);
  ProfScope prof(PK_EW_OTHER, st);
  copy_out_kernel<<<dim3(blocks, G.batch), EW_THREADS, 0, st>>>(G.X[0], (long long)G.m * G.ldn, G.ldn,
                                                                 reinterpret_cast<bf16*>(G.final_out), R, C,
                                                                 G.final_trans);
  return launch_ok();
}

struct MuonShape {
  int R, C, m, n, trans;
};

MuonShape muon_shape(const lsr_muon_group& g) {
  MuonShape s;
  s.R = g.rows;
  s.C = g.cols;
  s.trans = g.rows > g.cols;
  s.m = s.trans ? g.cols : g.rows;
  s.n = s.trans ? g.rows : g.cols;
  return s;
}

bool valid_groups(const lsr_muon_group* groups, int ngroups) {
  if (!groups || ngroups < 0) return false;
  for (int i = 0; i < ngroups; ++i) {
    const lsr_muon_group& g = groups[i];
    if (g.rows <= 0 || g.cols <= 0 || g.count < 0) return false;
  }
  return true;
}

size_t muon_carve(const lsr_muon_group* groups, int ngroups, uint8_t* ws, std::vector<NsGroup>* out) {
  Carver cv{ws};
  for (int i = 0; i < ngroups; ++i) {
    const MuonShape s = muon_shape(groups[i]);
    NsGroup G;
    carve_group(cv, G, std::max(groups[i].count, 1), s.m, s.n, src_tiles(s.R, s.C));
    G.batch = groups[i].count;
    if (out) out->push_back(G);
  }
  return cv.used + 256;
}

// Momentum + orientation + normalisation + NS for all groups; results land in
// G.final_out when set, else in G.X[steps & 1].
// phase bit 1: momentum / orientation / normalisation into the workspace;
// phase bit 2: Newton–Schulz iterations from the workspace into the outputs.
int muon_orthogonalize(const lsr_muon_group* groups, int ngroups, std::vector<NsGroup>& gs, float mu, int nesterov,
                       int steps, float a, float b, float c, float eps, cudaStream_t st, int phase = 3) {
  std::vector<NsGroup> live;
  std::vector<int> live_idx;
  for (int i = 0; i < ngroups; ++i) {
    const lsr_muon_group& g = groups[i];
    if (g.count == 0) continue;
    if (!(phase & 1)) {
      live.push_back(gs[i]);
      live_idx.push_back(i);
      continue;
    }
    if (!g.grad_ptrs || !g.mom_ptrs) return LSR_ERR_ARG;
    const MuonShape s = muon_shape(g);
    NsGroup& G = gs[i];
    MatRef gr{g.grad_ptrs, nullptr, 0}, mo{g.mom_ptrs, nullptr, 0};
    ProfScope prof(PK_EW_ORIENT, st);
    orient_kernel<true><<<dim3(G.nparts, g.count), EW_THREADS, 0, st>>>(gr, mo, s.R, s.C, s.trans, G.X[0],
                                                                         (long long)G.m * G.ldn, G.ldn, G.partials,
                                                                         mu, nesterov);
    if (launch_ok()) return LSR_ERR_LAUNCH;
    int rc = normalize_group(G, eps, st);
    if (rc) return rc;
    live.push_back(G);
    live_idx.push_back(i);
  }
  if (!(phase & 2)) return LSR_OK;
  if (steps == 0) {
    for (size_t k = 0; k < live.size(); ++k) {
      NsGroup& G = live[k];
      if (G.final_out) {
        int rc = copy_final(G, G.m, G.n, st);
        if (rc) return rc;
      }
    }
    return LSR_OK;
  }
  return ns_iterations_all(live, steps, a, b, c, st);
}

int muon_apply(const lsr_muon_group* groups, int ngroups, const bf16* const* upd, const long long* upd_bs,
               const int* upd_ld, float wd, float base_lr, cudaStream_t st) {
  const float wd_factor = (float)(1.0 - (double)base_lr * (double)wd);
  for (int i = 0; i < ngroups; ++i) {
    const lsr_muon_group& g = groups[i];
    if (g.count == 0) continue;
    if (!g.param_ptrs || !upd[i]) return LSR_ERR_ARG;
    const MuonShape s = muon_shape(g);
    MatRef pr{g.param_ptrs, nullptr, 0};
    ProfScope prof(PK_EW_APPLY, st);
    apply_kernel<<<dim3(src_tiles(s.R, s.C), g.count), EW_THREADS, 0, st>>>(
        pr, s.R, s.C, s.trans, upd[i], upd_bs[i], upd_ld[i], wd_factor, wd != 0.f, -g.lr);
    if (launch_ok()) return LSR_ERR_LAUNCH;
  }
  return LSR_OK;
}

}  // namespace

// Newton–Schulz over a caller-provided scratch region that is already sized and
// 256-byte aligned; used by the allocation-free entry point (noalloc.cu). It
// makes no host or device allocation of its own.
int ns_bf16_fixed_scratch(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a,
                          float b, float c, float eps, uint8_t* scratch, cudaStream_t st) {
  const bool trans = orient && rows > cols;
  const int m = trans ? cols : rows, n = trans ? rows : cols;
  Carver cv{scratch};
  NsGroup G;
  carve_group(cv, G, batch, m, n, src_tiles(rows, cols));
  G.final_out = out;
  G.final_trans = trans;
  G.final_ld = trans ? m : n;
  G.final_bs = (long long)rows * cols;
  MatRef src{nullptr, in, (long long)rows * cols}, none{nullptr, nullptr, 0};
  {
    ProfScope prof(PK_EW_ORIENT, st);
    orient_kernel<false><<<dim3(G.nparts, batch), EW_THREADS, 0, st>>>(src, none, rows, cols, trans, G.X[0],
                                                                      (long long)m * G.ldn, G.ldn, G.partials, 0.f, 0);
  }
  if (launch_ok()) return LSR_ERR_LAUNCH;
  int rc = normalize_group(G, eps, st);
  if (rc) return rc;
  if (steps == 0) return copy_final(G, rows, cols, st);
  return ns_iterations(&G, 1, steps, a, b, c, st);
}

}  // namespace lsr

using namespace lsr;

extern "C" {

size_t lsr_ns_workspace_bytes(int batch, int rows, int cols, int orient) {
  if (batch < 0 || rows <= 0 || cols <= 0) return 0;
  const bool trans = orient && rows > cols;
  const int m = trans ? cols : rows, n = trans ? rows : cols;
  Carver cv{nullptr};
  NsGroup G;
  carve_group(cv, G, std::max(batch, 1), m, n, src_tiles(rows, cols));
  return cv.used + 256;
}

int lsr_ns_bf16(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a, float b,
                float c, float eps, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (batch < 0 || rows <= 0 || cols <= 0 || steps < 0 || batch > 65535) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!in || !out) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  const size_t need = lsr_ns_workspace_bytes(batch, rows, cols, orient);
  if (!ws || ws_bytes < need) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool trans = orient && rows > cols;
  const int m = trans ? cols : rows, n = trans ? rows : cols;
  uint8_t* base = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  Carver cv{base};
  NsGroup G;
  carve_group(cv, G, batch, m, n, src_tiles(rows, cols));
  G.final_out = out;
  G.final_trans = trans;
  G.final_ld = trans ? m : n;  // out has the input's shape rows x cols
  G.final_bs = (long long)rows * cols;
  MatRef src{nullptr, in, (long long)rows * cols}, none{nullptr, nullptr, 0};
  {
    ProfScope prof(PK_EW_ORIENT, st);
    orient_kernel<false><<<dim3(G.nparts, batch), EW_THREADS, 0, st>>>(src, none, rows, cols, trans, G.X[0],
                                                                      (long long)m * G.ldn, G.ldn, G.partials, 0.f, 0);
  }
  if (launch_ok()) return LSR_ERR_LAUNCH;
  rc = normalize_group(G, eps, st);
  if (rc) return rc;
  if (steps == 0) return copy_final(G, rows, cols, st);
  std::vector<NsGroup> gs{G};
  return ns_iterations_all(gs, steps, a, b, c, st);
}

size_t lsr_muon_workspace_bytes(const lsr_muon_group* groups, int ngroups) {
  if (!valid_groups(groups, ngroups)) return 0;
  return muon_carve(groups, ngroups, nullptr, nullptr);
}

int lsr_muon_step_bf16(const lsr_muon_group* groups, int ngroups, float momentum, int nesterov, float weight_decay,
                       float base_lr, int ns_steps, float a, float b, float c, float eps, void* ws, size_t ws_bytes,
                       lsr_stream_t stream) {
  if (!valid_groups(groups, ngroups) || ns_steps < 0) return LSR_ERR_ARG;
  for (int i = 0; i < ngroups; ++i)
    if (groups[i].count > 65535) return LSR_ERR_SHAPE;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_muon_workspace_bytes(groups, ngroups)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  std::vector<NsGroup> gs;
  muon_carve(groups, ngroups, reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256)), &gs);
  rc = muon_orthogonalize(groups, ngroups, gs, momentum, nesterov, ns_steps, a, b, c, eps, st);
  if (rc) return rc;
  std::vector<const bf16*> upd(ngroups);
  std::vector<long long> bs(ngroups);
  std::vector<int> ld(ngroups);
  for (int i = 0; i < ngroups; ++i) {
    upd[i] = gs[i].X[ns_steps & 1];
    bs[i] = (long long)gs[i].m * gs[i].ldn;
    ld[i] = gs[i].ldn;
  }
  return muon_apply(groups, ngroups, upd.data(), bs.data(), ld.data(), weight_decay, base_lr, st);
}

int lsr_muon_orthogonalize_bf16(const lsr_muon_group* groups, int ngroups, float momentum, int nesterov, int ns_steps,
                                float a, float b, float c, float eps, void* const* updates, void* ws, size_t ws_bytes,
                                lsr_stream_t stream) {
  return lsr_muon_orthogonalize_phase_bf16(groups, ngroups, momentum, nesterov, ns_steps, a, b, c, eps, updates, 3, ws,
                                           ws_bytes, stream);
}

int lsr_muon_orthogonalize_phase_bf16(const lsr_muon_group* groups, int ngroups, float momentum, int nesterov,
                                      int ns_steps, float a, float b, float c, float eps, void* const* updates,
                                      int phase, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (phase < 1 || phase > 3) return LSR_ERR_ARG;
  if (!valid_groups(groups, ngroups) || ns_steps < 0 || !updates) return LSR_ERR_ARG;
  for (int i = 0; i < ngroups; ++i) {
    if (groups[i].count > 65535) return LSR_ERR_SHAPE;
    if (groups[i].count > 0 && !updates[i]) return LSR_ERR_ARG;
  }
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_muon_workspace_bytes(groups, ngroups)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  std::vector<NsGroup> gs;
  muon_carve(groups, ngroups, reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256)), &gs);
  for (int i = 0; i < ngroups; ++i) {
    gs[i].final_out = updates[i];
    gs[i].final_ld = gs[i].n;
    gs[i].final_bs = (long long)gs[i].m * gs[i].n;
    gs[i].final_trans = 0;
  }
  return muon_orthogonalize(groups, ngroups, gs, momentum, nesterov, ns_steps, a, b, c, eps, st, phase);
}

int lsr_muon_apply_bf16(const lsr_muon_group* groups, int ngroups, const void* const* updates, float weight_decay,
                        float base_lr, lsr_stream_t stream) {
  if (!valid_groups(groups, ngroups) || !updates) return LSR_ERR_ARG;
  for (int i = 0; i < ngroups; ++i)
    if (groups[i].count > 65535) return LSR_ERR_SHAPE;
  int rc = check_device();
  if (rc) return rc;
  std::vector<const bf16*> upd(ngroups);
  std::vector<long long> bs(ngroups);
  std::vector<int> ld(ngroups);
  for (int i = 0; i < ngroups; ++i) {
    const MuonShape s = muon_shape(groups[i]);
    upd[i] = reinterpret_cast<const bf16*>(updates[i]);
    bs[i] = (long long)s.m * s.n;
    ld[i] = s.n;
  }
  return muon_apply(groups, ngroups, upd.data(), bs.data(), ld.data(), weight_decay, base_lr,
                    reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
