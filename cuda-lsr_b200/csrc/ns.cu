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
//   prologue: one persistent launch over every group: momentum / Nesterov
//             update (muon_lm_ddp.py:554-568), transpose of tall matrices
//             (muon_lm_ddp.py:647-650), deterministic per-matrix norm -> bf16,
//             clamp at eps, and X /= norm (muon_lm_ddp.py:388-401), the
//             division done while X is still in L2;
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

// ---------------------------------------------------------------------------
// Prologue: momentum / Nesterov, orientation and Frobenius normalisation of
// every matrix of up to kMaxProGroups shape groups in ONE persistent launch.
//
// Work items (claimed in order from one global counter) are of two kinds:
//   phase 1 — one 64x64 tile of a source matrix (R x C row-major):
//             buf = bf16(bf16(mu*buf) + g); u = nesterov ? bf16(g + bf16(mu*buf)) : buf
//             (muon_lm_ddp.py:554-568), u stored oriented into X (transposed
//             through shared memory when R > C, muon_lm_ddp.py:647-650), the
//             tile's sum of u^2 into partials; the block that completes a
//             matrix's last tile sums its partials in a fixed order and
//             publishes nrm = max(bf16(sqrt(sum)), bf16(eps)) and a ready flag
//             (muon_lm_ddp.py:388-401: the norm is a bf16 scalar);
//   phase 2 — one 64x128 tile of X: X = bf16(X / nrm)  (X.div_(norm)).
// Within a group, matrix k's phase-2 tiles follow matrix k+L's phase-1 tiles
// (L = the lag: roughly 16 MB of X), so a matrix is finished before its scale
// tiles are claimed and part of its X is still in L2 when it is rescaled: DRAM
// sees the 8 bytes per parameter of the momentum/orient pass (read g, buf;
// write buf, X) plus the rescale's L2 misses. Lags of 8, 16, 24, 32 and 48 MB
// measured 4.6, 4.55, 4.76, 4.79 and 4.82 ms per GPT-2-XL step: a shorter lag
// keeps more of X in L2, until the scale tiles start waiting for norms.
// Every phase-2 tile's wait is for phase-1 tiles claimed earlier from the same
// counter, i.e. already running, so it ends; it is bounded all the same
// (LSR_WAIT_TIMEOUT_NS, then a status code and the tile is skipped).
// ---------------------------------------------------------------------------

constexpr int PRO_THREADS = 256;
constexpr int kMaxProGroups = 8;
constexpr int P1_ROWS = 64, P1_COLS = 128;  // phase-1 item: source tile
constexpr int P2_ROWS = 64, P2_COLS = 256;  // phase-2 item: X tile

struct ProGroup {
  MatRef src, mom;  // gradients (or the matrices to orthogonalise) and momentum buffers, R x C
  bf16* X;          // oriented output [count][m][ldx]
  long long x_bs;
  int ldx;
  int R, C, trans, m, n;
  int count;
  int tiles_c;   // 64-wide source tiles per row
  int T;         // phase-1 tiles per matrix
  int p2_c;      // phase-2 tiles per X row band
  int S;         // phase-2 tiles per matrix
  int L;         // lag (matrices), 1 <= L <= count
  int vec;       // 16-byte vector path for phase 1
  unsigned item_begin, items;
  float* partials;  // [count][T]
  float* nrm;       // [count]
  unsigned* done;   // [count], zero at launch
  unsigned* ready;  // [count], zero at launch
};

struct ProParams {
  ProGroup g[kMaxProGroups];
  int ngroups;
  unsigned total_items;
  unsigned* claim;  // zero at launch
  int* status;
  float mu, eps;
  int nesterov;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Block-wide sum with a fixed reduction order; every thread gets the result.
__device__ __forceinline__ float block_sum_all(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();  // red[] free (previous use done)
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < PRO_THREADS / 32; ++i) t += red[i];
  return t;
}

struct ProItem {
  int g, phase, b, t;
};

__device__ __forceinline__ ProItem decode_pro(const ProParams& p, unsigned item) {
  ProItem it{0, 1, 0, 0};
  int g = 0;
  while (g + 1 < p.ngroups && item >= p.g[g + 1].item_begin) ++g;
  const ProGroup& G = p.g[g];
  it.g = g;
  unsigned local = item - G.item_begin;
  const unsigned T = G.T, S = G.S, L = G.L, B = G.count;
  const unsigned r1 = L * T, r2 = (B - L) * (T + S);
  if (local < r1) {
    it.b = local / T;
    it.t = local % T;
  } else if (local - r1 < r2) {
    const unsigned l2 = local - r1, k = L + l2 / (T + S), o = l2 % (T + S);
    if (o < T) {
      it.b = k;
      it.t = o;
    } else {
      it.phase = 2;
      it.b = k - L;
      it.t = o - T;
    }
  } else {
    const unsigned l3 = local - r1 - r2;
    it.phase = 2;
    it.b = B + l3 / S - L;
    it.t = l3 % S;
  }
  return it;
}

// Phase 1 on one 64 x 128 source tile (P1_ROWS x P1_COLS); returns this
// thread's share of the tile's sum of u^2. Vector path: thread t owns rows
// (t / 16) + 16 k, k < 4, and the 8 columns 8 (t % 16): four 16-byte vectors
// of g and of buf are loaded before anything is stored (128 bytes in flight
// per thread). Transposed groups go through a 64 x 128 bf16 tile in shared
// memory (rows of 64 words, XOR-swizzled by 8-row group).
__device__ __forceinline__ int swz128(int row, int word) { return row * 64 + (word ^ (((row >> 3) & 7) << 2)); }

__device__ __forceinline__ float tile128_get(const uint32_t* t, int row, int col) {
  const uint32_t w = t[swz128(row, col >> 1)];
  const uint16_t h = (col & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
  return __bfloat162float(__ushort_as_bfloat16(h));
}

template <bool MOMENTUM>
__device__ __forceinline__ float pro_phase1(const ProGroup& G, int b, int t, float mu, int nesterov, float* smem) {
  const int R = G.R, C = G.C, trans = G.trans;
  const int r0 = (t / G.tiles_c) * P1_ROWS;
  const int c0 = (t % G.tiles_c) * P1_COLS;
  const bf16* g = mat_at(G.src, b);
  bf16* buf = MOMENTUM ? mat_at(G.mom, b) : nullptr;
  bf16* xd = G.X + (long long)b * G.x_bs;
  const int ldx = G.ldx;
  const int tid = threadIdx.x;
  float ss = 0.f;
  // block-uniform: every thread of the block works on the same matrix
  if (G.vec && aligned16(g) && aligned16(xd) && (!MOMENTUM || aligned16(buf))) {
    uint32_t* tile = reinterpret_cast<uint32_t*>(smem);
    uint4 gv[4], bv[4];
    const int v = tid & 15;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = r0 + (tid >> 4) + 16 * k, c = c0 + 8 * v;
      gv[k] = bv[k] = make_uint4(0u, 0u, 0u, 0u);
      if (r < R && c < C) {
        const long long idx = (long long)r * C + c;
        gv[k] = __ldcs(reinterpret_cast<const uint4*>(g + idx));
        if constexpr (MOMENTUM) bv[k] = __ldcs(reinterpret_cast<const uint4*>(buf + idx));
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = (tid >> 4) + 16 * k;
      const int r = r0 + i, c = c0 + 8 * v;
      float u[8];
      if (r < R && c < C) {
        const long long idx = (long long)r * C + c;
        float gf[8], bf[8];
        unpack8(gv[k], gf);
        if constexpr (MOMENTUM) unpack8(bv[k], bf);
        momentum8<MOMENTUM>(gf, bf, u, mu, nesterov);
        if constexpr (MOMENTUM) __stcs(reinterpret_cast<uint4*>(buf + idx), pack8(bf));
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(u[e], u[e], ss);
        if (!trans) *reinterpret_cast<uint4*>(xd + (long long)r * ldx + c) = pack8(u);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) u[e] = 0.f;
      }
      if (trans) *reinterpret_cast<uint4*>(&tile[swz128(i, 4 * v)]) = pack8(u);
    }
    if (trans) {
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int cc = (tid >> 3) + 32 * k;  // source column offset = destination row offset (< 128)
        const int vv = tid & 7;              // destination columns = source rows r0 + 8 vv .. +7
        const int xr = c0 + cc, xc = r0 + 8 * vv;
        if (xr < C && xc < R) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = tile128_get(tile, 8 * vv + e, cc);
          *reinterpret_cast<uint4*>(xd + (long long)xr * ldx + xc) = pack8(f);
        }
      }
    }
    return ss;
  }
  // scalar path (ragged shapes or unaligned matrices): the tile as two 64 x 64 halves
  float(*tl)[TILE + 1] = reinterpret_cast<float(*)[TILE + 1]>(smem);
  const int tx = tid & 31, ty = tid >> 5;
  for (int half = 0; half < P1_COLS / TILE; ++half) {
    const int hc0 = c0 + half * TILE;
    if (trans && half) __syncthreads();  // the previous half's transposed reads are done
#pragma unroll 2
    for (int k = 0; k < TILE / 8; ++k) {
      const int i = ty + 8 * k;
      const int r = r0 + i;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * tx + e;
        const int c = hc0 + j;
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
        tl[i][j] = u;
      }
    }
    if (trans) {
      __syncthreads();
#pragma unroll 2
      for (int k = 0; k < TILE / 8; ++k) {
        const int jj = ty + 8 * k;
        const int dr = hc0 + jj;
        if (dr >= C) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int ii = 2 * tx + e;
          if (r0 + ii < R) xd[(long long)dr * ldx + (r0 + ii)] = __float2bfloat16_rn(tl[ii][jj]);
        }
      }
    }
  }
  return ss;
}

// Phase 2 on one 64 x 256 tile of X: X = bf16(X / d). Thread t owns rows
// (t / 32) + 8 k, k < 8, and the 8 columns 8 (t % 32). X rows are 16-byte
// aligned (ldx is a multiple of 8); vectors that start past n are skipped, the
// padding columns of a vector that straddles n are rescaled harmlessly (never read).
__device__ __forceinline__ void pro_phase2(const ProGroup& G, int b, int t, float d) {
  bf16* xb = G.X + (long long)b * G.x_bs;
  const int r0 = (t / G.p2_c) * P2_ROWS, c0 = (t % G.p2_c) * P2_COLS;
  const int tid = threadIdx.x;
  const int c = c0 + 8 * (tid & 31);
  uint4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + (tid >> 5) + 8 * k;
    v[k] = make_uint4(0u, 0u, 0u, 0u);
    if (r < G.m && c < G.n) v[k] = __ldcg(reinterpret_cast<const uint4*>(xb + (long long)r * G.ldx + c));
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + (tid >> 5) + 8 * k;
    if (r < G.m && c < G.n) {
      float f[8];
      unpack8(v[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __fdiv_rn(f[e], d);
      *reinterpret_cast<uint4*>(xb + (long long)r * G.ldx + c) = pack8(f);
    }
  }
}

template <bool MOMENTUM>
__global__ void __launch_bounds__(PRO_THREADS, 3) prologue_kernel(const __grid_constant__ ProParams p) {
  // 64 x 128 bf16 transpose tile (16 KB) or the scalar path's 64 x 65 fp32 tile
  __shared__ __align__(16) float smem[TILE * (TILE + 1)];
  __shared__ float red[PRO_THREADS / 32];
  __shared__ unsigned s_item[2];
  __shared__ int s_flag;
  if (threadIdx.x == 0) s_item[0] = atomicAdd(p.claim, 1u);
  __syncthreads();
  for (int it_no = 0;; ++it_no) {
    const unsigned item = s_item[it_no & 1];
    if (item >= p.total_items) break;
    // claim the next item now; its value is read after this item's work
    unsigned nxt = 0;
    if (threadIdx.x == 0) nxt = atomicAdd(p.claim, 1u);
    const ProItem w = decode_pro(p, item);
    const ProGroup& G = p.g[w.g];
    if (w.phase == 1) {
      const float ss = pro_phase1<MOMENTUM>(G, w.b, w.t, p.mu, p.nesterov, smem);
      const float tot = block_sum_all(ss, red);
      if (threadIdx.x == 0) {
        G.partials[(long long)w.b * G.T + w.t] = tot;
        __threadfence();
        const unsigned prev = atomicAdd(G.done + w.b, 1u);
        s_flag = (prev == (unsigned)G.T - 1);
      }
      __syncthreads();
      if (s_flag) {
        // last tile of this matrix: every tile's partial sum is visible
        __threadfence();
        float s = 0.f;
        for (int i = threadIdx.x; i < G.T; i += PRO_THREADS) s += __ldcg(G.partials + (long long)w.b * G.T + i);
        const float sum = block_sum_all(s, red);
        if (threadIdx.x == 0) {
          const float n = bf16r(sqrtf(sum));
          const float e = bf16r(p.eps);
          G.nrm[w.b] = n < e ? e : n;
          __threadfence();
          st_release_u32(G.ready + w.b, 1u);
        }
      }
    } else {
      if (threadIdx.x == 0) {
        int ok = 1;
        if (!ld_acquire_u32(G.ready + w.b)) {
          const uint64_t t0 = globaltimer_ns();
          while (!ld_acquire_u32(G.ready + w.b)) {
            if (globaltimer_ns() - t0 > LSR_WAIT_TIMEOUT_NS) {
              set_status(p.status, ST_TIMEOUT_PROLOGUE);
              ok = 0;
              break;
            }
          }
        }
        s_flag = ok;
      }
      __syncthreads();
      if (s_flag) pro_phase2(G, w.b, w.t, __ldcg(G.nrm + w.b));
    }
    if (threadIdx.x == 0) s_item[(it_no + 1) & 1] = nxt;
    __syncthreads();
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
  unsigned* done = nullptr;   // prologue: finished phase-1 tiles per matrix (control region)
  unsigned* ready = nullptr;  // prologue: norm published per matrix (control region)
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

// phase-1 items (and partial sums) per matrix of R x C
inline int src_tiles(int R, int C) { return cdiv(R, P1_ROWS) * cdiv(C, P1_COLS); }

int launch_ok() { return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH; }

// Control words of the prologue launches: one claim counter per launch (own
// 32-byte sector) and done / ready words per matrix. Cleared with one memset
// before the prologue runs.
struct Control {
  unsigned* base = nullptr;
  size_t bytes = 0;
  int nlaunch = 0;
};

inline int prologue_launches(int ngroups) { return std::max(1, cdiv(ngroups, kMaxProGroups)); }

Control carve_control(Carver& cv, int ngroups, long long total_mats) {
  Control c;
  c.nlaunch = prologue_launches(ngroups);
  c.bytes = ((size_t)c.nlaunch * 8 + 2 * (size_t)total_mats) * 4;
  c.base = cv.take<unsigned>(c.bytes);
  return c;
}

// Point each group's done / ready words into the control region.
void bind_control(const Control& c, NsGroup* gs, int ng, long long total_mats) {
  if (!c.base) return;
  long long off = 0;
  for (int i = 0; i < ng; ++i) {
    gs[i].done = c.base + (size_t)c.nlaunch * 8 + off;
    gs[i].ready = c.base + (size_t)c.nlaunch * 8 + total_mats + off;
    off += std::max(gs[i].batch, 1);
  }
}

// Source of a group's prologue: the matrices (rows R x cols C, row-major) and,
// for the Muon step, their momentum buffers.
struct ProSource {
  MatRef src, mom;
  int R, C, trans;
};

template <bool MOMENTUM>
int prologue_grid(int items) {
  static int per_sm = 0;
  if (!per_sm) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, prologue_kernel<MOMENTUM>, PRO_THREADS, 0) != cudaSuccess ||
        n < 1)
      n = 1;
    per_sm = n;
  }
  return std::max(1, std::min(items, per_sm * device_sm_count()));
}

// Momentum / orientation / normalisation of every matrix of the given groups
// into X[0] (one persistent launch per kMaxProGroups groups; see prologue_kernel).
int run_prologue(NsGroup* gs, const ProSource* srcs, int ng, const Control& ctl, bool momentum, float mu,
                 int nesterov, float eps, cudaStream_t st) {
  if (ng == 0) return LSR_OK;
  if (cudaMemsetAsync(ctl.base, 0, ctl.bytes, st) != cudaSuccess) return LSR_ERR_LAUNCH;
  for (int g0 = 0, launch = 0; g0 < ng; g0 += kMaxProGroups, ++launch) {
    ProParams p{};
    p.ngroups = std::min(kMaxProGroups, ng - g0);
    unsigned item = 0;
    for (int k = 0; k < p.ngroups; ++k) {
      const NsGroup& S = gs[g0 + k];
      const ProSource& src = srcs[g0 + k];
      ProGroup& G = p.g[k];
      G.src = src.src;
      G.mom = src.mom;
      G.X = S.X[0];
      G.x_bs = (long long)S.m * S.ldn;
      G.ldx = S.ldn;
      G.R = src.R;
      G.C = src.C;
      G.trans = src.trans;
      G.m = S.m;
      G.n = S.n;
      G.count = S.batch;
      G.tiles_c = cdiv(src.C, P1_COLS);
      G.T = S.nparts;
      G.p2_c = cdiv(S.n, P2_COLS);
      G.S = cdiv(S.m, P2_ROWS) * G.p2_c;
      const double xbytes = 2.0 * S.m * S.ldn;
      G.L = (int)std::min<double>(S.batch, std::max(1.0, std::ceil(16.0 * (1 << 20) / xbytes)));
      G.vec = (src.C % 8 == 0) && (!src.trans || src.R % 8 == 0);  // and 16-byte bases, checked per matrix
      G.partials = S.partials;
      G.nrm = S.nrm;
      G.done = S.done;
      G.ready = S.ready;
      G.item_begin = item;
      G.items = (unsigned)S.batch * (unsigned)(G.T + G.S);
      item += G.items;
    }
    p.total_items = item;
    p.claim = ctl.base + 8 * launch;
    p.status = status_ptr();
    p.mu = mu;
    p.eps = eps;
    p.nesterov = nesterov;
    if (!p.status) return LSR_ERR_LAUNCH;
    if (item == 0) continue;
    ProfScope prof(PK_EW_ORIENT, st);
    if (momentum)
      prologue_kernel<true><<<prologue_grid<true>((int)item), PRO_THREADS, 0, st>>>(p);
    else
      prologue_kernel<false><<<prologue_grid<false>((int)item), PRO_THREADS, 0, st>>>(p);
    if (launch_ok()) return LSR_ERR_LAUNCH;
  }
  return LSR_OK;
}

// `steps` quintic iterations over up to kMaxGroups groups.
template <int EPI, int BN = NS_BN, int KS = 1>
int launch_ns(GemmParams& p, cudaStream_t st, int kind, bool pair) {
  if (pair) return launch_gemm<BN, EPI, default_stages<EPI, 1, BN, KS>(), 0, 0, 1, KS>(p, st, kind);
  return launch_gemm<BN, EPI, default_stages<EPI, 0, BN, KS>(), 0, 0, 0, KS>(p, st, kind);
}

// The update runs two K blocks (128 elements) per pipeline stage when its K
// length (m) and the MN-major rows of X (n) are whole numbers of 64-element
// blocks: half the TMA operations and barrier round trips per flop (GPT-2-XL
// step: 23.5 vs 25.4 ms per step). The symmetric products keep one block per
// stage: their single-CTA tiles fit only two double-width stages, and lost more
// to the shallower pipeline than they gained (X X^T 14.9 vs 13.3 ms).
bool ns_use_ks2(const NsGroup* gs, int ng) {
  for (int g = 0; g < ng; ++g)
    if (gs[g].m % BK || gs[g].n % BK) return false;
  return ng > 0;
}

// Narrow tiles: when every group's oriented row count m is a multiple of
// NS_BN_NARROW but not of the 256-row pair tile (GPT-2-XL: m = 1600 = 10 x 160 =
// 6.25 x 256), the m-wide dimension of every product is tiled exactly:
//   * X X^T and A A (m x m, single CTAs): 128 x 160 tiles, no padded columns;
//   * the update runs transposed, X'^T = X^T B (B is symmetric): the n x m
//     output in 256 x 160 pair tiles, X^T read MN-major, the a X term read
//     transposed by the epilogue and the tile stored transposed.
// Otherwise 128 x 256 / 256 x 256 tiles with the update in its own orientation.
constexpr int NS_BN_NARROW = 160;

constexpr bool kNsNarrowTiles = false;

bool ns_use_narrow(const NsGroup* gs, int ng) {
  if (!kNsNarrowTiles) return false;
  for (int g = 0; g < ng; ++g) {
    const NsGroup& S = gs[g];
    if (S.m % NS_BN_NARROW != 0 || S.m % (2 * BM) == 0) return false;
    // the transposed update needs the staged (TMA) epilogue for its output
    if (S.final_out && ((reinterpret_cast<uintptr_t>(S.final_out) & 15) || S.final_ld % 8 || S.final_bs % 8))
      return false;
  }
  return ng > 0;
}

int ns_iterations(NsGroup* gs, int ng, int steps, float a, float b, float c, cudaStream_t st) {
  const bool narrow = ns_use_narrow(gs, ng);
  const int BN = narrow ? NS_BN_NARROW : NS_BN;
  const int ks = (!narrow && ns_use_ks2(gs, ng)) ? 2 : 1;
  // The update of matrices taller than one 128-row tile runs on CTA pairs:
  // 256-row tiles, each CTA loading half of operand B, so the tensor cores need
  // a third less operand bandwidth per flop. The symmetric products (X X^T and
  // A A, upper-triangle tiles) run on single CTAs: 128-row tiles pad a 1600-row
  // output to 1664 rows instead of 1792 (measured on the GPT-2-XL step with
  // 256-wide tiles: X X^T 12.4 vs 13.4 ms, b A + c A^2 4.9 vs 5.4 ms per step,
  // while the paired update is 1.6 ms faster than single-CTA tiles).
  bool pair = false;
  for (int g = 0; g < ng; ++g) pair |= (narrow ? gs[g].n : gs[g].m) > BM;
  const int BB = pair ? BN / 2 : BN;  // operand-B box rows of the update
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
      if (!rc) rc = make_operand_map(&p1.mapB[g][0], xk, true, BN);
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
      if (!rc) rc = make_operand_map(&p2.mapB[g][0], ak, true, BN);
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
      // phase 3: X' = a X + B X
      GroupDesc& G3 = p3.g[g];
      G3.batch = S.batch;
      G3.tri = 0;
      G3.nseg = 1;
      G3.aux = S.X[cur];
      G3.aux_bs = xbs;
      G3.ld_aux = S.ldn;
      G3.alpha = a;
      Operand bk{S.B, S.m, S.m, S.ldm, abs_, S.batch, 0};
      Operand xmn{S.X[cur], S.m, S.n, S.ldn, xbs, S.batch, 1};
      const bool to_final = last && S.final_out;
      if (!narrow) {
        // X' (m x n) = B X: B K-major, X the MN-major B operand
        G3.seg[0] = SegDesc{cdiv(S.m, BK), 0, 1, 0, 0};
        if (!rc) rc = make_operand_map(&p3.mapA[g][0], bk, false, BN, nullptr, ks);
        if (!rc) rc = make_operand_map(&p3.mapB[g][0], xmn, true, BB, &G3.seg[0].b_mn, ks);
        G3.M = S.m;
        G3.N = S.n;
        G3.out_trans = to_final ? S.final_trans : 0;
      } else {
        // X'^T (n x m) = X^T B: X^T the MN-major A operand, B (symmetric) K-major;
        // the tile's (j, i) element is X'[i][j]
        G3.seg[0] = SegDesc{cdiv(S.m, BK), 1, 0, 0, 0};
        if (!rc) rc = make_operand_map(&p3.mapA[g][0], xmn, false, BN, &G3.seg[0].a_mn);
        if (!rc) rc = make_operand_map(&p3.mapB[g][0], bk, true, BB);
        G3.M = S.n;
        G3.N = S.m;
        G3.aux_trans = 1;
        G3.out_trans = to_final ? !S.final_trans : 1;
      }
      if (rc) return rc;
      if (to_final) {
        G3.out = S.final_out;
        G3.out_bs = S.final_bs;
        G3.ldo = S.final_ld;
      } else {
        G3.out = S.X[nxt];
        G3.out_bs = xbs;
        G3.ldo = S.ldn;
      }
    }
    int rc;
    if (narrow) {
      rc = launch_ns<EPI_NS_GRAM, NS_BN_NARROW>(p1, st, PK_GEMM_GRAM, false);
      if (!rc) rc = launch_ns<EPI_NS_POLY, NS_BN_NARROW>(p2, st, PK_GEMM_POLY, false);
      if (!rc) rc = launch_ns<EPI_NS_UPDATE, NS_BN_NARROW>(p3, st, PK_GEMM_UPDATE, pair);
    } else if (ks == 2) {
      rc = launch_ns<EPI_NS_GRAM>(p1, st, PK_GEMM_GRAM, false);
      if (!rc) rc = launch_ns<EPI_NS_POLY>(p2, st, PK_GEMM_POLY, false);
      if (!rc) rc = launch_ns<EPI_NS_UPDATE, NS_BN, 2>(p3, st, PK_GEMM_UPDATE, pair);
    } else {
      rc = launch_ns<EPI_NS_GRAM>(p1, st, PK_GEMM_GRAM, false);
      if (!rc) rc = launch_ns<EPI_NS_POLY>(p2, st, PK_GEMM_POLY, false);
      if (!rc) rc = launch_ns<EPI_NS_UPDATE>(p3, st, PK_GEMM_UPDATE, pair);
    }
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

size_t muon_carve(const lsr_muon_group* groups, int ngroups, uint8_t* ws, std::vector<NsGroup>* out,
                  Control* ctl_out = nullptr) {
  Carver cv{ws};
  long long total = 0;
  for (int i = 0; i < ngroups; ++i) total += std::max(groups[i].count, 1);
  const Control ctl = carve_control(cv, ngroups, total);
  std::vector<NsGroup> gs;
  for (int i = 0; i < ngroups; ++i) {
    const MuonShape s = muon_shape(groups[i]);
    NsGroup G;
    carve_group(cv, G, std::max(groups[i].count, 1), s.m, s.n, src_tiles(s.R, s.C));
    gs.push_back(G);
  }
  bind_control(ctl, gs.data(), ngroups, total);
  for (int i = 0; i < ngroups; ++i) gs[i].batch = groups[i].count;
  if (out) *out = gs;
  if (ctl_out) *ctl_out = ctl;
  return cv.used + 256;
}

// Momentum + orientation + normalisation + NS for all groups; results land in
// G.final_out when set, else in G.X[steps & 1].
// phase bit 1: momentum / orientation / normalisation into the workspace;
// phase bit 2: Newton–Schulz iterations from the workspace into the outputs.
int muon_orthogonalize(const lsr_muon_group* groups, int ngroups, std::vector<NsGroup>& gs, const Control& ctl,
                       float mu, int nesterov, int steps, float a, float b, float c, float eps, cudaStream_t st,
                       int phase = 3) {
  std::vector<NsGroup> live;
  std::vector<ProSource> srcs;
  for (int i = 0; i < ngroups; ++i) {
    const lsr_muon_group& g = groups[i];
    if (g.count == 0) continue;
    if ((phase & 1) && (!g.grad_ptrs || !g.mom_ptrs)) return LSR_ERR_ARG;
    const MuonShape s = muon_shape(g);
    live.push_back(gs[i]);
    srcs.push_back(ProSource{MatRef{g.grad_ptrs, nullptr, 0}, MatRef{g.mom_ptrs, nullptr, 0}, s.R, s.C, s.trans});
  }
  if (phase & 1) {
    int rc = run_prologue(live.data(), srcs.data(), (int)live.size(), ctl, true, mu, nesterov, eps, st);
    if (rc) return rc;
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
    apply_kernel<<<dim3(cdiv(s.R, TILE) * cdiv(s.C, TILE), g.count), EW_THREADS, 0, st>>>(
        pr, s.R, s.C, s.trans, upd[i], upd_bs[i], upd_ld[i], wd_factor, wd != 0.f, -g.lr);
    if (launch_ok()) return LSR_ERR_LAUNCH;
  }
  return LSR_OK;
}

}  // namespace

// Newton–Schulz over a scratch region that is already sized
// (lsr_ns_workspace_bytes) and 256-byte aligned: the caller's workspace for
// lsr_ns_bf16, the library's fixed array for lsr_ns_bf16_noalloc (noalloc.cu).
// It makes no host or device allocation of its own.
int ns_bf16_fixed_scratch(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a,
                          float b, float c, float eps, uint8_t* scratch, cudaStream_t st) {
  const bool trans = orient && rows > cols;
  const int m = trans ? cols : rows, n = trans ? rows : cols;
  Carver cv{scratch};
  const Control ctl = carve_control(cv, 1, batch);
  NsGroup G;
  carve_group(cv, G, batch, m, n, src_tiles(rows, cols));
  bind_control(ctl, &G, 1, batch);
  G.final_out = out;
  G.final_trans = trans;
  G.final_ld = trans ? m : n;
  G.final_bs = (long long)rows * cols;
  const ProSource src{MatRef{nullptr, in, (long long)rows * cols}, MatRef{nullptr, nullptr, 0}, rows, cols,
                      (int)trans};
  int rc = run_prologue(&G, &src, 1, ctl, false, 0.f, 0, eps, st);
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
  carve_control(cv, 1, std::max(batch, 1));
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
  uint8_t* base = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  return ns_bf16_fixed_scratch(in, out, batch, rows, cols, orient, steps, a, b, c, eps, base,
                               reinterpret_cast<cudaStream_t>(stream));
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
  Control ctl;
  muon_carve(groups, ngroups, reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256)), &gs, &ctl);
  rc = muon_orthogonalize(groups, ngroups, gs, ctl, momentum, nesterov, ns_steps, a, b, c, eps, st);
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
  Control ctl;
  muon_carve(groups, ngroups, reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256)), &gs, &ctl);
  for (int i = 0; i < ngroups; ++i) {
    gs[i].final_out = updates[i];
    gs[i].final_ld = gs[i].n;
    gs[i].final_bs = (long long)gs[i].m * gs[i].n;
    gs[i].final_trans = 0;
  }
  return muon_orthogonalize(groups, ngroups, gs, ctl, momentum, nesterov, ns_steps, a, b, c, eps, st, phase);
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
