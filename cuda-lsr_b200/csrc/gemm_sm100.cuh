// Persistent, warp-specialised tcgen05 GEMM engine for sm_100a.
//
//   D[g][b] (tile of BM x BN) = sum over segments s of  opA_s[b] * opB_s[b]^T
//
// * one CTA per SM (persistent); tiles of a flat list that spans up to
//   kMaxGroups independent problem groups (e.g. the four parameter shapes of a
//   model, each a batch of equally shaped matrices) are claimed dynamically
//   from a global counter by the producer, which passes each tile index to the
//   MMA and epilogue warps through a small shared-memory ring; CTAs that start
//   late (their SM busy with another kernel) simply claim fewer tiles;
// * warp 0   : TMA producer (one elected thread), STAGES-deep smem ring;
// * warp 1   : owns TMEM (512 columns = two BN-wide fp32 accumulators) and one
//              thread issues tcgen05.mma (M=128, N=BN, K=16) per 16-wide K step;
// * warps 2-5: epilogue; each warp drains its 32 TMEM lanes with tcgen05.ld
//              while the MMA warp already accumulates the next tile into the
//              other accumulator.
// * operands are bf16 (or tf32) in 128-byte-swizzled smem tiles, either K-major
//   (TMA box 64 x rows) or MN-major (TMA boxes 64 x 64); a segment list lets one
//   accumulator sum two products (A*X + X*B^T for the Kronecker sum).
// * triangle mode computes only tiles touching the upper triangle of a
//   symmetric square output and mirrors each element into the lower triangle.
//
// No cluster multicast is used anywhere: every CTA loads its own tiles.
#pragma once

#include "lsr_common.cuh"

namespace lsr {

constexpr int kMaxGroups = 4;
constexpr int kMaxSeg = 6;
constexpr int BM = 128;
constexpr int BK = 64;       // bf16 elements in one 128-byte swizzle row (one K block)
constexpr int BK_TF32 = 32;  // fp32 (tf32) elements in one 128-byte swizzle row
constexpr int kTileRing = 8;  // tile indices in flight between the producer and the consumers

// Epilogue modes.
enum : int {
  EPI_STORE_BF16 = 0,  // out = bf16(alpha * acc)
  EPI_STORE_F32 = 1,   // out = alpha * acc
  EPI_NS_GRAM = 2,     // out = bf16(acc)                                  (symmetric)
  EPI_NS_POLY = 3,     // out = bf16(bf16(alpha*aux) + bf16(beta*bf16(acc))) (symmetric)
  EPI_NS_UPDATE = 4,   // out = bf16(bf16(alpha*aux) + bf16(acc))
  EPI_F32_EMA = 5,     // out = beta * out + alpha * acc                     (fp32)
  EPI_SPLIT_BF16X2 = 6,  // out = bf16(acc), out2 = bf16(acc - bf16(acc))   (hi/lo bf16 pair)
  EPI_SPLIT_TF32 = 7,    // out = tf32(acc), out2 = acc - tf32(acc)        (hi/lo fp32 pair)
  EPI_SOAP_ADAM = 8,     // Adam in the rotated basis on g = acc, fp32 moments st_m / st_v:
                         //   m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g^2
                         //   u = (m * c1) / (sqrt(v * c2) + eps) -> out = bf16(u),
                         //   out2 = bf16(u - bf16(u)) when out2 is set (hi/lo bf16 pair)
};

// Round an fp32 value to tf32 (10 explicit mantissa bits, nearest, ties away
// from zero); x - tf32_hi(x) is then exact in fp32.
__host__ __device__ __forceinline__ float tf32_hi(float x) {
#ifdef __CUDA_ARCH__
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
#else
  uint32_t u;
  memcpy(&u, &x, 4);
  u = (u + 0x1000u) & 0xFFFFE000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
#endif
}

struct SegDesc {
  int kblocks;   // number of K blocks (64 bf16 / 32 tf32 elements each)
  int a_mn;      // operand A stored MN-major (rows of A are columns in memory): 1 = one TMA box per
                 // 64-element MN chunk, 2 = all chunks of the tile in one 4-D box; 0 = K-major
  int b_mn;      // operand B likewise
  int a_bcast;   // operand A is shared by the whole batch (TMA z = 0)
  int b_bcast;
  int slot;      // dual-accumulator kernels: 0 = main products, 1 = small correction products
};

struct GroupDesc {
  int batch, M, N;
  int tiles_m, tiles_n, tiles_per_mat, tile_begin;
  int tri;  // symmetric output: upper-triangle tiles only, mirrored stores
  int nseg;
  SegDesc seg[kMaxSeg];
  void* out;
  long long out_bs;  // batch stride in elements
  int ldo;
  int out_trans;  // store element (r, c) at out[c * ldo + r]
  const void* aux;
  long long aux_bs;
  int ld_aux;
  int aux_trans;  // staged epilogues only: tile element (r, c) reads aux[c][r] (the tile is a transposed view)
  float alpha, beta;
  int tma_out;  // epilogue stages 32x32 chunks in smem and stores them with TMA (mapOut)
  void* out2;   // second output of the split epilogues (same layout as out)
  float* st_m;  // EPI_SOAP_ADAM: first / second moments (fp32, same layout as out)
  float* st_v;
  float b1, b2, c1, c2, eps;  // EPI_SOAP_ADAM scalars (c1, c2: bias corrections 1/(1-b^t))
  const int* active;  // optional per-batch-entry flags: tiles of entries whose flag is 0 are skipped
};

struct GemmParams {
  CUtensorMap mapA[kMaxGroups][kMaxSeg];
  CUtensorMap mapB[kMaxGroups][kMaxSeg];
  CUtensorMap mapOut[kMaxGroups];   // output in stored orientation, box 32 x 32
  CUtensorMap mapOut2[kMaxGroups];  // second output of the split epilogues
  GroupDesc g[kMaxGroups];
  int ngroups;
  int total_tiles;
  int* status;
  unsigned int* sched;  // [0]: next tile to claim, [1]: CTAs finished; both back to 0 when the launch ends
  int masked;           // some group has `active` flags
};

// First column tile of tile row ti touching the upper triangle (tiles of TM x BN).
template <int BN, int TM = BM>
__host__ __device__ constexpr int tri_first_col_tile(int ti) {
  return (ti * TM) / BN;
}

// Map a flat tile index to (group, batch entry, tile row, tile column).
template <int BN, int TM = BM>
__device__ __forceinline__ void decode_tile(const GemmParams& p, int t, int& g, int& b, int& ti, int& tj) {
  g = 0;
#pragma unroll 1
  while (g + 1 < p.ngroups && t >= p.g[g + 1].tile_begin) ++g;
  const GroupDesc& G = p.g[g];
  int local = t - G.tile_begin;
  b = local / G.tiles_per_mat;
  int r = local - b * G.tiles_per_mat;
  if (!G.tri) {
    ti = r / G.tiles_n;
    tj = r - ti * G.tiles_n;
  } else {
    ti = 0;
    tj = 0;
#pragma unroll 1
    for (; ti < G.tiles_m; ++ti) {
      const int cnt = max(0, G.tiles_n - tri_first_col_tile<BN, TM>(ti));
      if (r < cnt) {
        tj = tri_first_col_tile<BN, TM>(ti) + r;
        break;
      }
      r -= cnt;
    }
  }
}

// Status codes written when a bounded wait gives up.
enum : int {
  ST_TIMEOUT_PRODUCER = 101,
  ST_TIMEOUT_MMA_FULL = 102,
  ST_TIMEOUT_MMA_TMEM = 103,
  ST_TIMEOUT_EPILOGUE = 104,
  ST_TIMEOUT_TEARDOWN = 105,
  ST_TIMEOUT_TILE_QUEUE = 106,
  ST_TIMEOUT_PROLOGUE = 107,  // Muon prologue: a matrix's norm was not published in time
};

// ---------------------------------------------------------------------------
// Epilogue: one thread owns one output row and 32 consecutive columns.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, bool vec, int ncols, float (&v)[32]) {
  if (vec && ncols >= 32) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = __ldg(s4 + q);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        v[q * 8 + 2 * e] = f.x;
        v[q * 8 + 2 * e + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < ncols) ? __bfloat162float(src[j]) : 0.f;
  }
}

// Store 32 bf16 values of one row; only columns j with lo <= j < ncols are written.
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, bool vec, int lo, int ncols,
                                              const float (&v)[32]) {
  if (vec && lo <= 0 && ncols >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
      d4[q] = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j >= lo && j < ncols) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GroupDesc& G, int b, int row, int col0,
                                               const uint32_t (&r)[32]) {
  if (row >= G.M) return;
  const int ncols = min(32, G.N - col0);
  if (ncols <= 0) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);

  // Triangle mode: the thread writes columns c >= row directly and mirrors c > row.
  const int lo = G.tri ? max(0, row - col0) : 0;
  if (lo >= ncols) return;

  if constexpr (EPI == EPI_SOAP_ADAM) {
    const long long rowoff = (long long)b * G.out_bs + (long long)row * G.ldo + col0;
    float* pm = G.st_m + rowoff;
    float* pv = G.st_v + rowoff;
    __nv_bfloat16* pu = reinterpret_cast<__nv_bfloat16*>(G.out) + rowoff;
    __nv_bfloat16* pl = G.out2 ? reinterpret_cast<__nv_bfloat16*>(G.out2) + rowoff : nullptr;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= ncols) continue;
      const float g = v[j];
      const float mm = fmaf(G.b1, pm[j], (1.f - G.b1) * g);
      const float vv = fmaf(G.b2, pv[j], (1.f - G.b2) * g * g);
      pm[j] = mm;
      pv[j] = vv;
      const float u = (mm * G.c1) / (sqrtf(vv * G.c2) + G.eps);
      const __nv_bfloat16 h = __float2bfloat16_rn(u);
      pu[j] = h;
      if (pl) pl[j] = __float2bfloat16_rn(u - __bfloat162float(h));
    }
    return;
  } else if constexpr (EPI == EPI_SPLIT_BF16X2 || EPI == EPI_SPLIT_TF32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < lo || j >= ncols) continue;
      const long long idx = (long long)b * G.out_bs +
                            (G.out_trans ? (long long)(col0 + j) * G.ldo + row : (long long)row * G.ldo + col0 + j);
      // symmetric output: the mirrored element too
      const bool mir = G.tri && col0 + j > row;
      const long long midx = (long long)b * G.out_bs + (long long)(col0 + j) * G.ldo + row;
      if constexpr (EPI == EPI_SPLIT_TF32) {
        const float h = tf32_hi(v[j]);
        reinterpret_cast<float*>(G.out)[idx] = h;
        reinterpret_cast<float*>(G.out2)[idx] = v[j] - h;
        if (mir) {
          reinterpret_cast<float*>(G.out)[midx] = h;
          reinterpret_cast<float*>(G.out2)[midx] = v[j] - h;
        }
      } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
        const __nv_bfloat16 l = __float2bfloat16_rn(v[j] - __bfloat162float(h));
        reinterpret_cast<__nv_bfloat16*>(G.out)[idx] = h;
        reinterpret_cast<__nv_bfloat16*>(G.out2)[idx] = l;
        if (mir) {
          reinterpret_cast<__nv_bfloat16*>(G.out)[midx] = h;
          reinterpret_cast<__nv_bfloat16*>(G.out2)[midx] = l;
        }
      }
    }
    return;
  } else if constexpr (EPI == EPI_STORE_F32 || EPI == EPI_F32_EMA) {
    float* out = reinterpret_cast<float*>(G.out) + (long long)b * G.out_bs;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < lo || j >= ncols) continue;
      const int c = col0 + j;
      float val = G.alpha * v[j];
      long long idx = G.out_trans ? (long long)c * G.ldo + row : (long long)row * G.ldo + c;
      if constexpr (EPI == EPI_F32_EMA) {
        if (G.beta != 0.f) val = fmaf(G.beta, out[idx], val);
      }
      out[idx] = val;
      if (G.tri && c > row) out[(long long)c * G.ldo + row] = val;
    }
    return;
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(G.out) + (long long)b * G.out_bs;
    if constexpr (EPI == EPI_STORE_BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = G.alpha * v[j];
    } else if constexpr (EPI == EPI_NS_GRAM) {
      // value = bf16(acc): rounding happens in the store
    } else if constexpr (EPI == EPI_NS_POLY || EPI == EPI_NS_UPDATE) {
      const __nv_bfloat16* aux =
          reinterpret_cast<const __nv_bfloat16*>(G.aux) + (long long)b * G.aux_bs + (long long)row * G.ld_aux + col0;
      const bool avec = ((G.ld_aux & 7) == 0) && ((reinterpret_cast<uintptr_t>(aux) & 15) == 0);
      float x[32];
      load_bf16x32(aux, avec, ncols, x);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if constexpr (EPI == EPI_NS_POLY)
          v[j] = bf16r(G.alpha * x[j]) + bf16r(G.beta * bf16r(v[j]));
        else
          v[j] = bf16r(G.alpha * x[j]) + bf16r(v[j]);
      }
    }
    if (!G.out_trans) {
      __nv_bfloat16* dst = out + (long long)row * G.ldo + col0;
      const bool vec = ((G.ldo & 7) == 0) && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
      store_bf16x32(dst, vec, lo, ncols, v);
    } else {
      // transposed store: lanes of a warp hold consecutive rows, so each
      // column j is one coalesced 64-byte segment.
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j >= lo && j < ncols) out[(long long)(col0 + j) * G.ldo + row] = __float2bfloat16_rn(v[j]);
    }
    if (G.tri) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int c = col0 + j;
        if (j < ncols && c > row) out[(long long)c * G.ldo + row] = __float2bfloat16_rn(v[j]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Staged epilogue: each epilogue warp owns 32 rows of the tile and walks the
// tile's 32-column chunks. Per chunk:
//   * the aux operand (A for POLY, X for UPDATE, the old statistic for EMA) is
//     read with coalesced 16-byte loads one chunk ahead, written into a
//     swizzled 32x32 smem staging buffer, and each thread reads back its row;
//   * results go back into the same buffer (own row only) and, for mirrored /
//     transposed outputs, column-wise into a second buffer;
//   * one lane stores the buffer(s) with TMA (OOB rows/cols are clipped).
// Staging rows are 64 B (bf16) or 128 B (fp32), laid out with the TMA 64B /
// 128B swizzle so thread-per-row accesses are conflict-free.
// ---------------------------------------------------------------------------

template <int EPI>
struct EpiT {
  static constexpr bool F32 =
      (EPI == EPI_STORE_F32 || EPI == EPI_F32_EMA || EPI == EPI_SPLIT_TF32 || EPI == EPI_SOAP_ADAM);
  static constexpr bool SPLIT = (EPI == EPI_SPLIT_BF16X2 || EPI == EPI_SPLIT_TF32);
  static constexpr int ESZ = F32 ? 4 : 2;
  static constexpr int ROWB = 32 * ESZ;  // bytes per staged row
  static constexpr int CHB = 32 * ROWB;  // bytes per staged 32x32 chunk
  static constexpr int VPR = ROWB / 16;  // 16-byte vectors per staged row
  static constexpr int EPV = 16 / ESZ;   // elements per 16-byte vector
  static constexpr bool AUX = (EPI == EPI_NS_POLY || EPI == EPI_NS_UPDATE || EPI == EPI_F32_EMA);
};

// Epilogue warps per CTA. The SOAP epilogue (Adam on the rotated gradient) moves
// 20 bytes of moments and output per element and walks its chunks one after
// another; it runs 8 warps, the two warps of each TMEM lane quarter taking
// alternate 32-column chunks. Every other epilogue runs 4.
template <int EPI>
constexpr int epi_warps() {
  return EPI == EPI_SOAP_ADAM ? 8 : 4;
}
template <int EPI>
constexpr int gemm_threads() {
  return 64 + 32 * epi_warps<EPI>();  // producer warp, MMA warp, epilogue warps
}
// Staging chunks per epilogue warp: 2 direct + 2 transposed; the SOAP epilogue
// stages only the accumulator (double-buffered).
template <int EPI>
constexpr int epi_slots() {
  return EPI == EPI_SOAP_ADAM ? 2 : 4;
}

template <int ROWB>
__device__ __forceinline__ uint32_t stg_off(int r, int j) {
  if constexpr (ROWB == 64)
    return (uint32_t)(r * 64 + 16 * (j ^ ((r >> 1) & 3)));
  else
    return (uint32_t)(r * 128 + 16 * (j ^ (r & 7)));
}

// Coalesced load of the aux chunk (32 rows x 32 cols at row0/col0) into
// registers: lane l holds vectors l + 32 i (row = idx / VPR, vector = idx % VPR).
template <int EPI>
__device__ __forceinline__ void aux_prefetch(const GroupDesc& G, int b, int row0, int col0, int lane,
                                             uint4 (&pre)[EpiT<EPI>::VPR]) {
  using T = EpiT<EPI>;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(G.aux) + (long long)b * G.aux_bs * T::ESZ;
  // aux_trans: the 32 x 32 aux block at aux rows col0.., aux columns row0.. (staged as is,
  // read back column-wise)
  const int ar0 = G.aux_trans ? col0 : row0, ac0 = G.aux_trans ? row0 : col0;
  const int arows = G.aux_trans ? G.N : G.M, acols = G.aux_trans ? G.M : G.N;
#pragma unroll
  for (int i = 0; i < T::VPR; ++i) {
    const int idx = lane + 32 * i;
    const int r = idx / T::VPR, j = idx % T::VPR;
    const int gr = ar0 + r, gc = ac0 + j * T::EPV;
    if (gr < arows && gc < acols)
      pre[i] = __ldg(reinterpret_cast<const uint4*>(base + ((long long)gr * G.ld_aux + gc) * T::ESZ));
    else
      pre[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Adam moments of one 32 x 32 chunk for the EPI_SOAP_ADAM epilogue, held in
// registers: lane l owns the 16-byte vectors (row (l / 8) + 4 i, columns 4 (l % 8)
// .. + 3) for i < 8, so m and v move in coalesced 128-byte row segments. They
// are loaded while the chunk's accumulator columns come out of TMEM. Empty for
// the other epilogues.
template <int EPI>
struct MomentChunk {
  __device__ __forceinline__ void load(const GroupDesc&, int, int, int, int) {}
};

template <>
struct MomentChunk<EPI_SOAP_ADAM> {
  float4 m[8], v[8];
  __device__ __forceinline__ void load(const GroupDesc& G, int b, int row0, int col0, int lane) {
    const int jv = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int gr = row0 + (lane >> 3) + 4 * i, gc = col0 + 4 * jv;
      m[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gr < G.M && gc < G.N) {
        const long long idx = (long long)b * G.out_bs + (long long)gr * G.ldo + gc;
        m[i] = __ldcs(reinterpret_cast<const float4*>(G.st_m + idx));
        v[i] = __ldcs(reinterpret_cast<const float4*>(G.st_v + idx));
      }
    }
  }
};

template <int EPI>
__device__ __forceinline__ void epilogue_chunk_staged(const GemmParams& p, int g, const GroupDesc& G, int b,
                                                      int row0, int col0, int lane, const uint32_t (&r)[32],
                                                      const uint4 (&cur)[EpiT<EPI>::VPR], uint8_t* dbuf,
                                                      uint8_t* tbuf, const MomentChunk<EPI>& mom) {
  using T = EpiT<EPI>;
  if constexpr (EPI == EPI_SOAP_ADAM) {
    // Work row-contiguously: 8 lanes per row, 16-byte vectors, so m / v / u move
    // in coalesced segments.
    const int jv = lane & 7;
    __syncwarp();  // the previous chunk's reads of dbuf are done
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(dbuf + stg_off<128>(lane, j)) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = (lane >> 3) + 4 * i;
      const int gr = row0 + rr, gc = col0 + 4 * jv;
      if (gr >= G.M || gc >= G.N) continue;
      const float4 g4 = *reinterpret_cast<const float4*>(dbuf + stg_off<128>(rr, jv));
      const long long idx = (long long)b * G.out_bs + (long long)gr * G.ldo + gc;
      const float4 m4 = mom.m[i];
      const float4 v4 = mom.v[i];
      const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
      float mm[4] = {m4.x, m4.y, m4.z, m4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w}, uu[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mm[e] = fmaf(G.b1, mm[e], (1.f - G.b1) * gg[e]);
        vv[e] = fmaf(G.b2, vv[e], (1.f - G.b2) * gg[e] * gg[e]);
        uu[e] = (mm[e] * G.c1) / (sqrtf(vv[e] * G.c2) + G.eps);
      }
      __stcs(reinterpret_cast<float4*>(G.st_m + idx), make_float4(mm[0], mm[1], mm[2], mm[3]));
      __stcs(reinterpret_cast<float4*>(G.st_v + idx), make_float4(vv[0], vv[1], vv[2], vv[3]));
      uint2 u2;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u2);
      h[0] = __floats2bfloat162_rn(uu[0], uu[1]);
      h[1] = __floats2bfloat162_rn(uu[2], uu[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(G.out) + idx) = u2;
      if (G.out2) {
        // lo part of the pair: what bf16 rounding of u dropped
        const float2 h0 = __bfloat1622float2(h[0]), h1 = __bfloat1622float2(h[1]);
        uint2 l2;
        __nv_bfloat162* l = reinterpret_cast<__nv_bfloat162*>(&l2);
        l[0] = __floats2bfloat162_rn(uu[0] - h0.x, uu[1] - h0.y);
        l[1] = __floats2bfloat162_rn(uu[2] - h1.x, uu[3] - h1.y);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(G.out2) + idx) = l2;
      }
    }
    return;
  }
  // buffers of chunk k-2 must have been read by their TMA store
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if constexpr (T::AUX) {
#pragma unroll
    for (int i = 0; i < T::VPR; ++i) {
      const int idx = lane + 32 * i;
      *reinterpret_cast<uint4*>(dbuf + stg_off<T::ROWB>(idx / T::VPR, idx % T::VPR)) = cur[i];
    }
    __syncwarp();
    float x[32];
    if (!T::F32 && G.aux_trans) {
      // column `lane` of the staged block: element (k, lane) for k < 32 (one row per step:
      // the warp reads 64 contiguous bytes, two lanes per 32-bit word)
#pragma unroll
      for (int k = 0; k < 32; ++k)
        x[k] = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(
            dbuf + stg_off<T::ROWB>(k, (lane * T::ESZ) / 16) + (lane * T::ESZ) % 16));
    } else {
#pragma unroll
      for (int j = 0; j < T::VPR; ++j) {
        const uint4 u = *reinterpret_cast<const uint4*>(dbuf + stg_off<T::ROWB>(lane, j));
        if constexpr (T::F32) {
          x[4 * j] = __uint_as_float(u.x);
          x[4 * j + 1] = __uint_as_float(u.y);
          x[4 * j + 2] = __uint_as_float(u.z);
          x[4 * j + 3] = __uint_as_float(u.w);
        } else {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            x[8 * j + 2 * e] = f.x;
            x[8 * j + 2 * e + 1] = f.y;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if constexpr (EPI == EPI_NS_POLY)
        v[j] = bf16r(G.alpha * x[j]) + bf16r(G.beta * bf16r(v[j]));
      else if constexpr (EPI == EPI_NS_UPDATE)
        v[j] = bf16r(G.alpha * x[j]) + bf16r(v[j]);
      else  // EMA
        v[j] = (G.beta != 0.f) ? fmaf(G.beta, x[j], G.alpha * v[j]) : G.alpha * v[j];
    }
  } else if constexpr (EPI == EPI_STORE_BF16 || EPI == EPI_STORE_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = G.alpha * v[j];
  }
  if constexpr (T::SPLIT) {
    // hi part -> dbuf (mapOut), lo part -> tbuf (mapOut2); transposed when out_trans
    if (G.out_trans) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const uint32_t off = stg_off<T::ROWB>(j, (lane * T::ESZ) / 16) + (lane * T::ESZ) % 16;
        if constexpr (T::F32) {
          const float h = tf32_hi(v[j]);
          *reinterpret_cast<float*>(dbuf + off) = h;
          *reinterpret_cast<float*>(tbuf + off) = v[j] - h;
        } else {
          const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
          *reinterpret_cast<__nv_bfloat16*>(dbuf + off) = h;
          *reinterpret_cast<__nv_bfloat16*>(tbuf + off) = __float2bfloat16_rn(v[j] - __bfloat162float(h));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&p.mapOut[g], dbuf, row0, col0, b);
        tma_store_3d(&p.mapOut2[g], tbuf, row0, col0, b);
        bulk_commit();
      }
      return;
    }
#pragma unroll
    for (int j = 0; j < T::VPR; ++j) {
      uint4 uh, ul;
      if constexpr (T::F32) {
        float h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = tf32_hi(v[4 * j + e]);
          l[e] = v[4 * j + e] - h[e];
        }
        uh = make_uint4(__float_as_uint(h[0]), __float_as_uint(h[1]), __float_as_uint(h[2]), __float_as_uint(h[3]));
        ul = make_uint4(__float_as_uint(l[0]), __float_as_uint(l[1]), __float_as_uint(l[2]), __float_as_uint(l[3]));
      } else {
        __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&uh);
        __nv_bfloat162* ll = reinterpret_cast<__nv_bfloat162*>(&ul);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a0 = v[8 * j + 2 * e], a1 = v[8 * j + 2 * e + 1];
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(a0, a1);
          const float2 hf = __bfloat1622float2(h2);
          hh[e] = h2;
          ll[e] = __floats2bfloat162_rn(a0 - hf.x, a1 - hf.y);
        }
      }
      *reinterpret_cast<uint4*>(dbuf + stg_off<T::ROWB>(lane, j)) = uh;
      *reinterpret_cast<uint4*>(tbuf + stg_off<T::ROWB>(lane, j)) = ul;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(&p.mapOut[g], dbuf, col0, row0, b);
      tma_store_3d(&p.mapOut2[g], tbuf, col0, row0, b);
      bulk_commit();
    }
    if (G.tri && col0 > row0) {
      // symmetric output: the mirrored chunk goes out from the same buffers
      // once the TMA engine has read them
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const uint32_t off = stg_off<T::ROWB>(j, (lane * T::ESZ) / 16) + (lane * T::ESZ) % 16;
        if constexpr (T::F32) {
          const float h = tf32_hi(v[j]);
          *reinterpret_cast<float*>(dbuf + off) = h;
          *reinterpret_cast<float*>(tbuf + off) = v[j] - h;
        } else {
          const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
          *reinterpret_cast<__nv_bfloat16*>(dbuf + off) = h;
          *reinterpret_cast<__nv_bfloat16*>(tbuf + off) = __float2bfloat16_rn(v[j] - __bfloat162float(h));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&p.mapOut[g], dbuf, row0, col0, b);
        tma_store_3d(&p.mapOut2[g], tbuf, row0, col0, b);
        bulk_commit();
      }
    }
    return;
  }
  const bool diag = G.tri && col0 == row0;
  const bool direct = !G.out_trans;
  const bool transposed = G.out_trans || (G.tri && col0 > row0);
  if (direct) {
#pragma unroll
    for (int j = 0; j < T::VPR; ++j) {
      uint4 u;
      if constexpr (T::F32) {
        u = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                       __float_as_uint(v[4 * j + 3]));
      } else {
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
      }
      *reinterpret_cast<uint4*>(dbuf + stg_off<T::ROWB>(lane, j)) = u;
    }
  }
  if (diag) {
    // symmetric diagonal block: overwrite the lower triangle with the mirror of the upper
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j > lane) {
        uint8_t* dst = dbuf + stg_off<T::ROWB>(j, (lane * T::ESZ) / 16) + (lane * T::ESZ) % 16;
        if constexpr (T::F32)
          *reinterpret_cast<float*>(dst) = v[j];
        else
          *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16_rn(v[j]);
      }
    }
  } else if (transposed) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      uint8_t* dst = tbuf + stg_off<T::ROWB>(j, (lane * T::ESZ) / 16) + (lane * T::ESZ) % 16;
      if constexpr (T::F32)
        *reinterpret_cast<float*>(dst) = v[j];
      else
        *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16_rn(v[j]);
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const CUtensorMap* mo = &p.mapOut[g];
    if (direct) tma_store_3d(mo, dbuf, col0, row0, b);
    if (transposed && !diag) tma_store_3d(mo, tbuf, row0, col0, b);
    bulk_commit();
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------

// PAIR = 1: the tile is computed by a cluster of two CTAs; each CTA holds
// 128 rows of A and BN/2 rows of B per stage.
// KS = 2: a stage holds two K blocks (two 128-byte swizzle atoms per K-major
// operand row block, 2 x KE K-rows per MN-major chunk).
template <int BN, int STAGES, int EPI, int PAIR = 0, int KS = 1>
struct GemmSmem {
  static constexpr int A_BYTES = BM * 128 * KS;  // 128-byte K rows, for bf16 and tf32 alike
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * 128 * KS;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int EPI_BYTES = epi_warps<EPI>() * epi_slots<EPI>() * EpiT<EPI>::CHB;
  static constexpr int BAR_OFFSET = EPI_OFFSET + EPI_BYTES;
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5 + 2 * kTileRing) + 16 + 4 * kTileRing;
  static constexpr int TOTAL = BAR_OFFSET + BAR_BYTES + 1024;  // + alignment slack
};

// Pipeline depth that fits next to the epilogue staging buffers (at most 8).
template <int EPI, int PAIR = 0, int BN = 256, int KS = 1>
constexpr int default_stages() {
  using S8 = GemmSmem<BN, 8, EPI, PAIR, KS>;
  int st = 8;
  while (st > 2 && S8::TOTAL - (8 - st) * (S8::STAGE_BYTES + 16) > 232448) --st;
  return st;
}

// TF32 = 0: bf16 operands (kind::f16); TF32 = 1: fp32 operands read as tf32
// (kind::tf32). Both use 128-byte K rows: 64 bf16 or 32 fp32 per K block, four
// UMMAs of K = 16 (bf16) / 8 (tf32) per block.
// DUAL = 1: each tile owns two TMEM accumulators (segment slot 0 and 1) that
// the epilogue adds in fp32; the tensor core's accumulation then never adds
// small correction products into a large running sum (3xTF32 accuracy). One
// tile's accumulators fill TMEM, so tiles are not double-buffered.
// PAIR = 1: launched as clusters of two CTAs. A tile is 256 x BN; CTA rank r
// loads rows [128 r, 128 r + 128) of A and rows [r BN/2, (r+1) BN/2) of B, the
// leader (rank 0) issues tcgen05.mma.cta_group::2 (M = 256) reading both CTAs'
// shared memory, and each CTA's TMEM holds its 128 output rows. The peer's TMA
// loads count on the leader's full barriers; the leader's commits arrive on
// both CTAs' barriers; both epilogues arrive on the leader's accumulator-empty
// barriers. No multicast is used.
// KS = 2: each stage carries two K blocks, loaded with one 4-D TMA box per
// operand (K-major: two 128-byte atoms; MN-major: 2 KE K-rows per chunk), so
// the TMA operations and barrier round trips per flop halve; the MMA thread
// issues 8 UMMAs per stage (4 when the segment's last stage holds one block).
template <int BN, int STAGES, int EPI, int TF32, int DUAL, int PAIR, int KS = 1>
__global__ void __launch_bounds__(gemm_threads<EPI>(), 1) gemm_sm100_kernel(const __grid_constant__ GemmParams p) {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 32 in [64, 256]");
  constexpr int KE = TF32 ? BK_TF32 : BK;        // elements per K block (= MN elements per MN-major chunk)
  constexpr int CHUNK = KE * 128 * KS;           // bytes of one MN-major chunk (KS KE K-rows of 128 B)
  constexpr uint32_t MN_STEP = (TF32 ? 8 : 16) * 128;  // bytes between UMMA K steps, MN-major
  constexpr int ACC_COLS = DUAL ? 2 * BN : BN;          // TMEM columns per tile in flight
  constexpr int TM = PAIR ? 2 * BM : BM;                // output rows per tile
  constexpr int BNC = PAIR ? BN / 2 : BN;               // B rows loaded by this CTA
  static_assert(2 * BN <= 512, "two BN-wide accumulators must fit in TMEM");
  static_assert(BNC % 8 == 0, "B rows per CTA must be whole 8-row swizzle groups");
  // MN-major B needs BNC to be whole MN chunks (KE elements); launch_gemm checks it.
  static_assert(KS == 1 || KS == 2, "a stage holds one or two K blocks");
  static_assert(KS == 1 || !TF32, "two-block stages are bf16 only");
  using L = GemmSmem<BN, STAGES, EPI, PAIR, KS>;
  constexpr int A_HALF = BM * 128;   // bytes of one K block of the A tile (K-major)
  constexpr int B_HALF = (PAIR ? BN / 2 : BN) * 128;
  using ET = EpiT<EPI>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint64_t* tq_full = done_bar + 1;          // tile ring: slot written
  uint64_t* tq_empty = tq_full + kTileRing;  // tile ring: slot read by every consumer (leader's barriers)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tq_empty + kTileRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* tile_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  // Consumers of one tile-ring slot: the MMA thread and the epilogue warps of
  // the leader, plus (pair) the peer's producer and epilogue warps.
  constexpr int EW = epi_warps<EPI>();
  constexpr uint32_t kTileConsumers = (PAIR ? 2u : 1u) * (1u + (uint32_t)EW);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 32 * EW * (PAIR ? 2 : 1));
    }
    mbar_init(done_bar, 1);
    for (int r = 0; r < kTileRing; ++r) {
      mbar_init(tq_full + r, 1);
      mbar_init(tq_empty + r, kTileConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int g = 0; g < p.ngroups; ++g)
      for (int s = 0; s < p.g[g].nseg; ++s) {
        tma_prefetch_desc(&p.mapA[g][s]);
        tma_prefetch_desc(&p.mapB[g][s]);
      }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int r = 0;         // tile-ring slot
      uint32_t rph = 0;  // its phase
      auto claim = [&]() -> int {
        while (true) {
          const int c = (int)atomicAdd(p.sched, 1u);
          if (c >= p.total_tiles) return -1;
          if (!p.masked) return c;
          int g, b, ti, tj;
          decode_tile<BN, TM>(p, c, g, b, ti, tj);
          const int* act = p.g[g].active;
          if (!act || *reinterpret_cast<const volatile int*>(act + b)) return c;
        }
      };
      int t_next = rank == 0 ? claim() : -1;
      while (ok) {
        int t;
        if (rank == 0) {
          // hand the claimed tile (or the end marker -1) to every consumer
          if (!mbar_wait(tq_empty + r, rph ^ 1, abort_flag, p.status, ST_TIMEOUT_TILE_QUEUE)) break;
          t = t_next;
          tile_ring[r] = t;
          if constexpr (PAIR) {
            st_shared_cluster_u32(mapa_shared(smem_u32((const void*)(tile_ring + r)), 1), (uint32_t)t);
            mbar_arrive_cluster(mapa_shared(smem_u32(tq_full + r), 1));
          }
          mbar_arrive(tq_full + r);
          if (t >= 0) t_next = claim();  // in flight while this tile's loads are issued
        } else {
          // pair peer: load the tile the leader claimed
          if (!mbar_wait_acq_cluster(tq_full + r, rph, abort_flag, p.status, ST_TIMEOUT_TILE_QUEUE)) break;
          t = tile_ring[r];
          mbar_arrive_cluster(mapa_shared(smem_u32(tq_empty + r), 0));
        }
        if (++r == kTileRing) {
          r = 0;
          rph ^= 1;
        }
        if (t < 0) break;
        int g, b, ti, tj;
        decode_tile<BN, TM>(p, t, g, b, ti, tj);
        const GroupDesc& G = p.g[g];
        const int m0 = ti * TM + (int)rank * BM, n0 = tj * BN + (int)rank * BNC;
        for (int sg = 0; ok && sg < G.nseg; ++sg) {
          const SegDesc S = G.seg[sg];
          const CUtensorMap* ma = &p.mapA[g][sg];
          const CUtensorMap* mb = &p.mapB[g][sg];
          const int za = S.a_bcast ? 0 : b;
          const int zb = S.b_bcast ? 0 : b;
          for (int kb = 0; kb < S.kblocks; kb += KS) {
            if (!mbar_wait(empty + s, ph ^ 1, abort_flag, p.status, ST_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + s * L::STAGE_BYTES;
            uint8_t* sb = sa + L::A_BYTES;
            const int k0 = kb * KE;
            if constexpr (KS == 2) {
              // one 4-D box per operand: K-major (K element, row, K block, batch) from K block kb,
              // MN-major (MN element, K row, MN chunk, batch) over 2 KE K rows
              if constexpr (PAIR) {
                if (rank == 0) mbar_arrive_expect_tx(full + s, 2 * L::STAGE_BYTES);
                const uint32_t fb = mapa_shared(smem_u32(full + s), 0);
                if (!S.a_mn)
                  tma_load_4d_pair(sa, ma, fb, 0, m0, kb, za);
                else
                  tma_load_4d_pair(sa, ma, fb, 0, k0, m0 / KE, za);
                if (!S.b_mn)
                  tma_load_4d_pair(sb, mb, fb, 0, n0, kb, zb);
                else
                  tma_load_4d_pair(sb, mb, fb, 0, k0, n0 / KE, zb);
              } else {
                mbar_arrive_expect_tx(full + s, L::STAGE_BYTES);
                if (!S.a_mn)
                  tma_load_4d(sa, ma, full + s, 0, m0, kb, za);
                else
                  tma_load_4d(sa, ma, full + s, 0, k0, m0 / KE, za);
                if (!S.b_mn)
                  tma_load_4d(sb, mb, full + s, 0, n0, kb, zb);
                else
                  tma_load_4d(sb, mb, full + s, 0, k0, n0 / KE, zb);
              }
            } else if constexpr (PAIR) {
              // the leader's full barrier counts both CTAs' bytes
              if (rank == 0) mbar_arrive_expect_tx(full + s, 2 * L::STAGE_BYTES);
              const uint32_t fb = mapa_shared(smem_u32(full + s), 0);
              if (!S.a_mn) {
                tma_load_3d_pair(sa, ma, fb, k0, m0, za);
              } else if (S.a_mn == 2) {
                tma_load_4d_pair(sa, ma, fb, 0, k0, m0 / KE, za);
              } else {
#pragma unroll
                for (int c = 0; c < BM / KE; ++c) tma_load_3d_pair(sa + c * CHUNK, ma, fb, m0 + KE * c, k0, za);
              }
              if (!S.b_mn) {
                tma_load_3d_pair(sb, mb, fb, k0, n0, zb);
              } else if (S.b_mn == 2) {
                tma_load_4d_pair(sb, mb, fb, 0, k0, n0 / KE, zb);
              } else {
#pragma unroll
                for (int c = 0; c < BNC / KE; ++c) tma_load_3d_pair(sb + c * CHUNK, mb, fb, n0 + KE * c, k0, zb);
              }
            } else {
              mbar_arrive_expect_tx(full + s, L::STAGE_BYTES);
              if (!S.a_mn) {
                tma_load_3d(sa, ma, full + s, k0, m0, za);
              } else if (S.a_mn == 2) {
                tma_load_4d(sa, ma, full + s, 0, k0, m0 / KE, za);
              } else {
#pragma unroll
                for (int c = 0; c < BM / KE; ++c) tma_load_3d(sa + c * CHUNK, ma, full + s, m0 + KE * c, k0, za);
              }
              if (!S.b_mn) {
                tma_load_3d(sb, mb, full + s, k0, n0, zb);
              } else if (S.b_mn == 2) {
                tma_load_4d(sb, mb, full + s, 0, k0, n0 / KE, zb);
              } else {
#pragma unroll
                for (int c = 0; c < BN / KE; ++c) tma_load_3d(sb + c * CHUNK, mb, full + s, n0 + KE * c, k0, zb);
              }
            }
            if (++s == STAGES) {
              s = 0;
              ph ^= 1;
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair: leader only)
    if (lane == 0 && rank == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      int r = 0;
      uint32_t rph = 0;
      while (ok) {
        if (!mbar_wait(tq_full + r, rph, abort_flag, p.status, ST_TIMEOUT_TILE_QUEUE)) break;
        const int t = tile_ring[r];
        mbar_arrive(tq_empty + r);
        if (++r == kTileRing) {
          r = 0;
          rph ^= 1;
        }
        if (t < 0) break;
        int g, b, ti, tj;
        decode_tile<BN, TM>(p, t, g, b, ti, tj);
        const GroupDesc& G = p.g[g];
        if (!mbar_wait(tempty + acc, aph ^ 1, abort_flag, p.status, ST_TIMEOUT_MMA_TMEM)) break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
        uint32_t acc_flags = 0;  // bit s: slot s already holds a partial sum
        for (int sg = 0; ok && sg < G.nseg; ++sg) {
          const SegDesc S = G.seg[sg];
          const int slot = DUAL ? S.slot : 0;
          const uint32_t d_tmem = d_base + static_cast<uint32_t>(slot * BN);
          uint32_t accumulate = (acc_flags >> slot) & 1u;
          acc_flags |= 1u << slot;
          const uint32_t idesc = make_idesc(TM, BN, TF32 ? 2u : 1u, S.a_mn ? 1u : 0u, S.b_mn ? 1u : 0u);
          // per-UMMA descriptor advance along K, in 16-byte units: 32 B within a
          // K-major row, MN_STEP bytes (UMMA_K rows) for MN-major
          const uint32_t a_step = S.a_mn ? (MN_STEP >> 4) : (32u >> 4);
          const uint32_t b_step = S.b_mn ? (MN_STEP >> 4) : (32u >> 4);
          for (int kb = 0; kb < S.kblocks; kb += KS) {
            if (!mbar_wait(full + s, ph, abort_flag, p.status, ST_TIMEOUT_MMA_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * L::STAGE_BYTES);
            const uint32_t sb = sa + L::A_BYTES;
            const uint64_t adesc = S.a_mn ? smem_desc_sw128(sa, CHUNK, 1024) : smem_desc_sw128(sa, 16, 1024);
            const uint64_t bdesc = S.b_mn ? smem_desc_sw128(sb, CHUNK, 1024) : smem_desc_sw128(sb, 16, 1024);
            // UMMAs in this stage: 4 per K block present (the last stage of an odd K-block count
            // holds one block; its second half is zero-filled and skipped)
            const int nk = (KS == 2 && kb + 1 >= S.kblocks) ? 4 : 4 * KS;
#pragma unroll
            for (int k = 0; k < 4 * KS; ++k) {
              if (k >= nk) break;
              // K-major: the second K block's atom follows the first (A_HALF / B_HALF bytes on);
              // MN-major: K rows continue within each chunk
              const uint32_t a_off = S.a_mn ? (uint32_t)(k * a_step) : (uint32_t)((k >> 2) * (A_HALF >> 4) + (k & 3) * a_step);
              const uint32_t b_off = S.b_mn ? (uint32_t)(k * b_step) : (uint32_t)((k >> 2) * (B_HALF >> 4) + (k & 3) * b_step);
              const uint64_t ad = adesc + (uint64_t)a_off, bd = bdesc + (uint64_t)b_off;
              if constexpr (PAIR) {
                if constexpr (TF32)
                  umma_tf32_pair(d_tmem, ad, bd, idesc, accumulate);
                else
                  umma_bf16_pair(d_tmem, ad, bd, idesc, accumulate);
              } else {
                if constexpr (TF32)
                  umma_tf32(d_tmem, ad, bd, idesc, accumulate);
                else
                  umma_bf16(d_tmem, ad, bd, idesc, accumulate);
              }
              accumulate = 1;
            }
            // frees this smem stage (in both CTAs of a pair) once the MMAs have read it
            if constexpr (PAIR) {
              umma_commit_pair(mapa_shared(smem_u32(empty + s), 0));
              umma_commit_pair(mapa_shared(smem_u32(empty + s), 1));
            } else {
              umma_commit(empty + s);
            }
            if (++s == STAGES) {
              s = 0;
              ph ^= 1;
            }
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue(s)
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(tfull + acc), 0));
          umma_commit_pair(mapa_shared(smem_u32(tfull + acc), 1));
        } else {
          umma_commit(tfull + acc);
        }
        if (DUAL) {
          aph ^= 1;
        } else {
          acc ^= 1;
          if (acc == 0) aph ^= 1;
        }
      }
      // Drain: make sure no MMA is still writing TMEM before it is released.
      if constexpr (PAIR)
        umma_commit_pair(mapa_shared(smem_u32(done_bar), 0));
      else
        umma_commit(done_bar);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(done_bar, 0)) {
        if (globaltimer_ns() - t0 > LSR_WAIT_TIMEOUT_NS) {
          set_status(p.status, ST_TIMEOUT_TEARDOWN);
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // with 8 epilogue warps, warps 2-5 take the even and warps 6-9 the odd chunks
    const uint32_t chunk_mask = EW == 8 ? ((warp - 2) >= 4 ? 0xAAAAAAAAu : 0x55555555u) : 0xFFFFFFFFu;
    uint8_t* ebase = smem + L::EPI_OFFSET + (warp - 2) * epi_slots<EPI>() * ET::CHB;
    int acc = 0;
    uint32_t aph = 0;
    uint32_t kchunk = 0;  // chunks processed by this warp (staging buffer parity)
    int r = 0;
    uint32_t rph = 0;
    while (true) {
      const bool got = (PAIR && rank != 0)
                           ? mbar_wait_acq_cluster(tq_full + r, rph, abort_flag, p.status, ST_TIMEOUT_TILE_QUEUE)
                           : mbar_wait(tq_full + r, rph, abort_flag, p.status, ST_TIMEOUT_TILE_QUEUE);
      if (!got) break;
      const int t = tile_ring[r];
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0)
          mbar_arrive_cluster(mapa_shared(smem_u32(tq_empty + r), 0));
        else
          mbar_arrive(tq_empty + r);
      }
      if (++r == kTileRing) {
        r = 0;
        rph ^= 1;
      }
      if (t < 0) break;
      int g, b, ti, tj;
      decode_tile<BN, TM>(p, t, g, b, ti, tj);
      const GroupDesc& G = p.g[g];
      const int row0 = ti * TM + (int)rank * BM + q * 32;  // first row of this warp
      // warp-uniform mask of live 32-column chunks
      uint32_t live = 0;
      if (row0 < G.M) {
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          const int col0 = tj * BN + cc * 32;
          if (col0 < G.N && !(G.tri && col0 < row0)) live |= 1u << cc;
        }
        live &= chunk_mask;
      }
      uint4 pre[ET::VPR];
#pragma unroll
      for (int i = 0; i < ET::VPR; ++i) pre[i] = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (ET::AUX) {
        if (G.tma_out && live) aux_prefetch<EPI>(G, b, row0, tj * BN + (__ffs(live) - 1) * 32, lane, pre);
      }
      if (!mbar_wait(tfull + acc, aph, abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * ACC_COLS);
      bool second = false;  // dual: does slot 1 hold products for this group?
      if (DUAL) {
        for (int sg = 0; sg < G.nseg; ++sg) second |= (G.seg[sg].slot == 1);
      }
      uint32_t rem = live;
      while (rem) {
        const int cc = __ffs(rem) - 1;
        rem &= rem - 1;
        const int col0 = tj * BN + cc * 32;
        uint32_t r[32];
        tmem_ld32(tbase + static_cast<uint32_t>(cc * 32), r);
        if (DUAL && second) {
          uint32_t r2[32];
          tmem_ld32(tbase + static_cast<uint32_t>(BN + cc * 32), r2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(r2[j]));
        }
        if (G.tma_out) {
          uint4 cur[ET::VPR];
#pragma unroll
          for (int i = 0; i < ET::VPR; ++i) cur[i] = pre[i];
          if constexpr (ET::AUX) {
            if (rem) aux_prefetch<EPI>(G, b, row0, tj * BN + (__ffs(rem) - 1) * 32, lane, pre);
          }
          MomentChunk<EPI> mom;
          mom.load(G, b, row0, col0, lane);  // in flight while the accumulator chunk arrives
          tmem_ld_wait();
          uint8_t* dbuf = ebase + (kchunk & 1) * ET::CHB;
          uint8_t* tbuf = ebase + (2 + (kchunk & 1)) * ET::CHB;
          epilogue_chunk_staged<EPI>(p, g, G, b, row0, col0, lane, r, cur, dbuf, tbuf, mom);
          ++kchunk;
        } else {
          tmem_ld_wait();
          epilogue_chunk<EPI>(G, b, row0 + lane, col0, r);
        }
      }
      tc_fence_before();
      if constexpr (PAIR)
        mbar_arrive_cluster(mapa_shared(smem_u32(tempty + acc), 0));  // the leader's MMA waits on it
      else
        mbar_arrive(tempty + acc);
      if (DUAL) {
        aph ^= 1;
      } else {
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // Pair: neither CTA releases TMEM or exits while the other may still read its
  // shared memory (leader MMAs) or arrive on its barriers (peer epilogue).
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, 512);
    else
      tmem_dealloc(tmem_base, 512);
  }
  // The last CTA to finish returns the tile counter to zero for the next
  // launch that uses this slot (every claim of this launch precedes it).
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(p.sched + 1, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(p.sched, 0u);
      atomicExch(p.sched + 1, 0u);
    }
  }
}

}  // namespace lsr
