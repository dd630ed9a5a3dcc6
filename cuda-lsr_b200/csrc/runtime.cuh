// Host-side runtime helpers shared by the liblsr translation units.
#pragma once

#include <algorithm>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm_sm100.cuh"

namespace lsr {

// Status word of the current device (device pointer), or nullptr on failure.
int* status_ptr();
// Two zeroed tile counters of the GEMM engine's dynamic scheduler for one
// launch on the current device (nullptr on failure).
unsigned int* sched_slot();
// Number of SMs of the current device.
int device_sm_count();
// LSR_OK if the current device is sm_100 (B200 class).
int check_device();

// Encode a 3-D bf16 tensor map over [batch][outer][inner] with row stride
// `ld` and batch stride `bstride` (elements), 128-byte swizzle, the given box.
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t batch, uint64_t ld, uint64_t bstride, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// Launch accounting / optional per-launch timing. Kinds group the library's
// kernels for the profile read-out (lsr_profile_read).
enum ProfKind : int {
  PK_GEMM_GRAM = 0,     // NS phase 1: A = X X^T
  PK_GEMM_POLY = 1,     // NS phase 2: B = bA + cA^2
  PK_GEMM_UPDATE = 2,   // NS phase 3: X = aX + BX
  PK_EW_ORIENT = 3,     // momentum / orientation / sum of squares
  PK_EW_NORMALIZE = 4,  // norm finalize + scale
  PK_EW_APPLY = 5,      // parameter update
  PK_GEMM_OTHER = 6,    // plain GEMM / Gram / Kronecker / SOAP
  PK_EW_OTHER = 7,      // other elementwise
  PK_PEER_PUSH = 8,     // parameter shards stored into the peers' replicas
  PK_COUNT = 9
};
void count_launch();
// Records a CUDA event on `st` before (begin) and after (end) a launch when
// profiling is enabled; no-ops otherwise.
void prof_begin(int kind, cudaStream_t st);
void prof_end(int kind, cudaStream_t st);

struct ProfScope {
  int kind;
  cudaStream_t st;
  ProfScope(int k, cudaStream_t s) : kind(k), st(s) {
    count_launch();
    prof_begin(kind, st);
  }
  ~ProfScope() { prof_end(kind, st); }
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// A GEMM operand as stored in memory: `batch` matrices of rows x cols
// (row-major, row stride ld, batch stride bs, in elements). For operand A
// (M x K) K-major means stored [M][K]; MN-major means stored [K][M]. Likewise
// for operand B (N x K).
struct Operand {
  const void* base;
  int rows, cols, ld;
  long long bs;
  int batch;
  int mn;
  int f32 = 0;  // fp32 storage read as tf32 (else bf16)
};

// [batch][K rows][nchunks][chunk] view of a row-major MN-major operand whose row length is a
// whole number of 128-byte chunks: one TMA box then carries all of a tile's chunks.
int encode_tmap_mn_chunks(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                          uint64_t chunk, uint64_t krows, uint64_t nchunks, uint64_t batch, uint64_t ld,
                          uint64_t bstride, uint32_t box_chunks, uint32_t box_krows);
// [batch][K blocks][rows][block] view of a K-major operand whose K length is a
// whole number of 128-byte blocks: one TMA box carries two K blocks of a tile.
int encode_tmap_k_blocks(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                         uint64_t block, uint64_t rows, uint64_t nblocks, uint64_t batch, uint64_t ld,
                         uint64_t bstride, uint32_t box_rows, uint32_t box_blocks);

// Tensor map for operand A (is_b = false, box rows BM) or B (box rows BN):
// K-major box = one 128-byte K row x rows; MN-major box = 128 bytes of MN x one K
// block, or, when the MN length is a whole number of 128-byte chunks, all of the
// tile's MN chunks in one 4-D box (one TMA operation instead of one per chunk).
// *mode receives the operand's load mode for SegDesc::a_mn / b_mn:
// 0 K-major, 1 MN-major chunk boxes, 2 MN-major single 4-D box.
// ks = 2 (two K blocks per pipeline stage): K-major operands need a K length of
// whole blocks, MN-major ones whole MN chunks; both become single 4-D boxes
// (LSR_ERR_SHAPE otherwise, and the caller keeps ks = 1).
inline int make_operand_map(CUtensorMap* map, const Operand& o, bool is_b, int BN, int* mode = nullptr, int ks = 1) {
  const uint32_t ke = o.f32 ? BK_TF32 : BK;
  const CUtensorMapDataType dt = o.f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int esz = o.f32 ? 4 : 2;
  const uint64_t bs = (uint64_t)std::max<long long>(o.bs, (long long)o.rows * o.ld);
  const int box_rows = is_b ? BN : BM;
  if (ks == 2) {
    if (o.f32 || o.cols % (int)ke) return LSR_ERR_SHAPE;
    if (mode) *mode = o.mn ? 2 : 0;
    if (!o.mn)
      return encode_tmap_k_blocks(map, dt, esz, o.base, ke, (uint64_t)o.rows, (uint64_t)(o.cols / ke),
                                  (uint64_t)std::max(o.batch, 1), (uint64_t)o.ld, bs, (uint32_t)box_rows, 2u);
    if (box_rows % (int)ke) return LSR_ERR_SHAPE;
    return encode_tmap_mn_chunks(map, dt, esz, o.base, ke, (uint64_t)o.rows, (uint64_t)(o.cols / ke),
                                 (uint64_t)std::max(o.batch, 1), (uint64_t)o.ld, bs, (uint32_t)(box_rows / ke), 2 * ke);
  }
  if (o.mn && o.cols % (int)ke == 0 && box_rows % (int)ke == 0 &&
      encode_tmap_mn_chunks(map, dt, esz, o.base, ke, (uint64_t)o.rows, (uint64_t)(o.cols / ke),
                            (uint64_t)std::max(o.batch, 1), (uint64_t)o.ld, bs, (uint32_t)(box_rows / ke),
                            ke) == LSR_OK) {
    if (mode) *mode = 2;
    return LSR_OK;
  }
  if (mode) *mode = o.mn ? 1 : 0;
  const uint32_t box_outer = o.mn ? ke : static_cast<uint32_t>(box_rows);
  return encode_tmap_3d(map, dt, esz, o.base, (uint64_t)o.cols, (uint64_t)o.rows, (uint64_t)std::max(o.batch, 1),
                        (uint64_t)o.ld, bs, ke, box_outer);
}

// Fill tile counts and the flat tile numbering of every group (tiles of TM x BN).
template <int BN, int TM = BM>
inline void finalize_tiles(GemmParams& p) {
  int t = 0;
  for (int g = 0; g < p.ngroups; ++g) {
    GroupDesc& G = p.g[g];
    G.tiles_m = cdiv(G.M, TM);
    G.tiles_n = cdiv(G.N, BN);
    if (!G.tri) {
      G.tiles_per_mat = G.tiles_m * G.tiles_n;
    } else {
      int c = 0;
      for (int ti = 0; ti < G.tiles_m; ++ti) c += std::max(0, G.tiles_n - tri_first_col_tile<BN, TM>(ti));
      G.tiles_per_mat = c;
    }
    G.tile_begin = t;
    t += G.tiles_per_mat * G.batch;
  }
  p.total_tiles = t;
}

// Set up the TMA-staged epilogue of group g when its output (and aux operand)
// satisfy the TMA alignment rules; otherwise the group keeps the direct-store
// epilogue.
template <int EPI>
inline void setup_out_map(GemmParams& p, int g) {
  using T = EpiT<EPI>;
  GroupDesc& G = p.g[g];
  G.tma_out = 0;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (EPI == EPI_SOAP_ADAM) {  // coalesced staged path without TMA: 16-byte m / v, 8-byte u vectors
    G.tma_out = (G.N % 4 == 0) && (G.ldo % 4 == 0) && (G.out_bs % 4 == 0) && a16(G.st_m) && a16(G.st_v) &&
                ((reinterpret_cast<uintptr_t>(G.out) & 7) == 0) &&
                ((reinterpret_cast<uintptr_t>(G.out2) & 7) == 0);
    return;
  }
  if (!G.out || !a16(G.out) || (G.ldo * T::ESZ) % 16 || (G.out_bs * T::ESZ) % 16 || G.N % T::EPV) return;
  if (T::AUX && (!G.aux || !a16(G.aux) || (G.ld_aux * T::ESZ) % 16 || (G.aux_bs * T::ESZ) % 16)) return;
  const int rows = G.out_trans ? G.N : G.M;
  const int cols = G.out_trans ? G.M : G.N;
  const long long bs = std::max<long long>(G.out_bs, (long long)rows * G.ldo);
  const int rc = encode_tmap_3d(&p.mapOut[g], T::F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                T::ESZ, G.out, (uint64_t)cols, (uint64_t)rows, (uint64_t)std::max(G.batch, 1),
                                (uint64_t)G.ldo, (uint64_t)bs, 32u, 32u,
                                T::F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc != LSR_OK) return;
  if constexpr (T::SPLIT) {
    if (!G.out2 || !a16(G.out2)) return;
    const int rc2 = encode_tmap_3d(&p.mapOut2[g], T::F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                   T::ESZ, G.out2, (uint64_t)cols, (uint64_t)rows, (uint64_t)std::max(G.batch, 1),
                                   (uint64_t)G.ldo, (uint64_t)bs, 32u, 32u,
                                   T::F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc2 != LSR_OK) return;
  }
  G.tma_out = 1;
}

// Launch the engine. PAIR = 1 launches clusters of two CTAs (256-row tiles;
// the caller builds operand-B tensor maps with BN / 2-row boxes).
template <int BN, int EPI, int STAGES = default_stages<EPI>(), int TF32 = 0, int DUAL = 0, int PAIR = 0, int KS = 1>
inline int launch_gemm(GemmParams& p, cudaStream_t st, int kind = PK_GEMM_OTHER) {
  using L = GemmSmem<BN, STAGES, EPI, PAIR, KS>;
  static_assert(L::TOTAL <= 232448, "shared memory budget exceeded");
  constexpr int TM = PAIR ? 2 * BM : BM;
  finalize_tiles<BN, TM>(p);
  if (p.total_tiles == 0) return LSR_OK;
  for (int g = 0; g < p.ngroups; ++g) {
    setup_out_map<EPI>(p, g);
    const GroupDesc& G = p.g[g];
    // a transposed aux read exists only in the staged bf16 epilogue
    if (G.aux_trans && (!G.tma_out || EpiT<EPI>::F32)) return LSR_ERR_SHAPE;
    // MN-major operands are loaded as whole chunks of one 128-byte row of MN elements
    constexpr int KE = TF32 ? BK_TF32 : BK;
    for (int sg = 0; sg < G.nseg; ++sg) {
      if (G.seg[sg].b_mn && ((PAIR ? BN / 2 : BN) % KE)) return LSR_ERR_SHAPE;
      // two-block stages load MN-major operands as single 4-D boxes only
      if (KS == 2 && (G.seg[sg].a_mn == 1 || G.seg[sg].b_mn == 1)) return LSR_ERR_SHAPE;
    }
  }
  p.status = status_ptr();
  p.sched = sched_slot();
  if (!p.status || !p.sched) return LSR_ERR_LAUNCH;
  auto kfn = gemm_sm100_kernel<BN, STAGES, EPI, TF32, DUAL, PAIR, KS>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) != cudaSuccess)
    return LSR_ERR_LAUNCH;
  ProfScope prof(kind, st);
  if constexpr (PAIR) {
    const int clusters = std::min(device_sm_count() / 2, p.total_tiles);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(gemm_threads<EPI>());
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kfn, p) != cudaSuccess) return LSR_ERR_LAUNCH;
  } else {
    const int grid = std::min(device_sm_count(), p.total_tiles);
    kfn<<<grid, gemm_threads<EPI>(), L::TOTAL, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

// One Kronecker-apply term with bf16 operands, Y (+)= A X B^T over a batch
// (kron.cu); Th/Tl: bf16 scratch for the hi/lo intermediate, batch*m*n each.
int kron_term_bf16(const void* A, int a_trans, const void* X, const void* B, float* Y, void* Th, void* Tl, int batch,
                   int m, int n, int accumulate, cudaStream_t st, int fac_batched);

}  // namespace lsr
