// Shampoo / SOAP preconditioner math on the tcgen05 engine, for stacks of
// equally shaped parameter blocks (blocks of at most max_preconditioner_dim
// on each side, as DistributedShampoo blocks its parameters).
//
//   statistics  L = b2 L + (1-b2) G G^T,  R = b2 R + (1-b2) G^T G   (fp32, triangle + mirror)
//   Shampoo     P = L^{-1/4} G R^{-1/4}                              (precomputed inverse roots)
//   SOAP        G' = Q_L^T G Q_R ; Adam on G' (m, v in the rotated basis, fused
//               into the epilogue of the second rotation GEMM) ; U = Q_L U' Q_R^T
//
// The reference gets this math from the third-party distributed_shampoo package
// (DistributedShampoo built in shampoo_soap_lm_ddp_zero1.py:312-400, stepped at
// :609); its in-repo pieces are kron_apply_shared_2d (hft.py:108-140) for the
// two-sided product and coupled_newton_one (shampoo.py:277-347) for the roots.
//
// Operands are bf16 with fp32 accumulation. Each two-sided product is two
// chained GEMMs, the cheaper association first. Shampoo keeps its intermediate
// as a bf16 hi + lo pair (fp32-level apply); the SOAP chain rounds its
// intermediates and the Adam direction to bf16 like every other operand.
#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int S_BN = 256;
typedef __nv_bfloat16 bf16;

size_t a256(size_t x) { return align_up(x, 256); }

Operand bmat(const void* base, int rows, int cols, int batch, int mn) {
  return Operand{base, rows, cols, cols, (long long)rows * cols, batch, mn};
}

int set_pairs(GemmParams& p, const Operand (*pairs)[2], int nseg, int kblocks) {
  int rc = 0;
  for (int t = 0; t < nseg && !rc; ++t) {
    rc = make_operand_map(&p.mapA[0][t], pairs[t][0], false, S_BN);
    if (!rc) rc = make_operand_map(&p.mapB[0][t], pairs[t][1], true, S_BN);
    p.g[0].seg[t] = SegDesc{kblocks, pairs[t][0].mn, pairs[t][1].mn, 0, 0, 0};
  }
  p.g[0].nseg = nseg;
  return rc;
}

void out_desc(GroupDesc& G, int batch, int r, int c, void* out, void* out2) {
  G.batch = batch;
  G.M = r;
  G.N = c;
  G.out = out;
  G.out2 = out2;
  G.out_bs = (long long)r * c;
  G.ldo = c;
  G.alpha = 1.f;
}

bool dims_ok(int batch, int r, int c) { return batch >= 0 && batch <= 65535 && r > 0 && c > 0; }

// Statistics update of both sides (skipped when beta2 is negative).
int stats_update(const void* G, float* L, float* R, int batch, int r, int c, float beta2, lsr_stream_t stream) {
  int rc = lsr_gram_update_f32(G, L, batch, r, c, 0, beta2, 1.f - beta2, stream);
  if (!rc) rc = lsr_gram_update_f32(G, R, batch, r, c, 1, beta2, 1.f - beta2, stream);
  return rc;
}

__global__ void blocks_gather_kernel(const uint64_t* ptrs, const int* lds, int rows, int cols, bf16* stack) {
  const int b = blockIdx.y;
  const bf16* src = reinterpret_cast<const bf16*>(ptrs[b]);
  const int ld = lds[b];
  bf16* dst = stack + (long long)b * rows * cols;
  const long long n = (long long)rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    dst[i] = src[(long long)r * ld + c];
  }
}

// p = bf16(p * (1 - lr*wd)); p = bf16(p - lr * U)  on each block (decoupled weight decay)
__global__ void blocks_apply_kernel(const uint64_t* ptrs, const int* lds, int rows, int cols, const float* U,
                                    float wd_factor, int apply_wd, float neg_lr) {
  const int b = blockIdx.y;
  bf16* dst = reinterpret_cast<bf16*>(ptrs[b]);
  const int ld = lds[b];
  const float* u = U + (long long)b * rows * cols;
  const long long n = (long long)rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    bf16* q = dst + (long long)r * ld + c;
    float pv = __bfloat162float(*q);
    if (apply_wd) pv = bf16r(pv * wd_factor);
    *q = __float2bfloat16_rn(fmaf(neg_lr, u[i], pv));
  }
}

}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

size_t lsr_soap_workspace_bytes(int batch, int rows, int cols) {
  if (!dims_ok(batch, rows, cols)) return 0;
  return 2 * a256((size_t)std::max(batch, 1) * rows * cols * 2) + 256;  // bf16 intermediate + direction
}

int lsr_soap_direction_bf16(const void* G, float* L, float* R, const void* QL, const void* QR, float* m, float* v,
                            float* U, int batch, int rows, int cols, float beta1, float beta2, float eps, int step,
                            int update_stats, void* ws, size_t ws_bytes, lsr_stream_t stream) {
  if (!dims_ok(batch, rows, cols) || step < 1) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!G || !QL || !QR || !m || !v || !U || (update_stats && (!L || !R))) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_soap_workspace_bytes(batch, rows, cols)) return LSR_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int r = rows, c = cols, B = batch;
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  void* P1 = w;                                   // bf16 intermediate of each two-sided product
  void* Ud = w + a256((size_t)B * r * c * 2);     // bf16 Adam direction in the rotated basis
  if (update_stats) {
    rc = stats_update(G, L, R, B, r, c, beta2, stream);
    if (rc) return rc;
  }
  // Every GEMM operand is bf16 (the intermediates included), accumulation fp32;
  // each two-sided product runs the cheaper association first.
  const bool right_first = c > r;
  // ---- G' = Q_L^T G Q_R, Adam fused into the second GEMM's epilogue
  {
    GemmParams p{};
    p.ngroups = 1;
    out_desc(p.g[0], B, r, c, P1, nullptr);
    if (right_first) {  // S = G Q_R : (i,k) = G[i][k], (j,k) = Q_R[k][j]
      const Operand pr[1][2] = {{bmat(G, r, c, B, 0), bmat(QR, c, c, B, 1)}};
      rc = set_pairs(p, pr, 1, cdiv(c, BK));
    } else {  // T = Q_L^T G : (i,k) = Q_L[k][i], (j,k) = G[k][j]
      const Operand pr[1][2] = {{bmat(QL, r, r, B, 1), bmat(G, r, c, B, 1)}};
      rc = set_pairs(p, pr, 1, cdiv(r, BK));
    }
    if (!rc) rc = launch_gemm<S_BN, EPI_STORE_BF16>(p, st);
    if (rc) return rc;
  }
  {
    GemmParams p{};
    p.ngroups = 1;
    GroupDesc& Gd = p.g[0];
    out_desc(Gd, B, r, c, Ud, nullptr);
    Gd.st_m = m;
    Gd.st_v = v;
    Gd.b1 = beta1;
    Gd.b2 = beta2;
    Gd.c1 = (float)(1.0 / (1.0 - std::pow((double)beta1, step)));
    Gd.c2 = (float)(1.0 / (1.0 - std::pow((double)beta2, step)));
    Gd.eps = eps;
    if (right_first) {  // G' = Q_L^T S : (i,k) = Q_L[k][i], (j,k) = S[k][j]
      const Operand pr[1][2] = {{bmat(QL, r, r, B, 1), bmat(P1, r, c, B, 1)}};
      rc = set_pairs(p, pr, 1, cdiv(r, BK));
    } else {  // G' = T Q_R : (i,k) = T[i][k], (j,k) = Q_R[k][j]
      const Operand pr[1][2] = {{bmat(P1, r, c, B, 0), bmat(QR, c, c, B, 1)}};
      rc = set_pairs(p, pr, 1, cdiv(c, BK));
    }
    if (!rc) rc = launch_gemm<S_BN, EPI_SOAP_ADAM>(p, st);
    if (rc) return rc;
  }
  // ---- U = Q_L U' Q_R^T
  {
    GemmParams p{};
    p.ngroups = 1;
    out_desc(p.g[0], B, r, c, P1, nullptr);
    if (right_first) {  // V = U' Q_R^T : (i,k) = U'[i][k], (j,k) = Q_R[j][k]
      const Operand pr[1][2] = {{bmat(Ud, r, c, B, 0), bmat(QR, c, c, B, 0)}};
      rc = set_pairs(p, pr, 1, cdiv(c, BK));
    } else {  // T = Q_L U' : (i,k) = Q_L[i][k], (j,k) = U'[k][j]
      const Operand pr[1][2] = {{bmat(QL, r, r, B, 0), bmat(Ud, r, c, B, 1)}};
      rc = set_pairs(p, pr, 1, cdiv(r, BK));
    }
    if (!rc) rc = launch_gemm<S_BN, EPI_STORE_BF16>(p, st);
    if (rc) return rc;
  }
  GemmParams p{};
  p.ngroups = 1;
  out_desc(p.g[0], B, r, c, U, nullptr);
  if (right_first) {  // U = Q_L V : (i,k) = Q_L[i][k], (j,k) = V[k][j]
    const Operand pr[1][2] = {{bmat(QL, r, r, B, 0), bmat(P1, r, c, B, 1)}};
    rc = set_pairs(p, pr, 1, cdiv(r, BK));
  } else {  // U = T Q_R^T : (i,k) = T[i][k], (j,k) = Q_R[j][k]
    const Operand pr[1][2] = {{bmat(P1, r, c, B, 0), bmat(QR, c, c, B, 0)}};
    rc = set_pairs(p, pr, 1, cdiv(c, BK));
  }
  return rc ? rc : launch_gemm<S_BN, EPI_STORE_F32>(p, st);
}

size_t lsr_shampoo_workspace_bytes(int batch, int rows, int cols) {
  if (!dims_ok(batch, rows, cols)) return 0;
  return 2 * a256((size_t)std::max(batch, 1) * rows * cols * 2) + 256;
}

int lsr_shampoo_direction_bf16(const void* G, float* L, float* R, const void* Lroot, const void* Rroot, float* P,
                               int batch, int rows, int cols, float beta2, int update_stats, void* ws,
                               size_t ws_bytes, lsr_stream_t stream) {
  if (!dims_ok(batch, rows, cols)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!G || !Lroot || !Rroot || !P || (update_stats && (!L || !R))) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (!ws || ws_bytes < lsr_shampoo_workspace_bytes(batch, rows, cols)) return LSR_ERR_WORKSPACE;
  if (update_stats) {
    rc = stats_update(G, L, R, batch, rows, cols, beta2, stream);
    if (rc) return rc;
  }
  uint8_t* w = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 256));
  const size_t h = a256((size_t)batch * rows * cols * 2);
  // P = Lroot G Rroot^T (the roots are symmetric), one factor pair per block
  return kron_term_bf16(Lroot, 0, G, Rroot, P, w, w + h, batch, rows, cols, 0, reinterpret_cast<cudaStream_t>(stream),
                        1);
}

int lsr_blocks_gather_bf16(const uint64_t* ptrs, const int* lds, int nblocks, int rows, int cols, void* stack,
                           lsr_stream_t stream) {
  if (nblocks < 0 || nblocks > 65535 || rows <= 0 || cols <= 0) return LSR_ERR_ARG;
  if (nblocks == 0) return LSR_OK;
  if (!ptrs || !lds || !stack) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)std::min<long long>(((long long)rows * cols + 255) / 256, 1024);
  ProfScope prof(PK_EW_OTHER, st);
  blocks_gather_kernel<<<dim3(blocks, nblocks), 256, 0, st>>>(ptrs, lds, rows, cols, reinterpret_cast<bf16*>(stack));
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

int lsr_blocks_apply_bf16(const uint64_t* ptrs, const int* lds, int nblocks, int rows, int cols, const float* U,
                          float lr, float weight_decay, lsr_stream_t stream) {
  if (nblocks < 0 || nblocks > 65535 || rows <= 0 || cols <= 0) return LSR_ERR_ARG;
  if (nblocks == 0) return LSR_OK;
  if (!ptrs || !lds || !U) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)std::min<long long>(((long long)rows * cols + 255) / 256, 1024);
  const float wd_factor = (float)(1.0 - (double)lr * (double)weight_decay);
  ProfScope prof(PK_EW_APPLY, st);
  blocks_apply_kernel<<<dim3(blocks, nblocks), 256, 0, st>>>(ptrs, lds, rows, cols, U, wd_factor,
                                                             weight_decay != 0.f, -lr);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

}  // extern "C"
