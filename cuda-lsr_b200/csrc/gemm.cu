// Plain batched GEMM and symmetric Gram update entry points over the tcgen05
// engine (gemm_sm100.cuh).
#include "runtime.cuh"

namespace lsr {
namespace {
constexpr int G_BN = 256;
}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

int lsr_gemm_bf16(const void* A, const void* B, void* D, int batch, int M, int N, int K, int a_trans, int b_trans,
                  int out_f32, float alpha, lsr_stream_t stream) {
  if (batch < 0 || M <= 0 || N <= 0 || K <= 0 || batch > 65535) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!A || !B || !D) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  Operand oa = a_trans ? Operand{A, K, M, M, (long long)K * M, batch, 1} : Operand{A, M, K, K, (long long)M * K, batch, 0};
  Operand ob = b_trans ? Operand{B, N, K, K, (long long)N * K, batch, 0} : Operand{B, K, N, N, (long long)K * N, batch, 1};
  // Problems taller than one 128-row tile run on CTA pairs (256-row tiles, half of B per CTA).
  const bool pair = M > BM;
  GroupDesc& G = p.g[0];
  G.seg[0] = SegDesc{cdiv(K, BK), oa.mn, ob.mn, 0, 0};
  rc = make_operand_map(&p.mapA[0][0], oa, false, G_BN, &G.seg[0].a_mn);
  if (!rc) rc = make_operand_map(&p.mapB[0][0], ob, true, pair ? G_BN / 2 : G_BN, &G.seg[0].b_mn);
  if (rc) return rc;
  G.batch = batch;
  G.M = M;
  G.N = N;
  G.nseg = 1;
  G.out = D;
  G.out_bs = (long long)M * N;
  G.ldo = N;
  G.alpha = alpha;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pair)
    return out_f32 ? launch_gemm<G_BN, EPI_STORE_F32, default_stages<EPI_STORE_F32, 1>(), 0, 0, 1>(p, st)
                   : launch_gemm<G_BN, EPI_STORE_BF16, default_stages<EPI_STORE_BF16, 1>(), 0, 0, 1>(p, st);
  return out_f32 ? launch_gemm<G_BN, EPI_STORE_F32>(p, st) : launch_gemm<G_BN, EPI_STORE_BF16>(p, st);
}

int lsr_gram_update_f32(const void* Gm, void* S, int batch, int rows, int cols, int side, float beta, float alpha,
                        lsr_stream_t stream) {
  if (batch < 0 || rows <= 0 || cols <= 0 || batch > 65535 || (side != 0 && side != 1)) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!Gm || !S) return LSR_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  GemmParams p{};
  p.ngroups = 1;
  const int n = side == 0 ? rows : cols;  // statistic is n x n
  // side 0: G G^T (operands are rows of G, K-major); side 1: G^T G (columns of G, MN-major)
  Operand o = side == 0 ? Operand{Gm, rows, cols, cols, (long long)rows * cols, batch, 0}
                        : Operand{Gm, rows, cols, cols, (long long)rows * cols, batch, 1};
  const bool pair = n > BM;
  GroupDesc& G = p.g[0];
  G.seg[0] = SegDesc{cdiv(side == 0 ? cols : rows, BK), o.mn, o.mn, 0, 0};
  rc = make_operand_map(&p.mapA[0][0], o, false, G_BN, &G.seg[0].a_mn);
  if (!rc) rc = make_operand_map(&p.mapB[0][0], o, true, pair ? G_BN / 2 : G_BN, &G.seg[0].b_mn);
  if (rc) return rc;
  G.batch = batch;
  G.M = G.N = n;
  G.tri = 1;
  G.nseg = 1;
  G.out = S;
  G.out_bs = (long long)n * n;
  G.ldo = n;
  G.aux = S;  // the old statistic, read by the EMA epilogue
  G.aux_bs = (long long)n * n;
  G.ld_aux = n;
  G.alpha = alpha;
  G.beta = beta;
  if (pair)
    return launch_gemm<G_BN, EPI_F32_EMA, default_stages<EPI_F32_EMA, 1>(), 0, 0, 1>(
        p, reinterpret_cast<cudaStream_t>(stream));
  return launch_gemm<G_BN, EPI_F32_EMA>(p, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
