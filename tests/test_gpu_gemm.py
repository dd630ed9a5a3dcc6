"""GPU parity of the tcgen05 GEMM engine through the C ABI (lsr_gemm_bf16,
lsr_gram_update_f32) against fp32 torch products of the same bf16 operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from lsr import _lib
    return _lib


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def _gemm(A, B, batch, M, N, K, a_trans, b_trans, out_f32, alpha=1.0):
    L = _lib()
    D = torch.empty(batch, M, N, device="cuda", dtype=torch.float32 if out_f32 else torch.bfloat16)
    rc = L.load().lsr_gemm_bf16(A.data_ptr(), B.data_ptr(), D.data_ptr(), batch, M, N, K, a_trans, b_trans, out_f32,
                                alpha, L.stream_handle())
    L.check(rc, "lsr_gemm_bf16")
    return D


@pytest.mark.parametrize("a_trans", [0, 1])
@pytest.mark.parametrize("b_trans", [0, 1])
@pytest.mark.parametrize("shape", [(2, 256, 512, 320), (1, 200, 264, 136), (3, 128, 256, 64), (1, 8, 8, 8)])
def test_gemm_majorness(a_trans, b_trans, shape):
    batch, M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + 100 * a_trans + 10 * b_trans)
    A = torch.randn(batch, K, M, device="cuda", generator=g).bfloat16() if a_trans else \
        torch.randn(batch, M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(batch, N, K, device="cuda", generator=g).bfloat16() if b_trans else \
        torch.randn(batch, K, N, device="cuda", generator=g).bfloat16()
    Af = A.float().transpose(1, 2) if a_trans else A.float()
    Bf = B.float().transpose(1, 2) if b_trans else B.float()
    ref = torch.bmm(Af, Bf)
    D32 = _gemm(A, B, batch, M, N, K, a_trans, b_trans, 1, 1.0)
    assert _rel(D32, ref) < 1e-5
    D16 = _gemm(A, B, batch, M, N, K, a_trans, b_trans, 0, 0.5)
    assert _rel(D16, 0.5 * ref) < 4e-3
    assert _lib().device_status() == 0


@pytest.mark.parametrize("side", [0, 1])
@pytest.mark.parametrize("shape", [(2, 320, 512), (1, 1600, 640), (1, 200, 136)])
def test_gram_update(side, shape):
    batch, rows, cols = shape
    g = torch.Generator(device="cuda").manual_seed(rows + cols + side)
    G = torch.randn(batch, rows, cols, device="cuda", generator=g).bfloat16()
    n = rows if side == 0 else cols
    S0 = torch.randn(batch, n, n, device="cuda", generator=g)
    S0 = S0 + S0.transpose(1, 2)
    S = S0.clone()
    L = _lib()
    rc = L.load().lsr_gram_update_f32(G.data_ptr(), S.data_ptr(), batch, rows, cols, side, 0.95, 0.05,
                                      L.stream_handle())
    L.check(rc, "lsr_gram_update_f32")
    Gf = G.float()
    prod = torch.bmm(Gf, Gf.transpose(1, 2)) if side == 0 else torch.bmm(Gf.transpose(1, 2), Gf)
    ref = 0.95 * S0 + 0.05 * prod
    assert _rel(S, ref) < 1e-5
    assert torch.equal(S, S.transpose(1, 2))
    # beta = 0 ignores the old contents (even NaN)
    S.fill_(float("nan"))
    rc = L.load().lsr_gram_update_f32(G.data_ptr(), S.data_ptr(), batch, rows, cols, side, 0.0, 1.0,
                                      L.stream_handle())
    L.check(rc, "lsr_gram_update_f32")
    assert _rel(S, prod) < 1e-5
    assert L.device_status() == 0


def test_gemm_rejects_unaligned_rows():
    L = _lib()
    A = torch.zeros(1, 16, 12, device="cuda", dtype=torch.bfloat16)  # K = 12: 24-byte rows
    B = torch.zeros(1, 16, 12, device="cuda", dtype=torch.bfloat16)
    D = torch.zeros(1, 16, 16, device="cuda")
    rc = L.load().lsr_gemm_bf16(A.data_ptr(), B.data_ptr(), D.data_ptr(), 1, 16, 16, 12, 0, 1, 1, 1.0,
                                L.stream_handle())
    assert rc == -2
