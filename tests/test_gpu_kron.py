"""GPU parity of the Kronecker sum / apply kernels through the Python surface and C ABI.

Tolerances (relative Frobenius): bf16 operands within 1e-3 of an fp32/fp64
product of the SAME bf16-rounded operands (fp32 accumulation, fp32 output);
fp32 operands (3xTF32) within 1e-5 of the float64 oracle.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kron as ok
from oracle.bf16 import rel_fro

pytestmark = pytest.mark.gpu
TOL_BF16, TOL_F32 = 1e-3, 1e-5
GOLD = Path(__file__).parent / "golden" / "kron_golden.npz"


def _sym(n, g, dev="cuda"):
    M = torch.randn(n, n, generator=g, device=dev) / (n ** 0.5)
    return ((M + M.T) / 2).contiguous()


@pytest.mark.parametrize("shape", [(4, 1024, 1024), (3, 200, 136), (2, 64, 8), (1, 256, 512)])
def test_kron_sum_bf16_and_f32(shape):
    import lsr.kron as K
    batch, m, n = shape
    g = torch.Generator(device="cuda").manual_seed(m + n)
    A, B = _sym(m, g), _sym(n, g)
    X = torch.randn(batch, m, n, generator=g, device="cuda")
    # fp32 (3xTF32)
    Y = K.kron_sum(A, X, B)
    ref = ok.kron_sum(X.cpu().numpy(), A.cpu().numpy(), B.cpu().numpy())
    assert rel_fro(Y.cpu().numpy(), ref) < TOL_F32
    # bf16 operands, compared with the exact product of the same rounded operands
    Ab, Xb, Bb = A.bfloat16(), X.bfloat16(), B.bfloat16()
    Yb = K.kron_sum(Ab, Xb, Bb)
    refb = ok.kron_sum(Xb.float().cpu().numpy(), Ab.float().cpu().numpy(), Bb.float().cpu().numpy())
    assert rel_fro(Yb.cpu().numpy(), refb) < TOL_BF16


def test_kron_sum_1024_64rhs_workload():
    """The Kronecker-sum workload as specified: A, B = (M + M^T)/2 with M ~ N(0, 1/1024), 1024^2,
    drawn A then B from seed 1; X = 64 right-hand sides of 1024^2, N(0, 1), seed 2 (CPU
    generators, the inputs bench.py times). fp32 (3xTF32) within 1e-5 of the float64 oracle;
    bf16 within 1e-3 of the exact product of the same bf16-rounded operands."""
    import lsr.kron as K
    g = torch.Generator().manual_seed(1)
    Ms = [torch.randn(1024, 1024, generator=g) / 32.0 for _ in range(2)]
    A, B = [((m + m.T) / 2).contiguous() for m in Ms]
    X = torch.randn(64, 1024, 1024, generator=torch.Generator().manual_seed(2))
    Ad, Bd, Xd = A.cuda(), B.cuda(), X.cuda()
    errs = {}
    Y = K.kron_sum(Ad, Xd, Bd).cpu().numpy()
    errs["fp32"] = rel_fro(Y, ok.kron_sum(X.numpy(), A.numpy(), B.numpy()))
    del Y
    Ab, Xb, Bb = Ad.bfloat16(), Xd.bfloat16(), Bd.bfloat16()
    Yb = K.kron_sum(Ab, Xb, Bb).cpu().numpy()
    errs["bf16"] = rel_fro(Yb, ok.kron_sum(Xb.float().cpu().numpy(), Ab.float().cpu().numpy(),
                                           Bb.float().cpu().numpy()))
    print(f"Kronecker sum 1024^2 x 64 RHS: fp32 {errs['fp32']:.2e}, bf16 {errs['bf16']:.2e}")
    assert errs["fp32"] < TOL_F32 and errs["bf16"] < TOL_BF16, errs


def test_kron_sum_matches_dense_operator():
    """(A ⊕ B) vec(X) against the explicitly formed A⊗I + I⊗B on a small case."""
    import lsr.kron as K
    g = torch.Generator(device="cuda").manual_seed(5)
    m, n = 16, 24
    A, B = _sym(m, g), _sym(n, g)
    X = torch.randn(3, m, n, generator=g, device="cuda")
    W = ok.dense_operator(np.stack([A.cpu().numpy(), np.eye(m)]), np.stack([np.eye(n), B.cpu().numpy()]))
    ref = (X.cpu().numpy().reshape(3, -1).astype(np.float64) @ W.T).reshape(3, m, n)
    assert rel_fro(K.kron_sum(A, X, B).cpu().numpy(), ref) < TOL_F32


@pytest.mark.parametrize("shape,S", [((3, 128, 320), 1), ((2, 320, 128), 2), ((5, 64, 8), 4), ((2, 96, 96), 3)])
def test_kron_apply(shape, S):
    import lsr.kron as K
    batch, m, n = shape
    g = torch.Generator(device="cuda").manual_seed(S * 100 + m)
    A = torch.randn(S, m, m, generator=g, device="cuda") / m ** 0.5
    B = torch.randn(S, n, n, generator=g, device="cuda") / n ** 0.5
    X = torch.randn(batch, m, n, generator=g, device="cuda")
    ref = ok.kron_apply(X.cpu().numpy(), A.cpu().numpy(), B.cpu().numpy())
    assert rel_fro(K.kron_apply(X, A, B).cpu().numpy(), ref) < TOL_F32
    Ab, Xb, Bb = A.bfloat16(), X.bfloat16(), B.bfloat16()
    refb = ok.kron_apply(Xb.float().cpu().numpy(), Ab.float().cpu().numpy(), Bb.float().cpu().numpy())
    assert rel_fro(K.kron_apply(Xb, Ab, Bb).cpu().numpy(), refb) < TOL_BF16


def test_golden_reference_outputs():
    """Outputs of the reference's kron_apply_shared_2d / S-term sums (tests/golden/kron_golden.npz)."""
    import lsr.kron as K
    z = np.load(GOLD)
    cu = lambda k: torch.from_numpy(z[k]).cuda()  # noqa: E731
    for i in range(3):
        Y = K.kron_apply_shared_2d(cu(f"apply{i}_X"), cu(f"apply{i}_A"), cu(f"apply{i}_B"))
        assert rel_fro(Y.cpu().numpy(), z[f"apply{i}_Y"]) < TOL_F32
    for i in range(2):
        Y = K.kron_sum(cu(f"ksum{i}_A"), cu(f"ksum{i}_X"), cu(f"ksum{i}_B"))
        assert rel_fro(Y.cpu().numpy(), z[f"ksum{i}_Y"]) < TOL_F32
    for S in (1, 2, 4):
        x, A, b = cu(f"multi{S}_X"), cu(f"multi{S}_A"), cu(f"multi{S}_B")
        out = torch.empty_like(x)
        K.kron_sum_out(x, A.transpose(1, 2).contiguous(), b, out)
        assert rel_fro(out.cpu().numpy(), z[f"multi{S}_Y"]) < TOL_F32
        assert rel_fro(out.cpu().numpy(), z[f"multi{S}_Ydense"]) < TOL_F32


def test_kron_sum_out_errors():
    import lsr.kron as K
    x = torch.zeros(4, 64, 8, device="cuda")
    at = torch.zeros(2, 64, 64, device="cuda")
    b = torch.zeros(2, 8, 8, device="cuda")
    with pytest.raises(RuntimeError, match="must be float32"):
        K.kron_sum_out(x.double(), at, b, torch.zeros_like(x))
    with pytest.raises(RuntimeError, match="b must have shape"):
        K.kron_sum_out(x, at, torch.zeros(3, 8, 8, device="cuda"), torch.zeros_like(x))
    with pytest.raises(RuntimeError, match="out must match"):
        K.kron_sum_out(x, at, b, torch.zeros(4, 64, 4, device="cuda"))
    with pytest.raises(RuntimeError, match="must be CUDA"):
        K.kron_sum_out(x.cpu(), at, b, torch.zeros_like(x))


def test_native_reconstruct_matches_reference_golden():
    """W = Σ_s F0⊗...⊗F_{K-1} on the reference's K = 5 / 4 / 3 factor sets (kron_cuda.py)."""
    import lsr.kron as K_
    z = np.load(Path(__file__).parent / "golden" / "kronrec_golden.npz")
    for S in (1, 7, 64):
        outs = {}
        for K in (5, 4, 3):
            fs = [torch.from_numpy(z[f"S{S}_K{K}_f{i}"]).cuda() for i in range(K)]
            outs[K] = K_.native_reconstruct(fs, K, torch.empty(16, 768, device="cuda"))
            assert rel_fro(outs[K].cpu().numpy(), z[f"S{S}_K{K}_W"]) < TOL_F32
        # exact-merge identity of the three representations (kron_cuda.py:748-770)
        assert rel_fro(outs[3].cpu().numpy(), outs[5].cpu().numpy()) < TOL_F32
        assert rel_fro(outs[4].cpu().numpy(), outs[5].cpu().numpy()) < TOL_F32


def test_native_reconstruct_general_shapes():
    import lsr.kron as K_
    g = torch.Generator(device="cuda").manual_seed(9)
    fs = [torch.randn(300, r, c, generator=g, device="cuda") * 0.5 for r, c in [(3, 2), (1, 5), (4, 4), (2, 3)]]
    W = K_.native_reconstruct(fs, 4)
    ref = ok.reconstruct([f.cpu().numpy() for f in fs])
    assert W.shape == ref.shape == (24, 120)
    assert rel_fro(W.cpu().numpy(), ref) < TOL_F32


def test_kron_small_path_matches_fp64():
    """Small fp32 problems run as one FFMA launch (no workspace): the reference's 64 x 8 shape at the
    sweep sizes where that launch is chosen, ragged batches (not a multiple of the 16 right-hand sides per block), row counts
    that are not a multiple of 16, every supported n, A given transposed (kron_sum_out's `at`) or
    not (kron_apply), S from 1 to 8."""
    import lsr.kron as K
    from lsr import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(31)
    cases = [(256, 64, 8, 1), (256, 64, 8, 8), (1024, 64, 8, 4), (4096, 64, 8, 1), (1, 64, 8, 3),
             (300, 64, 8, 4), (17, 48, 4, 3), (100, 20, 16, 2), (129, 64, 1, 2), (5, 64, 2, 8), (33, 7, 8, 5)]
    for M, m, n, S in cases:
        assert lib.lsr_kron_apply_workspace_bytes(M, m, n, S, 1) == 0, (M, m, n, S)  # the small path
        x = torch.randn(M, m, n, device="cuda", generator=g)
        A = torch.randn(S, m, m, device="cuda", generator=g) / m ** 0.5
        b = torch.randn(S, n, n, device="cuda", generator=g) / n ** 0.5
        ref = torch.einsum("sik,mkl,sjl->mij", A.double(), x.double(), b.double()).cpu().numpy()
        out = torch.full_like(x, float("nan"))
        K.kron_sum_out(x, A.transpose(1, 2).contiguous(), b, out)
        assert rel_fro(out.cpu().numpy(), ref) < TOL_F32, (M, m, n, S)
        Y = K.kron_apply(x, A, b)
        assert rel_fro(Y.cpu().numpy(), ref) < TOL_F32, (M, m, n, S)


def test_kron_sum_out_dense_operator_follows_factor_updates():
    """Small factors with many right-hand sides run through a cached dense operator
    W = sum_s A_s (x) B_s: an in-place change of the factors (a new version of the tensor) must be
    seen by the next call."""
    import lsr.kron as K
    from lsr import _lib
    assert _lib.load().lsr_kron_apply_workspace_bytes(20000, 64, 8, 4, 1) > 0  # not the small path
    g = torch.Generator(device="cuda").manual_seed(77)
    x = torch.randn(20000, 64, 8, device="cuda", generator=g)
    at = torch.randn(4, 64, 64, device="cuda", generator=g) / 8
    b = torch.randn(4, 8, 8, device="cuda", generator=g) / 3
    out = torch.empty_like(x)
    for _ in range(2):
        K.kron_sum_out(x, at, b, out)
        ref = torch.einsum("ski,mkl,sjl->mij", at.double(), x.double(), b.double())
        assert rel_fro(out.cpu().numpy(), ref.cpu().numpy()) < TOL_F32
        at.mul_(-0.5)
        b.add_(0.1)
