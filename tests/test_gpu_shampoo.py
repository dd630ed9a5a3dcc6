"""GPU: Shampoo / SOAP preconditioner kernels against the float64 oracle.

Parity is unpinned upstream (distributed_shampoo is third-party and absent);
the oracle restates the workload's formulas. Only the kernels' inputs (G,
Q_L, Q_R, the inverse roots) are rounded to bf16 before the oracle sees them;
the oracle then computes in float64, as the reference's fp32 path computes
every intermediate in fp32. Tolerance: 1e-3 relative Frobenius (the bf16
bound of the path).
"""
import numpy as np
import pytest
import torch

from oracle import shampoo as osh
from oracle.bf16 import rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _orth(n, g, batch):
    Q = torch.linalg.qr(torch.randn(batch, n, n, generator=g, dtype=torch.float64))[0]
    return Q.to(torch.bfloat16)


@pytest.mark.parametrize("shape", [(2, 256, 1024), (2, 512, 256), (1, 1600, 640), (2, 200, 136), (3, 96, 72)])
def test_soap_direction(shape):
    from lsr.shampoo import soap_direction
    n, r, c = shape
    g = torch.Generator().manual_seed(r + c)
    G = (torch.randn(n, r, c, generator=g) * 0.01).bfloat16()
    QL, QR = _orth(r, g, n), _orth(c, g, n)
    m0 = torch.randn(n, r, c, generator=g) * 1e-3
    v0 = torch.rand(n, r, c, generator=g) * 1e-4 + 1e-5
    L0 = torch.zeros(n, r, r)
    R0 = torch.zeros(n, c, c)
    dev = lambda t: t.cuda().contiguous()  # noqa: E731
    L, R, m, v = dev(L0), dev(R0), dev(m0), dev(v0)
    U = soap_direction(dev(G), L, R, dev(QL), dev(QR), m, v, 0.95, 0.95, 1e-8, step=5, update_stats=True)
    Gn = G.float().numpy()
    Lr, Rr = osh.stats_update(L0.numpy(), R0.numpy(), Gn, 0.95)
    Ur, mr, vr = osh.soap_direction(Gn, QL.float().numpy(), QR.float().numpy(), m0.numpy(), v0.numpy(),
                                    0.95, 0.95, 1e-8, 5)
    assert rel_fro(L.cpu().numpy(), Lr) < 1e-5
    assert rel_fro(R.cpu().numpy(), Rr) < 1e-5
    assert rel_fro(m.cpu().numpy(), mr) < TOL
    assert rel_fro(v.cpu().numpy(), vr) < TOL
    assert rel_fro(U.cpu().numpy(), Ur) < TOL


def test_soap_config3_two_steps():
    """The SOAP step on the 1600 x 6400 GPT-2-XL MLP weight: G ~ N(0, 0.01^2) from seed 3,
    eigenbases from QR of N(0, 1), betas (0.95, 0.95), eps 1e-8. Step 1 starts from zero
    moments; step 2 takes a second gradient (seed 4). Moments and statistics are checked against
    the float64 oracle on the same bf16 inputs at both steps, and so is the direction.

    At step 1 from zero moments the rotated Adam direction is m / (|m| + eps'), i.e. the sign of
    the rotated gradient: where that is within rounding of zero, any fp32 evaluation (the
    reference's included) can return the opposite sign from float64. Those few elements (where
    |m| is below 1e-3 of its RMS) are compared against the oracle's rotation of the kernel's own
    sign there; every other element must match."""
    from lsr.shampoo import soap_direction
    r, c = 1600, 6400
    b1 = b2 = 0.95
    g = torch.Generator().manual_seed(3)
    G1 = (torch.randn(1, r, c, generator=g) * 0.01).bfloat16()
    G2 = (torch.randn(1, r, c, generator=torch.Generator().manual_seed(4)) * 0.01).bfloat16()
    gq = torch.Generator().manual_seed(11)
    QL = torch.linalg.qr(torch.randn(1, r, r, generator=gq, dtype=torch.float64).cuda())[0].bfloat16().contiguous()
    QR = torch.linalg.qr(torch.randn(1, c, c, generator=gq, dtype=torch.float64).cuda())[0].bfloat16().contiguous()
    L = torch.zeros(1, r, r, device="cuda")
    R = torch.zeros(1, c, c, device="cuda")
    m = torch.zeros(1, r, c, device="cuda")
    v = torch.zeros(1, r, c, device="cuda")
    qln, qrn = QL.float().cpu().numpy(), QR.float().cpu().numpy()
    mr, vr = np.zeros((1, r, c)), np.zeros((1, r, c))
    Lr, Rr = np.zeros((1, r, r)), np.zeros((1, c, c))
    for t, Gt in ((1, G1), (2, G2)):
        U = soap_direction(Gt.cuda(), L, R, QL, QR, m, v, b1, b2, 1e-8, step=t, update_stats=True)
        Gn = Gt.float().numpy()
        Lr, Rr = osh.stats_update(Lr, Rr, Gn, 0.95)
        Ur, mr, vr, Upr = osh.soap_direction_parts(Gn, qln, qrn, mr, vr, b1, b2, 1e-8, t)
        mg, vg = m.cpu().numpy(), v.cpu().numpy()
        errs = {"U": rel_fro(U.cpu().numpy(), Ur), "m": rel_fro(mg, mr), "v": rel_fro(vg, vr),
                "L": rel_fro(L.cpu().numpy(), Lr), "R": rel_fro(R.cpu().numpy(), Rr)}
        flips = np.sign(mg) != np.sign(mr)
        nflip = int(flips.sum())
        if t == 1 and nflip:
            rms = np.sqrt(np.mean(mr ** 2))
            assert np.abs(mr[flips]).max() < 1e-3 * rms, "sign differences away from zero"
            assert nflip < 1e-5 * mr.size, nflip
            Up_fixed = Upr.copy()
            Up_fixed[flips] = osh.adam_in_basis(mg, vg, b1, b2, 1e-8, t)[flips]
            errs["U_same_signs"] = rel_fro(U.cpu().numpy(), osh.soap_rotate_back(Up_fixed, qln, qrn))
        print(f"config-3 SOAP step {t}: " + ", ".join(f"{k} {e:.2e}" for k, e in errs.items()) +
              f", sign differences {nflip}")
        assert errs["m"] < TOL and errs["v"] < TOL, (t, errs)
        # statistics: bf16 operands, fp32 accumulation over K = 6400 (L) / 1600 (R) products
        assert errs["L"] < 5e-5 and errs["R"] < 5e-5, (t, errs)
        assert errs["U_same_signs" if (t == 1 and nflip) else "U"] < TOL, (t, errs)
        if t == 2:
            assert errs["U"] < TOL, errs


def test_soap_gpt2xl_layer_every_block_shape():
    """DistributedShampoo (SOAP, max_preconditioner_dim 1024) on one GPT-2-XL layer's four
    matrices, whose 42 blocks cover all 10 block shapes of the 48-layer model. Step 2 (after a
    refresh of the eigenbases from the statistics) is replayed per block in float64 from the
    bases and moments the optimizer holds; directions within 1e-3, statistics within 1e-5."""
    from lsr.shampoo import DefaultSOAPConfig, DistributedShampoo
    shapes = [(1600, 4800), (1600, 1600), (1600, 6400), (6400, 1600)]
    g = torch.Generator().manual_seed(5)
    params = [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().cuda()) for s in shapes]
    opt = DistributedShampoo(params, lr=0.01, betas=(0.95, 0.95), epsilon=1e-8, weight_decay=0.01,
                             max_preconditioner_dim=1024, precondition_frequency=1, start_preconditioning_step=1,
                             preconditioner_config=DefaultSOAPConfig)
    grads = [[(torch.randn(*s, generator=g) * 0.01).bfloat16() for s in shapes] for _ in range(2)]
    for p, gr in zip(params, grads[0]):
        p.grad = gr.cuda()
    opt.step()
    before = {shape: (grp.m.clone(), grp.v.clone(), grp.L.clone(), grp.R.clone())
              for shape, grp, _ in opt._groups}
    for p, gr in zip(params, grads[1]):
        p.grad = gr.cuda()
    opt.step()
    assert len(opt._groups) == 10
    worst = 0.0
    for shape, grp, _ in opt._groups:
        r, c = shape
        m0, v0, L0, R0 = (x.cpu().numpy() for x in before[shape])
        for k, (p, r0, c0) in enumerate(grp.refs):
            i = next(j for j, q in enumerate(params) if q is p)
            Gb = grads[1][i].float().numpy()[r0:r0 + r, c0:c0 + c]
            Lr, Rr = osh.stats_update(L0[k], R0[k], Gb, 0.95)
            assert rel_fro(grp.L[k].cpu().numpy(), Lr) < 1e-5, (shape, k)
            assert rel_fro(grp.R[k].cpu().numpy(), Rr) < 1e-5, (shape, k)
            Ur, mr, vr = osh.soap_direction(Gb, grp.QL[k].float().cpu().numpy(), grp.QR[k].float().cpu().numpy(),
                                            m0[k], v0[k], 0.95, 0.95, 1e-8, 2)
            e = rel_fro(grp.U[k].cpu().numpy(), Ur)
            worst = max(worst, e)
            assert e < TOL, (shape, k, e)
            assert rel_fro(grp.m[k].cpu().numpy(), mr) < TOL, (shape, k)
            assert rel_fro(grp.v[k].cpu().numpy(), vr) < TOL, (shape, k)
    print(f"GPT-2-XL layer, 42 SOAP blocks in 10 shapes: worst direction error {worst:.2e}")


@pytest.mark.parametrize("shape", [(2, 256, 1024), (3, 576, 1024), (1, 1600, 6400)])
def test_shampoo_direction(shape):
    from lsr.shampoo import shampoo_direction
    n, r, c = shape
    g = torch.Generator().manual_seed(7 * r + c)
    G = (torch.randn(n, r, c, generator=g) * 0.01).bfloat16()
    Lroot = [osh.inverse_root(np.cov(np.random.default_rng(i).standard_normal((r, 2 * r))) , 4, 1e-6)
             for i in range(n)]
    Rroot = [osh.inverse_root(np.cov(np.random.default_rng(100 + i).standard_normal((c, 2 * c))), 4, 1e-6)
             for i in range(n)]
    Lb = torch.tensor(np.stack(Lroot), dtype=torch.float32).bfloat16()
    Rb = torch.tensor(np.stack(Rroot), dtype=torch.float32).bfloat16()
    P = shampoo_direction(G.cuda(), Lb.cuda(), Rb.cuda())
    ref = osh.shampoo_precondition(G.float().numpy(), Lb.float().numpy(), Rb.float().numpy())
    assert rel_fro(P.cpu().numpy(), ref) < TOL


def test_distributed_shampoo_soap_plumbing():
    """Blocking, gather, statistics, refresh and apply of the optimizer, replayed in numpy with its own bases."""
    from lsr.shampoo import DefaultSOAPConfig, DistributedShampoo, param_blocks
    g = torch.Generator().manual_seed(3)
    shapes = [(128, 384), (1104, 256), (64, 64)]
    P0 = [(torch.randn(*s, generator=g) * 0.02).bfloat16() for s in shapes]
    params = [torch.nn.Parameter(p.clone().cuda()) for p in P0]
    bias = torch.nn.Parameter(torch.zeros(64, device="cuda"))
    opt = DistributedShampoo(params + [bias], lr=0.01, betas=(0.95, 0.95), epsilon=1e-8, weight_decay=0.01,
                             max_preconditioner_dim=512, precondition_frequency=1, start_preconditioning_step=1,
                             preconditioner_config=DefaultSOAPConfig)
    grads = [(torch.randn(*s, generator=g) * 0.01).bfloat16() for s in shapes]
    for p, gr in zip(params, grads):
        p.grad = gr.cuda()
    bias.grad = torch.randn(64, device="cuda") * 0.01
    opt.step()
    # replay: one SOAP step per block with the bases the optimizer computed
    for (shape, grp, lst) in opt._groups:
        assert grp is not None
        for k, (p, r0, c0) in enumerate(grp.refs):
            i = next(j for j, q in enumerate(params) if q is p)
            r, c = shape
            Gb = grads[i].float().numpy()[r0:r0 + r, c0:c0 + c]
            U, _, _ = osh.soap_direction(Gb, grp.QL[k].float().cpu().numpy(), grp.QR[k].float().cpu().numpy(),
                                         np.zeros((r, c)), np.zeros((r, c)), 0.95, 0.95, 1e-8, 1)
            p_ref = P0[i].float().numpy()[r0:r0 + r, c0:c0 + c] * np.float32(1 - 0.01 * 0.01) - 0.01 * U
            got = params[i].detach().float().cpu().numpy()[r0:r0 + r, c0:c0 + c]
            # parameters are bf16: compare the change
            d_got = got - P0[i].float().numpy()[r0:r0 + r, c0:c0 + c]
            d_ref = p_ref - P0[i].float().numpy()[r0:r0 + r, c0:c0 + c]
            assert rel_fro(d_got, d_ref) < 0.05, (shape, k)
    n_blocks = sum(len(param_blocks(s, 512)) for s in shapes)
    assert sum(len(grp.refs) for _, grp, _ in opt._groups) == n_blocks
    assert torch.isfinite(bias).all() and bias.abs().sum() > 0


def test_shampoo_roots_by_coupled_newton_match_eigh():
    """root_inverse_method="coupled_newton": the inverse 4th roots of L + eps I, R + eps I from the
    batched coupled Newton kernel agree with the eigendecomposition path (bf16-stored roots)."""
    from lsr.shampoo import DistributedShampoo
    g = torch.Generator().manual_seed(8)
    shapes = [(128, 384), (256, 256)]
    P0 = [(torch.randn(*s, generator=g) * 0.02).bfloat16() for s in shapes]
    grads = [(torch.randn(*s, generator=g) * 0.01).bfloat16() for s in shapes]
    roots = {}
    for method in ("eigh", "coupled_newton"):
        params = [torch.nn.Parameter(p.clone().cuda()) for p in P0]
        opt = DistributedShampoo(params, lr=0.01, betas=(0.9, 0.95), epsilon=1e-3, weight_decay=0.0,
                                 max_preconditioner_dim=512, precondition_frequency=1, start_preconditioning_step=1,
                                 root_inverse_method=method)
        for p, gr in zip(params, grads):
            p.grad = gr.cuda()
        opt.step()
        roots[method] = [(grp.QL.float().cpu(), grp.QR.float().cpu()) for _, grp, _ in opt._groups]
    for (le, re), (ln, rn) in zip(roots["eigh"], roots["coupled_newton"]):
        assert rel_fro(ln.numpy(), le.numpy()) < 1e-2
        assert rel_fro(rn.numpy(), re.numpy()) < 1e-2
    with pytest.raises(ValueError):
        DistributedShampoo([torch.nn.Parameter(P0[0].cuda())], root_inverse_method="qr")


def test_refresh_happens_on_the_reference_periodic_steps():
    """start 3, frequency 2: the eigenbases change at steps 4 and 6 only (t >= start and t % freq == 0)."""
    from lsr.shampoo import DefaultSOAPConfig, DistributedShampoo
    g = torch.Generator().manual_seed(21)
    p = torch.nn.Parameter((torch.randn(128, 256, generator=g) * 0.02).bfloat16().cuda())
    opt = DistributedShampoo([p], lr=0.01, betas=(0.95, 0.95), epsilon=1e-8, max_preconditioner_dim=512,
                             precondition_frequency=2, start_preconditioning_step=3,
                             preconditioner_config=DefaultSOAPConfig)
    changed = []
    prev = None
    for t in range(1, 7):
        p.grad = (torch.randn(128, 256, generator=g) * 0.01).bfloat16().cuda()
        opt.step()
        grp = opt._groups[0][1]
        cur = (grp.QL.clone(), grp.QR.clone())
        if prev is not None and not (torch.equal(cur[0], prev[0]) and torch.equal(cur[1], prev[1])):
            changed.append(t)
        prev = cur
    assert changed == [4, 6]


def test_shampoo_grafting_kernels_match_torch_fp32():
    """lsr_shampoo_graft_prepare_bf16 / _scale_f32 against the same formulas in torch fp32 ops."""
    from lsr import _lib as L
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(31)
    n, r, c, t = 3, 576, 704, 4
    b1, gb2, geps = 0.9, 0.95, 1e-8
    G = (torch.randn(n, r, c, device="cuda", generator=g) * 0.01).bfloat16()
    m0 = torch.randn(n, r, c, device="cuda", generator=g) * 1e-3
    v0 = torch.rand(n, r, c, device="cuda", generator=g) * 1e-4
    m, v = m0.clone(), v0.clone()
    tiles = lib.lsr_graft_tiles(r, c)
    adam_sq = torch.empty(n, tiles, device="cuda")
    u_sq = torch.empty(n, tiles, device="cuda")
    Gf = torch.empty(n, r, c, dtype=torch.bfloat16, device="cuda")
    U = torch.empty(n, r, c, device="cuda")
    st = L.stream_handle()
    L.check(lib.lsr_shampoo_graft_prepare_bf16(G.data_ptr(), m.data_ptr(), v.data_ptr(), Gf.data_ptr(), U.data_ptr(),
                                               adam_sq.data_ptr(), n, r, c, b1, gb2, geps, t, st), "prepare")
    Gr = G.float()
    v_ref = gb2 * v0 + (1 - gb2) * Gr * Gr
    m_ref = b1 * m0 + (1 - b1) * Gr
    gf = m_ref / (1 - b1 ** t)
    adam = gf / ((v_ref / (1 - gb2 ** t)).sqrt() + geps)
    assert rel_fro(v.cpu().numpy(), v_ref.cpu().numpy()) < 1e-6
    assert rel_fro(m.cpu().numpy(), m_ref.cpu().numpy()) < 1e-6
    assert rel_fro(U.cpu().numpy(), adam.cpu().numpy()) < 1e-5
    assert rel_fro(Gf.float().cpu().numpy(), gf.bfloat16().float().cpu().numpy()) < 1e-3
    # scale a stand-in Shampoo direction to the Adam norm of each block
    P = torch.randn(n, r, c, device="cuda", generator=g)
    P_ref = P * (adam.flatten(1).norm(dim=1) / P.flatten(1).norm(dim=1))[:, None, None]
    L.check(lib.lsr_shampoo_graft_scale_f32(P.data_ptr(), adam_sq.data_ptr(), u_sq.data_ptr(), n, r, c, st), "scale")
    assert rel_fro(P.cpu().numpy(), P_ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_blocks_apply_any_dtype_and_slots(dtype):
    """lsr_blocks_apply_any: decoupled update of parameter blocks from a gathered buffer in the
    communication dtype, with padding slots skipped through the slot index."""
    from lsr import _lib as L
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(41)
    P = (torch.randn(64, 96, device="cuda", generator=g) * 0.02).bfloat16()
    P0 = P.clone()
    blocks = [(0, 0), (32, 48), (0, 48)]  # 32 x 48 blocks
    recv = torch.randn(5, 32, 48, device="cuda", generator=g).to(dtype)
    slots = torch.tensor([4, 0, 2], dtype=torch.int32, device="cuda")
    ptrs = torch.tensor([P.data_ptr() + 2 * (r0 * 96 + c0) for r0, c0 in blocks], dtype=torch.int64).cuda()
    lds = torch.full((3,), 96, dtype=torch.int32, device="cuda")
    lr, wd = 0.01, 0.1
    L.check(lib.lsr_blocks_apply_any(ptrs.data_ptr(), lds.data_ptr(), 3, 32, 48, recv.data_ptr(),
                                     L.DTYPE_CODES[dtype], slots.data_ptr(), lr, wd, L.stream_handle()), "apply_any")
    ref = P0.double()
    for k, (r0, c0) in enumerate(blocks):
        blk = (ref[r0:r0 + 32, c0:c0 + 48].float() * (1 - lr * wd)).bfloat16().double()
        ref[r0:r0 + 32, c0:c0 + 48] = blk - lr * recv[slots[k].item()].double()
    # one rounding of an exact result (the kernel's fma) to bf16: within half a bf16 ulp (+ a tie)
    err = (P.double() - ref).abs()
    assert bool((err <= ref.abs() * 2.0 ** -8 + 1e-30).all()), err.max().item()
    untouched = torch.ones_like(P, dtype=torch.bool)
    for r0, c0 in blocks:
        untouched[r0:r0 + 32, c0:c0 + 48] = False
    assert torch.equal(P[untouched], P0[untouched])


@pytest.mark.parametrize("shape", [(2, 96, 64, 128), (1, 1024, 576, 1024), (3, 200, 40, 96)])
def test_gemm_f32_3xtf32(shape):
    """lsr_gemm_f32 (3xTF32 on the tensor cores) against an fp64 product: fp32-level accuracy."""
    from lsr import _lib as L
    lib = L.load()
    b, M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(b, M, K, device="cuda", generator=g)
    B = torch.randn(b, K, N, device="cuda", generator=g)
    C = torch.empty(b, M, N, device="cuda")
    nb = lib.lsr_gemm_f32_workspace_bytes(b, M, N, K)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    L.check(lib.lsr_gemm_f32(A.data_ptr(), B.data_ptr(), C.data_ptr(), b, M, N, K, 0.5, ws.data_ptr(), nb,
                             L.stream_handle()), "lsr_gemm_f32")
    ref = 0.5 * (A.double() @ B.double())
    assert rel_fro(C.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("n", [32, 100, 257, 1024])
def test_householder_qr(n):
    """lsr_householder_qr_f32: Q orthonormal, R = Q^T W upper triangular with a non-negative diagonal,
    Q equal to the float64 Householder QR's Q with the same sign convention."""
    from lsr import _lib as L
    lib = L.load()
    b = 2
    g = torch.Generator(device="cuda").manual_seed(n)
    W0 = torch.randn(b, n, n, device="cuda", generator=g)
    W = W0.clone()
    Q = torch.empty_like(W)
    nb = lib.lsr_qr_workspace_bytes(b, n)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    L.check(lib.lsr_householder_qr_f32(W.data_ptr(), Q.data_ptr(), b, n, ws.data_ptr(), nb, L.stream_handle()),
            "lsr_householder_qr_f32")
    Qd = Q.double()
    eye = torch.eye(n, dtype=torch.float64, device="cuda")
    assert (Qd.transpose(1, 2) @ Qd - eye).abs().max().item() < 1e-4 * max(1.0, n / 256)
    R = Qd.transpose(1, 2) @ W0.double()
    assert torch.tril(R, -1).abs().max().item() < 1e-4 * R.abs().max().item()
    assert bool((torch.diagonal(R, dim1=1, dim2=2) >= -1e-6).all())
    Qr, Rr = torch.linalg.qr(W0.double())
    Qr = Qr * torch.sign(torch.diagonal(Rr, dim1=1, dim2=2)).unsqueeze(1)
    # Q's sensitivity grows with cond(W) (about n for a Gaussian W): an fp32 bound of that size
    assert rel_fro(Q.cpu().numpy(), Qr.cpu().numpy()) < 2e-6 * n


def test_eigenbasis_refresh_converges_to_eigenvectors():
    """lsr_eigenbasis_refresh_f32: power iteration with QR from the identity on S = V diag(l) V^T
    (well-separated eigenvalues) diagonalises S; one more refresh from a converged basis returns
    it unchanged up to rounding (no column sign flips); the bf16 copy is the rounded fp32 basis."""
    from lsr import _lib as L
    lib = L.load()
    b, n = 2, 256
    g = torch.Generator().manual_seed(9)
    V = torch.linalg.qr(torch.randn(b, n, n, generator=g, dtype=torch.float64))[0]
    lam = torch.logspace(0, -3, n, dtype=torch.float64)
    S = ((V * lam) @ V.transpose(1, 2)).float().cuda()
    Qf = torch.empty(b, n, n, device="cuda")
    Qb = torch.empty(b, n, n, dtype=torch.bfloat16, device="cuda")
    nb = lib.lsr_eigenbasis_refresh_workspace_bytes(b, n)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    st = L.stream_handle()
    L.check(lib.lsr_eigenbasis_refresh_f32(S.data_ptr(), Qf.data_ptr(), Qb.data_ptr(), b, n, 0.0, 1, 400,
                                           ws.data_ptr(), nb, st), "refresh")
    D = Qf.double().transpose(1, 2) @ S.double() @ Qf.double()
    off = D - torch.diag_embed(torch.diagonal(D, dim1=1, dim2=2))
    assert (off.norm() / D.norm()).item() < 1e-3
    Q1 = Qf.clone()
    L.check(lib.lsr_eigenbasis_refresh_f32(S.data_ptr(), Qf.data_ptr(), Qb.data_ptr(), b, n, 0.0, 0, 1,
                                           ws.data_ptr(), nb, st), "refresh")
    assert rel_fro(Qf.cpu().numpy(), Q1.cpu().numpy()) < 1e-2
    assert torch.equal(Qb, Qf.bfloat16())
