"""GPU: Shampoo / SOAP preconditioner kernels against the float64 oracle.

Parity is unpinned upstream (distributed_shampoo is third-party and absent);
the oracle restates the workload's formulas. Tolerance: 1e-3 relative
Frobenius (bf16 operands, fp32 accumulation; the bf16 bound of the path).
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


@pytest.mark.parametrize("shape", [(2, 256, 1024), (2, 512, 256), (1, 1600, 640)])
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
                                    0.95, 0.95, 1e-8, 5, bf16_operands=True)
    assert rel_fro(L.cpu().numpy(), Lr) < 1e-5
    assert rel_fro(R.cpu().numpy(), Rr) < 1e-5
    assert rel_fro(m.cpu().numpy(), mr) < TOL
    assert rel_fro(v.cpu().numpy(), vr) < TOL
    assert rel_fro(U.cpu().numpy(), Ur) < TOL


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
                                         np.zeros((r, c)), np.zeros((r, c)), 0.95, 0.95, 1e-8, 1,
                                         bf16_operands=True)
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
