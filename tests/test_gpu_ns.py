"""GPU parity of the Newton–Schulz / Muon path.

Tolerance: relative Frobenius error <= 2e-2 against the reference bf16 path
(the bound the optimizer path is specified to meet); the kernels round at the
reference's bf16 points, so the measured errors sit far below it. Checked
against (1) the numpy oracle, (2) golden outputs of the reference's own
functions, (3) the reference's torch op sequence run on this GPU (cuBLAS).
"""
import numpy as np
import pytest
import torch

from oracle import muon as om
from oracle.bf16 import from_bits, rel_fro

from _refpath import muon_step_torch, ns_torch

pytestmark = pytest.mark.gpu

TOL = 2e-2
GOLD = None


def gold():
    global GOLD
    if GOLD is None:
        from pathlib import Path
        GOLD = np.load(Path(__file__).parent / "golden" / "muon_golden.npz")
    return GOLD


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda().bfloat16()


def _np(t):
    return t.float().cpu().numpy()


def test_serial_matches_golden_and_oracle():
    import lsr
    z = gold()
    for i, (r, c) in enumerate(z["serial_shapes"]):
        G = from_bits(z[f"serial{i}_in"]).reshape(r, c)
        ref = from_bits(z[f"serial{i}_out"]).reshape(r, c)
        out = _np(lsr.zeropower_serial(_t(G), 5, 1e-7))
        assert out.shape == (r, c)
        e_ref = rel_fro(out, ref)
        e_or = rel_fro(out, om.zeropower(G, 5, 1e-7))
        assert e_ref < TOL and e_or < TOL, (r, c, e_ref, e_or)
    assert lsr._lib.device_status() == 0


def test_batched_matches_golden():
    import lsr
    z = gold()
    X = from_bits(z["batched_in"]).reshape(3, 64, 192)
    out = _np(lsr.zeropower_batched_oriented(_t(X), 5, 1e-7))
    assert rel_fro(out, from_bits(z["batched_out"]).reshape(3, 64, 192)) < TOL
    assert rel_fro(out, om.zeropower(X, 5, 1e-7, orient=False)) < TOL


@pytest.mark.parametrize("steps", [0, 1, 3])
def test_step_counts(steps):
    import lsr
    z = gold()
    G = from_bits(z["steps_in"]).reshape(48, 160)
    out = _np(lsr.zeropower_serial(_t(G), steps, 1e-7))
    assert rel_fro(out, from_bits(z[f"steps{steps}_out"]).reshape(48, 160)) < TOL


def test_config1_vs_reference_on_device():
    """Config 1: 12 of 768x3072 and 12 of 3072x768, N(0, 0.02^2), seed 0."""
    import lsr
    g = torch.Generator().manual_seed(0)
    wide = (torch.randn(12, 768, 3072, generator=g) * 0.02).bfloat16().cuda()
    tall = (torch.randn(12, 3072, 768, generator=g) * 0.02).bfloat16().cuda()
    for stack in (wide, tall):
        ours = torch.stack([lsr.zeropower_serial(stack[i], 5, 1e-7) for i in range(12)])
        batched = lsr.zeropower_via_newtonschulz5(stack, 5, 1e-7)
        assert torch.equal(ours, batched)
        ref = torch.stack([ns_torch(stack[i], 5, 1e-7) for i in range(12)])
        errs = [rel_fro(_np(ours[i]), _np(ref[i])) for i in range(12)]
        assert max(errs) < TOL, errs
    # golden checksums of the reference's own CPU run on the first matrices (same seed)
    z = gold()
    g0 = torch.Generator().manual_seed(0)
    for name, (r, c) in (("cfg1_wide", (768, 3072)), ("cfg1_tall", (3072, 768))):
        G = (torch.randn(r, c, generator=g0) * 0.02).bfloat16()
        Gd = G.double()
        assert np.allclose([Gd.sum().item(), (Gd * Gd).sum().item()], z[f"{name}_in_sums"])
        out = _np(lsr.zeropower_serial(G.cuda(), 5, 1e-7))
        assert rel_fro(out[:64], from_bits(z[f"{name}_out_rows"]).reshape(64, -1)) < TOL
        assert rel_fro(out.astype(np.float64).sum(0), z[f"{name}_out_colsum"]) < TOL


@pytest.mark.parametrize("shape", [(1, 5), (5, 1), (200, 300), (300, 200), (130, 130), (8, 2050)])
def test_ragged_shapes_vs_oracle(shape):
    import lsr
    r, c = shape
    g = torch.Generator().manual_seed(r * 1000 + c)
    G = (torch.randn(r, c, generator=g) * 0.02).bfloat16()
    out = _np(lsr.zeropower_serial(G.cuda(), 5, 1e-7))
    ref = om.zeropower(G.float().numpy(), 5, 1e-7)
    assert rel_fro(out, ref) < TOL


@pytest.mark.parametrize("shape", [(160, 480), (480, 160), (320, 320), (1600, 1600), (3, 320, 960), (3, 960, 320)])
def test_narrow_tile_shapes(shape):
    """Row counts that are multiples of 160 but not of 256 (GPT-2-XL's 1600) run on 160-wide tiles
    and the transposed update (X'^T = X^T B); wide, tall and batched inputs against the reference
    op sequence on this GPU and, for the small cases, the oracle."""
    import lsr
    g = torch.Generator().manual_seed(sum(shape))
    G = (torch.randn(*shape, generator=g) * 0.02).bfloat16()
    if len(shape) == 2:
        out = lsr.zeropower_serial(G.cuda(), 5, 1e-7)
    else:
        out = lsr.zeropower_via_newtonschulz5(G.cuda(), 5, 1e-7)
    assert out.shape == G.shape
    ref = ns_torch(G.cuda(), 5, 1e-7)
    assert rel_fro(_np(out), _np(ref)) < TOL
    if len(shape) == 2 and max(shape) <= 480:
        assert rel_fro(_np(out), om.zeropower(G.float().numpy(), 5, 1e-7)) < TOL
    assert lsr._lib.device_status() == 0


def test_zero_matrix_is_finite():
    import lsr
    out = lsr.zeropower_serial(torch.zeros(64, 128, device="cuda", dtype=torch.bfloat16), 5, 1e-7)
    assert torch.isfinite(out.float()).all() and out.float().abs().max().item() == 0.0


def test_muon_adamw_matches_golden():
    import lsr
    z = gold()
    names = [("h.0.attn.c_attn.weight", (64, 192)), ("h.0.attn.c_proj.weight", (64, 64)),
             ("h.0.mlp.c_fc.weight", (64, 256)), ("h.0.mlp.c_proj.weight", (256, 64)),
             ("h.1.mlp.c_fc.weight", (64, 256)), ("h.1.mlp.c_proj.weight", (256, 64)),
             ("wte.weight", (100, 64)), ("ln_f.bias", (64,))]
    for mode in ("batched", "serial"):
        params = {n: torch.nn.Parameter(_t(from_bits(z[f"muon_init_{n}"]).reshape(s))) for n, s in names}
        opt = lsr.MuonAdamW(list(params.items()), muon_mode=mode, muon_lr=0.02, muon_momentum=0.95,
                            muon_weight_decay=0.01, muon_nesterov=True, muon_ns_steps=5, muon_eps=1e-7,
                            muon_lr_adjust="original", muon_batch_matrices=8, adam_lr=3e-4,
                            adam_betas=(0.9, 0.95), adam_weight_decay=0.1, rank=0)
        for step in range(2):
            for n, s in names:
                params[n].grad = _t(from_bits(z[f"muon_grad{step}_{n}"]).reshape(s))
            opt.muon_step()
        for n, s in names:
            if len(s) == 2 and "wte" not in n:
                p0 = from_bits(z[f"muon_init_{n}"]).reshape(s)
                ref = from_bits(z[f"muon_{mode}_{n}"]).reshape(s)
                got = _np(params[n].data)
                # The parameter change is lr * update rounded into bf16 parameters: a
                # 1e-2 difference in the update flips some of those roundings, so the
                # change is compared at 0.1 and the update itself is checked at 2e-2
                # in test_muon_stages_vs_torch_reference_gpt2_shapes.
                assert rel_fro(got - p0, ref - p0) < 0.1, (mode, n)
                mom = from_bits(z[f"muon_{mode}_mom_{n}"]).reshape(s)
                assert rel_fro(_np(opt.momentum[params[n]]), mom) < 1e-6, (mode, n)
        summ = opt.summary()
        assert [summ["muon_param_count"], summ["adam_param_count"], summ["muon_matrix_count"]] == \
            list(z["summary_muon_count"])


def test_muon_stages_vs_torch_reference_gpt2_shapes():
    """A 2-layer slice of GPT-2-XL's Muon matrices, stage by stage, against the
    reference op sequence on this GPU: momentum bit-exact, orthogonalised update
    within 2e-2, and the apply given the reference's update within one bf16 ulp."""
    import lsr
    from lsr.muon import MuonStepEngine, adjusted_muon_lr
    shapes = [(1600, 4800), (1600, 1600), (1600, 6400), (6400, 1600)] * 2
    g = torch.Generator().manual_seed(4)
    P = [(torch.randn(*s, generator=g) * 0.02).bfloat16().cuda() for s in shapes]
    Gr = [(torch.randn(*s, generator=g) * 0.01).bfloat16().cuda() for s in shapes]
    M = [(torch.randn(*s, generator=g) * 0.01).bfloat16().cuda() for s in shapes]
    # reference stages
    M_ref = [m.clone() for m in M]
    U_ref = []
    for gr, buf in zip(Gr, M_ref):
        buf.mul_(0.95).add_(gr)
        U_ref.append(ns_torch(gr + 0.95 * buf, 5, 1e-7))
    # ours
    eng = MuonStepEngine()
    M_our = [m.clone() for m in M]
    items = [(p, gr, m, adjusted_muon_lr(0.02, p.shape, "original")) for p, gr, m in zip(P, Gr, M_our)]
    grouped = eng.group_items(items)
    upd = eng.orthogonalize(grouped, momentum=0.95, nesterov=True, ns_steps=5, eps=1e-7)
    for (shape, _, its), u in zip(grouped, upd):
        for k, it in enumerate(its):
            i = next(j for j in range(len(P)) if P[j] is it[0])
            assert torch.equal(M_our[i], M_ref[i])
            ref_o = U_ref[i] if shape[0] <= shape[1] else U_ref[i].T
            assert rel_fro(_np(u[k]), _np(ref_o)) < TOL, (shape, k)
    # apply the reference's own updates with our kernel
    upd_ref = []
    for shape, _, its in grouped:
        idx = [next(j for j in range(len(P)) if P[j] is it[0]) for it in its]
        upd_ref.append(torch.stack([U_ref[i] if shape[0] <= shape[1] else U_ref[i].T for i in idx]).contiguous())
    P_our = [p.clone() for p in P]
    items2 = [(p, gr, m, adjusted_muon_lr(0.02, p.shape, "original")) for p, gr, m in zip(P_our, Gr, M)]
    eng.apply(eng.group_items(items2), upd_ref, weight_decay=0.01, base_lr=0.02)
    for i in range(len(P)):
        p_ref = P[i].clone()
        p_ref.mul_(1.0 - 0.02 * 0.01)
        p_ref.add_(U_ref[i], alpha=-adjusted_muon_lr(0.02, P[i].shape, "original"))
        diff = (P_our[i].float() - p_ref.float()).abs()
        ulp = p_ref.float().abs().clamp_min(1e-30) * 2.0 ** -7
        assert bool((diff <= ulp).all()), i
    assert lsr._lib.device_status() == 0


def test_muon_optimizer_end_to_end():
    """torch.optim-style Muon: one step equals orthogonalize + apply."""
    import lsr
    shapes = [(256, 512), (512, 256), (384, 384)]
    g = torch.Generator().manual_seed(7)
    P = [(torch.randn(*s, generator=g) * 0.02).bfloat16().cuda() for s in shapes]
    Gr = [(torch.randn(*s, generator=g) * 0.01).bfloat16().cuda() for s in shapes]
    params = [torch.nn.Parameter(p.clone()) for p in P]
    opt = lsr.Muon(params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.01)
    for p, gr in zip(params, Gr):
        p.grad = gr
    opt.step()
    P_ref, M_ref = [p.clone() for p in P], [torch.zeros_like(p) for p in P]
    muon_step_torch(P_ref, Gr, M_ref, lr=0.02, mu=0.95, nesterov=True, wd=0.01, ns_steps=5, eps=1e-7)
    for i in range(len(P)):
        assert torch.equal(opt.state[params[i]]["momentum_buffer"], M_ref[i])
        # parameter change vs the reference's (bf16 parameter rounding adds noise of a few % here)
        assert rel_fro(_np(params[i].data.float() - P[i].float()), _np(P_ref[i].float() - P[i].float())) < 0.1


def test_cpu_tensor_raises():
    import lsr
    with pytest.raises(ValueError):
        lsr.zeropower_serial(torch.zeros(8, 8, dtype=torch.bfloat16), 5, 1e-7)


def test_orthogonalize_in_two_phases_is_identical():
    """lsr_muon_orthogonalize_phase_bf16: phase 1 then phase 2 over one workspace equals the
    one-call orthogonalize bit for bit (the sharded step runs every prologue first)."""
    from lsr.muon import MuonStepEngine, adjusted_muon_lr
    shapes = [(256, 768), (768, 256), (384, 384)]
    g = torch.Generator().manual_seed(12)
    P = [(torch.randn(*s, generator=g) * 0.02).bfloat16().cuda() for s in shapes]
    Gr = [(torch.randn(*s, generator=g) * 0.01).bfloat16().cuda() for s in shapes]
    M0 = [(torch.randn(*s, generator=g) * 0.01).bfloat16().cuda() for s in shapes]
    eng = MuonStepEngine()
    outs = []
    for phased in (False, True):
        M = [m.clone() for m in M0]
        grouped = eng.group_items([(p, gr, m, adjusted_muon_lr(0.02, p.shape, "original"))
                                   for p, gr, m in zip(P, Gr, M)])
        out = [torch.empty(len(its), min(s), max(s), dtype=torch.bfloat16, device="cuda") for s, _, its in grouped]
        kw = dict(momentum=0.95, nesterov=True, ns_steps=5, eps=1e-7, out=out)
        if phased:
            ws = torch.empty(eng.workspace_bytes(grouped) + 256, dtype=torch.uint8, device="cuda")
            eng.orthogonalize_phase(grouped, 1, ws, **kw)
            eng.orthogonalize_phase(grouped, 2, ws, **kw)
        else:
            eng.orthogonalize(grouped, **kw)
        outs.append((out, M))
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a, b)
    for a, b in zip(outs[0][1], outs[1][1]):
        assert torch.equal(a, b)
