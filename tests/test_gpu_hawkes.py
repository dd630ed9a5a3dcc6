"""Hawkes event update (hft.py:412-611) through lsr.hawkes against the float64 oracle, the identity
the reference checks between its dense and Kronecker kernels, and -- when the reference module is
staged -- the reference's own Triton kernels on the same GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import hawkes as oh
from oracle.bf16 import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-6  # one fp32 FMA (dense) or one product and one FMA (kron) per entry


def problem(N, NA, NE, seed):
    """Inputs distributed as benchmark_hawkes draws them (hft.py:615-735)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    KA = (torch.rand(NA, NA, device="cuda", generator=g) * 0.02).contiguous()
    KE = (torch.rand(NE, NE, device="cuda", generator=g) * 0.02).contiguous()
    Kcol = torch.kron(KA, KE).T.contiguous()
    state = torch.randn(N, NA * NE, device="cuda", generator=g)
    ea = torch.randint(0, NA, (N,), device="cuda", generator=g, dtype=torch.int32)
    et = torch.randint(0, NE, (N,), device="cuda", generator=g, dtype=torch.int32)
    decay = (0.90 + 0.099 * torch.rand(N, device="cuda", generator=g)).contiguous()
    return state, ea, et, (ea * NE + et).contiguous(), decay, KA, KE, Kcol


@pytest.mark.parametrize("N,NA,NE", [(1024, 128, 8), (8192, 128, 8), (1, 128, 8), (77, 5, 3), (300, 16, 1)])
def test_hawkes_matches_oracle(N, NA, NE):
    from lsr import hawkes as H
    state, ea, et, ev, decay, KA, KE, Kcol = problem(N, NA, NE, 123 + N)
    out_d = torch.full_like(state, float("nan"))
    out_k = torch.full_like(state, float("nan"))
    H.hawkes_dense(state, ev, decay, Kcol, out_d)
    H.hawkes_kron(state, ea, et, decay, KA, KE, out_k)
    c = lambda t: t.cpu().numpy()  # noqa: E731
    ref = oh.hawkes_dense(c(state), c(ev), c(decay), c(Kcol))
    assert rel_fro(c(out_d), ref) < TOL
    assert rel_fro(c(out_k), oh.hawkes_kron(c(state), c(ea), c(et), c(decay), c(KA), c(KE))) < TOL
    # the reference's own check: the Kronecker kernel reproduces the dense one (hft.py:742-745)
    assert rel_fro(c(out_k), c(out_d)) < TOL


def test_hawkes_in_place_int64_events_and_empty():
    from lsr import hawkes as H
    state, ea, et, ev, decay, KA, KE, Kcol = problem(257, 128, 8, 7)
    ref = oh.hawkes_kron(state.cpu().numpy(), ea.cpu().numpy(), et.cpu().numpy(), decay.cpu().numpy(),
                         KA.cpu().numpy(), KE.cpu().numpy())
    s2 = state.clone()
    H.hawkes_kron(s2, ea.long(), et.long(), decay, KA, KE, s2)  # out aliases state
    assert rel_fro(s2.cpu().numpy(), ref) < TOL
    s3 = state.clone()
    H.hawkes_dense(s3, ev.long(), decay, Kcol, s3)
    assert rel_fro(s3.cpu().numpy(), ref) < TOL
    e = torch.empty(0, 1024, device="cuda")
    H.hawkes_dense(e, torch.empty(0, dtype=torch.int32, device="cuda"), torch.empty(0, device="cuda"), Kcol, e)


def test_hawkes_event_out_of_range_is_reported_not_read():
    """An event index outside the matrix is caught by the kernel's own bounds check: the row becomes
    NaN, the other rows are right, and the device status word reads 110."""
    from lsr import _lib, hawkes as H
    state, ea, et, ev, decay, KA, KE, Kcol = problem(64, 128, 8, 9)
    _lib.device_status(clear=True)
    bad = ev.clone()
    bad[5] = 128 * 8  # one past the last column of K
    out = torch.empty_like(state)
    H.hawkes_dense(state, bad, decay, Kcol, out)
    assert _lib.device_status(clear=True) == 110
    o = out.cpu().numpy()
    assert np.isnan(o[5]).all() and not np.isnan(np.delete(o, 5, axis=0)).any()
    bad_t = et.clone()
    bad_t[0] = -1
    H.hawkes_kron(state, ea, bad_t, decay, KA, KE, out)
    assert _lib.device_status(clear=True) == 110
    assert np.isnan(out[0].cpu().numpy()).all()


def test_hawkes_errors():
    from lsr import hawkes as H
    state, ea, et, ev, decay, KA, KE, Kcol = problem(8, 16, 4, 1)
    with pytest.raises(ValueError, match="CUDA"):
        H.hawkes_dense(state.cpu(), ev, decay, Kcol, state)
    with pytest.raises(ValueError, match="D = "):
        H.hawkes_kron(state, ea, et, decay, KA, KE[:2, :2].contiguous(), state)
    with pytest.raises(ValueError, match="float32"):
        H.hawkes_dense(state.double(), ev, decay, Kcol, state)


def test_hawkes_matches_reference_triton_kernels():
    """The reference's own Triton kernels (function definitions of the staged hft.py) on the same
    inputs and GPU, at the reference benchmark's shape (128 assets x 8 event types, D = 1024)."""
    from oracle import stage_reference
    triton = pytest.importorskip("triton")
    ref = stage_reference.load_functions(
        "hft.py", ["hawkes_dense_kernel", "hawkes_kron_kernel", "hawkes_dense", "hawkes_kron"],
        {"torch": torch, "triton": triton, "tl": triton.language})
    if ref is None:
        pytest.skip("reference module not staged (oracle/stage_reference.py)")
    from lsr import hawkes as H
    state, ea, et, ev, decay, KA, KE, Kcol = problem(8192, 128, 8, 321)
    a, b = torch.empty_like(state), torch.empty_like(state)
    ref["hawkes_dense"](state, ev, decay, Kcol, a)
    H.hawkes_dense(state, ev, decay, Kcol, b)
    assert rel_fro(b.cpu().numpy(), a.cpu().numpy()) < TOL
    ref["hawkes_kron"](state, ea, et, decay, KA, KE, a)
    H.hawkes_kron(state, ea, et, decay, KA, KE, b)
    assert rel_fro(b.cpu().numpy(), a.cpu().numpy()) < TOL
