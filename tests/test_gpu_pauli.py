"""Pauli-string Hamiltonian apply (pauli.py:296-578) through lsr.pauli against the complex128
oracle and -- when the reference module is staged -- the reference's own Triton native_apply on
the same GPU."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import pauli as op

pytestmark = pytest.mark.gpu

TOL = 2e-6  # fp32 sums of up to 1500 terms of unit-scale amplitudes (relative to the output norm)


def problem(K, S, seed):
    """A random Hamiltonian and normalised state, drawn as make_problem draws them (pauli.py:202-268)."""
    from lsr.pauli import encode_pauli_strings
    g = torch.Generator().manual_seed(seed + 10007 * K + S)
    ops = torch.randint(0, 4, (S, K), generator=g, dtype=torch.int64)
    flip, sign, ny = encode_pauli_strings(ops)
    coeff = torch.randn(S, generator=g) / math.sqrt(S)
    psi_r = torch.randn(1 << K, generator=g)
    psi_i = torch.randn(1 << K, generator=g)
    nrm = torch.sqrt((psi_r ** 2).sum() + (psi_i ** 2).sum())
    cu = lambda t: t.cuda().contiguous()  # noqa: E731
    return {"K": K, "S": S, "N": 1 << K, "local_ops": ops, "flip": cu(flip), "sign": cu(sign), "ny": cu(ny),
            "coeff": cu(coeff), "psi_r": cu(psi_r / nrm), "psi_i": cu(psi_i / nrm)}


def rel(out_r, out_i, ref):
    got = out_r.double().cpu().numpy() + 1j * out_i.double().cpu().numpy()
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300)


@pytest.mark.parametrize("K,S", [(0, 3), (1, 1), (5, 7), (8, 1024), (12, 256), (16, 64), (20, 64), (10, 1500)])
def test_pauli_matches_oracle(K, S):
    from lsr.pauli import native_apply
    prob = problem(K, S, 17)
    out_r = torch.full_like(prob["psi_r"], float("nan"))
    out_i = torch.full_like(prob["psi_i"], float("nan"))
    native_apply(prob, 4, None, None, out_r, out_i)
    c = lambda t: t.cpu().numpy()  # noqa: E731
    ref = op.apply(c(prob["psi_r"]).astype(np.float64) + 1j * c(prob["psi_i"]), c(prob["flip"]), c(prob["sign"]),
                   c(prob["ny"]), c(prob["coeff"]))
    assert rel(out_r, out_i, ref) < TOL


def test_pauli_flip_bits_above_k_are_ignored_and_errors():
    from lsr.pauli import pauli_apply
    prob = problem(6, 40, 3)
    a = pauli_apply(prob["psi_r"], prob["psi_i"], prob["flip"], prob["sign"], prob["ny"], prob["coeff"])
    b = pauli_apply(prob["psi_r"], prob["psi_i"], prob["flip"] | (1 << 20), prob["sign"], prob["ny"], prob["coeff"])
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    with pytest.raises(ValueError, match="alias"):
        pauli_apply(prob["psi_r"], prob["psi_i"], prob["flip"], prob["sign"], prob["ny"], prob["coeff"],
                    prob["psi_r"], torch.empty_like(prob["psi_i"]))
    with pytest.raises(ValueError, match="2\\^K"):
        pauli_apply(prob["psi_r"][:63], prob["psi_i"][:63], prob["flip"], prob["sign"], prob["ny"], prob["coeff"])
    with pytest.raises(ValueError, match="CUDA"):
        pauli_apply(prob["psi_r"].cpu(), prob["psi_i"], prob["flip"], prob["sign"], prob["ny"], prob["coeff"])


def test_pauli_matches_reference_triton_kernels():
    """The reference's native_apply (its Triton partial + reduce kernels, from the staged pauli.py)
    at the reference benchmark's shapes."""
    pytest.importorskip("triton")
    import importlib.util
    from oracle import stage_reference
    path = stage_reference.staged_module_path("pauli.py")
    if path is None:
        pytest.skip("reference module not staged (oracle/stage_reference.py)")
    spec = importlib.util.spec_from_file_location("ref_pauli", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    from lsr.pauli import native_apply
    for K, S, P in ((8, 1024, 16), (12, 256, 4), (16, 64, 2), (20, 64, 1)):
        prob = ref.make_problem(K, S)
        N = prob["N"]
        pr = torch.empty(P * N, device="cuda")
        pi = torch.empty(P * N, device="cuda")
        rr, ri = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
        ref.native_apply(prob, P, pr, pi, rr, ri)
        out_r, out_i = native_apply(prob, P, None, None, torch.empty(N, device="cuda"), torch.empty(N, device="cuda"))
        want = rr.double().cpu().numpy() + 1j * ri.double().cpu().numpy()
        assert rel(out_r, out_i, want) < TOL, (K, S)
