"""CPU: the Pauli-string encoding of lsr.pauli against the oracle's, and the oracle's mask form of
H psi against H built as Kronecker products of the 2 x 2 Pauli matrices."""
from __future__ import annotations

import numpy as np
import torch

from oracle import pauli as op


def test_encoding_matches_oracle():
    from lsr.pauli import encode_pauli_strings
    g = torch.Generator().manual_seed(3)
    for S, K in ((1, 1), (7, 5), (64, 20), (300, 30)):
        ops = torch.randint(0, 4, (S, K), generator=g)
        flip, sign, ny = encode_pauli_strings(ops)
        f, s, y = op.encode(ops.numpy())
        assert flip.dtype == sign.dtype == ny.dtype == torch.int32
        assert np.array_equal(flip.numpy(), f) and np.array_equal(sign.numpy(), s) and np.array_equal(ny.numpy(), y)


def test_oracle_mask_form_matches_kronecker_form():
    rng = np.random.default_rng(5)
    for K, S in ((1, 4), (3, 9), (6, 17)):
        ops = rng.integers(0, 4, (S, K))
        coeff = rng.standard_normal(S)
        psi = rng.standard_normal(1 << K) + 1j * rng.standard_normal(1 << K)
        f, s, y = op.encode(ops)
        assert np.abs(op.apply(psi, f, s, y, coeff) - op.dense(ops, coeff) @ psi).max() < 1e-12


def test_wrapper_rejects_host_tensors():
    import pytest
    import torch
    from lsr import pauli as LP
    psi = torch.zeros(8)
    m = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        LP.pauli_apply(psi, psi.clone(), m, m, m, torch.ones(2))
