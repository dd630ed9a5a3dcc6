"""Hawkes event update: the oracle against the reference's own identity and a scalar loop, and the
host wrapper's argument checks (CPU only; the kernels are checked in test_gpu_hawkes.py).

The reference checks its two kernels against each other (hft.py:742-745): with
event = event_asset * NE + event_type and Kcol = kron(KA, KE)^T, the dense update and the
Kronecker update are the same."""
import numpy as np
import pytest
import torch

from oracle import hawkes as oh


def _case(N=37, NA=6, NE=4, seed=3):
    rng = np.random.default_rng(seed)
    D = NA * NE
    state = rng.standard_normal((N, D))
    decay = rng.uniform(0.5, 1.0, N)
    KA = rng.standard_normal((NA, NA))
    KE = rng.standard_normal((NE, NE))
    ea = rng.integers(0, NA, N)
    et = rng.integers(0, NE, N)
    return state, decay, KA, KE, ea, et


def test_kron_form_equals_dense_form_with_kron_column():
    state, decay, KA, KE, ea, et = _case()
    NE = KE.shape[0]
    dense = oh.hawkes_dense(state, ea * NE + et, decay, oh.kcol(KA, KE))
    kron = oh.hawkes_kron(state, ea, et, decay, KA, KE)
    np.testing.assert_allclose(kron, dense, rtol=0, atol=1e-12)


def test_kron_form_matches_scalar_loop():
    state, decay, KA, KE, ea, et = _case(N=5, NA=3, NE=2, seed=7)
    NE = KE.shape[0]
    out = oh.hawkes_kron(state, ea, et, decay, KA, KE)
    for n in range(state.shape[0]):
        for j in range(state.shape[1]):
            want = decay[n] * state[n, j] + KA[j // NE, ea[n]] * KE[j % NE, et[n]]
            assert abs(out[n, j] - want) < 1e-12


def test_wrapper_rejects_host_tensors():
    from lsr import hawkes as LH
    state = torch.zeros(4, 6)
    with pytest.raises(ValueError, match="CUDA"):
        LH.hawkes_dense(state, torch.zeros(4, dtype=torch.int32), torch.ones(4), torch.zeros(6, 6), state)
    with pytest.raises(ValueError, match="CUDA"):
        LH.hawkes_kron(state, torch.zeros(4, dtype=torch.int32), torch.zeros(4, dtype=torch.int32), torch.ones(4),
                       torch.zeros(3, 3), torch.zeros(2, 2), state)
