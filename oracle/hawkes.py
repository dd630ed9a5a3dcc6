"""CPU restatement of cuda-lsr's multivariate Hawkes event update (oracle / test infrastructure only).

* ``hawkes_dense(state, event, decay, Kcol)``  out[n] = decay[n] state[n] + Kcol[event[n]]
                                               (hawkes_dense_kernel, hft.py:413-464)
* ``hawkes_kron(state, ea, et, decay, KA, KE)`` out[n][j] = decay[n] state[n][j]
                                               + KA[j // NE][ea[n]] KE[j % NE][et[n]]
                                               (hawkes_kron_kernel, hft.py:468-536)
* ``kcol(KA, KE)``                              Kcol = (KA ⊗ KE)^T, as benchmark_hawkes builds it
                                               (hft.py:648-661)

Float64 arithmetic. The reference's own check is the identity the two kernels share: with
event = ea NE + et and Kcol = kron(KA, KE)^T, both give the same update (hft.py:742-745).
"""
from __future__ import annotations

import numpy as np


def kcol(KA, KE) -> np.ndarray:
    return np.kron(np.asarray(KA, np.float64), np.asarray(KE, np.float64)).T.copy()


def hawkes_dense(state, event, decay, Kcol) -> np.ndarray:
    state = np.asarray(state, np.float64)
    Kcol = np.asarray(Kcol, np.float64)
    return np.asarray(decay, np.float64)[:, None] * state + Kcol[np.asarray(event, np.int64)]


def hawkes_kron(state, event_asset, event_type, decay, KA, KE) -> np.ndarray:
    state = np.asarray(state, np.float64)
    KA = np.asarray(KA, np.float64)
    KE = np.asarray(KE, np.float64)
    NA, NE = KA.shape[0], KE.shape[0]
    j = np.arange(NA * NE)
    ea = np.asarray(event_asset, np.int64)[:, None]
    et = np.asarray(event_type, np.int64)[:, None]
    excite = KA[(j // NE)[None, :], ea] * KE[(j % NE)[None, :], et]  # [N, D]
    return np.asarray(decay, np.float64)[:, None] * state + excite
