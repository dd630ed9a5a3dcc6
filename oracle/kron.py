"""CPU restatement of cuda-lsr's Kronecker operators (oracle / test infrastructure only).

* ``kron_apply_shared_2d(X, A, B)`` = A X B^T per snapshot      hft.py:108-140,
                                                               hft_fused.py:463-509
* ``kron_apply(X, As, Bs)``         = Σ_s A_s X B_s^T           hft_fused.py:655-669
                                                               (kron_sum_64x8_kernel, :89-222)
* ``kron_sum(X, A, B)``             = A X + X B^T = (A ⊕ B) vec(X) (S = 2 with (A, I), (I, B))
* ``dense_operator(As, Bs)``        = Σ_s kron(A_s, B_s)        hft_fused.py:574-587 (small sizes)
* ``reconstruct(factors)``          = Σ_s F_0[s] ⊗ ... ⊗ F_{K-1}[s]  kron_cuda.py:242-583, :618-629

Row-major vec throughout: vec_row(A X B^T) = (A ⊗ B) vec_row(X) (hft.py:159-161).
Arithmetic in float64 so the oracle's own error is far below the kernels'.
"""
from __future__ import annotations

import numpy as np


def kron_apply_shared_2d(X, A, B) -> np.ndarray:
    X = np.asarray(X, dtype=np.float64)
    return np.matmul(np.matmul(np.asarray(A, np.float64), X), np.asarray(B, np.float64).T)


def kron_apply(X, As, Bs) -> np.ndarray:
    As = np.asarray(As, np.float64)
    Bs = np.asarray(Bs, np.float64)
    if As.ndim == 2:
        As, Bs = As[None], Bs[None]
    Y = np.zeros(np.shape(X), dtype=np.float64)
    for A, B in zip(As, Bs):
        Y += kron_apply_shared_2d(X, A, B)
    return Y


def kron_sum(X, A, B) -> np.ndarray:
    X = np.asarray(X, np.float64)
    return np.matmul(np.asarray(A, np.float64), X) + np.matmul(X, np.asarray(B, np.float64).T)


def dense_operator(As, Bs) -> np.ndarray:
    As = np.asarray(As, np.float64)
    Bs = np.asarray(Bs, np.float64)
    if As.ndim == 2:
        As, Bs = As[None], Bs[None]
    W = np.zeros((As.shape[1] * Bs.shape[1],) * 2)
    for A, B in zip(As, Bs):
        W += np.kron(A, B)
    return W


def kron_sum_flops(batch: int, m: int, n: int) -> float:
    """Algorithmic flops of (A ⊕ B) vec(X) over a batch: 2 m^2 n + 2 m n^2 per right-hand side."""
    return batch * (2.0 * m * m * n + 2.0 * m * n * n)


def reconstruct(factors) -> np.ndarray:
    """Σ_s kron(F_0[s], ..., F_{K-1}[s]) in float64 (kron_cuda.py vectorized_kron, :618-629)."""
    fs = [np.asarray(f, np.float64) for f in factors]
    W = None
    for s in range(fs[0].shape[0]):
        t = fs[0][s]
        for f in fs[1:]:
            t = np.kron(t, f[s])
        W = t if W is None else W + t
    return W
