"""CPU restatement of cuda-lsr's Pauli-string Hamiltonian apply (oracle / test infrastructure only).

* ``encode(local_ops)``          flip / sign / ny_mod4 masks of [S, K] codes 0..3 = I, X, Y, Z
                                 (encode_pauli_strings, pauli.py:159-199)
* ``apply(psi, flip, sign, ny, coeff)``
                                 out[r] = Σ_s coeff_s i^{ny_s} (-1)^{popcount((r ^ flip_s) & sign_s)} psi[r ^ flip_s]
                                 (pauli_partial_kernel + pauli_reduce_kernel, pauli.py:296-513)
* ``dense(local_ops, coeff)``    H = Σ_s coeff_s ⊗_k σ_{ops[s][k]} for small K, qubit k the k-th
                                 least significant bit of the basis index (build_dense_hamiltonian,
                                 pauli.py:764-840), to check ``apply`` against the Kronecker form

Complex128 arithmetic. The reference's own checks are native vs its torch paths and, for small K,
vs the dense Hamiltonian (pauli.py:984-1180).
"""
from __future__ import annotations

import numpy as np

_SIGMA = [np.eye(2), np.array([[0, 1], [1, 0]]), np.array([[0, -1j], [1j, 0]]), np.array([[1, 0], [0, -1]])]


def encode(local_ops):
    ops = np.asarray(local_ops, np.int64)
    S, K = ops.shape
    bits = 1 << np.arange(K, dtype=np.int64)
    flip = (((ops == 1) | (ops == 2)) * bits).sum(axis=1)
    sign = (((ops == 2) | (ops == 3)) * bits).sum(axis=1)
    ny = (ops == 2).sum(axis=1) % 4
    return flip.astype(np.int64), sign.astype(np.int64), ny.astype(np.int64)


def _popcount_parity(x: np.ndarray) -> np.ndarray:
    x = x.copy()
    for sh in (16, 8, 4, 2, 1):
        x ^= x >> sh
    return x & 1


def apply(psi, flip, sign, ny, coeff) -> np.ndarray:
    psi = np.asarray(psi, np.complex128)
    N = psi.shape[0]
    r = np.arange(N, dtype=np.int64)
    out = np.zeros(N, np.complex128)
    phase = np.array([1, 1j, -1, -1j])
    for f, sg, y, c in zip(np.asarray(flip, np.int64), np.asarray(sign, np.int64), np.asarray(ny, np.int64),
                           np.asarray(coeff, np.float64)):
        cidx = r ^ f
        par = _popcount_parity(cidx & sg)
        out += c * phase[y % 4] * np.where(par == 1, -1.0, 1.0) * psi[cidx]
    return out


def dense(local_ops, coeff) -> np.ndarray:
    ops = np.asarray(local_ops, np.int64)
    S, K = ops.shape
    H = np.zeros((1 << K, 1 << K), np.complex128)
    for s in range(S):
        term = np.ones((1, 1), np.complex128)
        for k in range(K - 1, -1, -1):  # most significant qubit first in the Kronecker product
            term = np.kron(term, _SIGMA[ops[s, k]])
        H += float(coeff[s]) * term
    return H
