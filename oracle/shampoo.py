"""CPU restatement of the Shampoo / SOAP preconditioner math (oracle / test infrastructure only).

PARITY UNPINNED: the reference takes this math from the third-party
``distributed_shampoo`` package (facebookresearch/optimizers, installed from
git HEAD without a pinned version, shampoo_soap_lm_ddp_zero1.py:31-36; used at
:132-168, :312-400, :609), which is absent here and has no golden vectors in
the reference. This module restates the published formulas of the workload
definition and reuses the reference's own in-repo pieces:

* two-sided product ``A X B^T``       — kron_apply_shared_2d, hft.py:108-140
* inverse p-th roots                  — coupled_newton_one, shampoo.py:277-347
                                        (and an fp64 eigendecomposition for precomputed roots)

Formulas (per block G of at most max_preconditioner_dim per side):
  statistics  L = b2 L + (1-b2) G G^T,   R = b2 R + (1-b2) G^T G
  Shampoo     P = L^{-1/4} G R^{-1/4}
  SOAP        G' = Q_L^T G Q_R; m = b1 m + (1-b1) G'; v = b2 v + (1-b2) G'^2;
              U' = (m/(1-b1^t)) / (sqrt(v/(1-b2^t)) + eps);  U = Q_L U' Q_R^T
Arithmetic in float64 on the given (bf16-valued) operands.
"""
from __future__ import annotations

import numpy as np


def stats_update(L, R, G, beta2):
    G = np.asarray(G, np.float64)
    Gt = np.swapaxes(G, -1, -2)
    L = beta2 * np.asarray(L, np.float64) + (1.0 - beta2) * (G @ Gt)
    R = beta2 * np.asarray(R, np.float64) + (1.0 - beta2) * (Gt @ G)
    return L, R


def inverse_root(S, root: int = 4, eps: float = 0.0):
    """(S + eps I)^{-1/root} of a symmetric positive (semi)definite matrix via fp64 eigh."""
    S = np.asarray(S, np.float64)
    n = S.shape[-1]
    w, V = np.linalg.eigh(S + eps * np.eye(n))
    w = np.maximum(w, 1e-300)
    return (V * w[..., None, :] ** (-1.0 / root)) @ np.swapaxes(V, -1, -2)


def shampoo_precondition(G, Lroot, Rroot):
    return np.asarray(Lroot, np.float64) @ np.asarray(G, np.float64) @ np.asarray(Rroot, np.float64)


def soap_direction(G, QL, QR, m, v, beta1, beta2, eps, step, bf16_operands=False):
    """Returns (U, m, v) for one SOAP step in the eigenbases QL, QR.

    Default: float64 arithmetic on the given operands (the caller passes G, QL,
    QR already rounded to bf16, the only roundings the reference's fp32 path
    applies to its inputs); this is what the kernels are checked against.

    bf16_operands=True is a diagnostic only: it also rounds every computed GEMM
    operand to bf16 (the intermediate of each two-sided product, cheaper
    association first, and the Adam direction U'), which shows how far a chain
    with plain-bf16 intermediates falls from the default.
    """
    U, m, v, _ = soap_direction_parts(G, QL, QR, m, v, beta1, beta2, eps, step, bf16_operands)
    return U, m, v


def soap_direction_parts(G, QL, QR, m, v, beta1, beta2, eps, step, bf16_operands=False):
    """soap_direction that also returns the Adam direction in the rotated basis: (U, m, v, U')."""
    from .bf16 import round_bf16
    rd = (lambda x: round_bf16(np.asarray(x, np.float32)).astype(np.float64)) if bf16_operands else (lambda x: x)
    QL = np.asarray(QL, np.float64)
    QR = np.asarray(QR, np.float64)
    QLt = np.swapaxes(QL, -1, -2)
    G = np.asarray(G, np.float64)
    right_first = G.shape[-1] > G.shape[-2]
    Gr = QLt @ rd(G @ QR) if right_first else rd(QLt @ G) @ QR
    m = beta1 * np.asarray(m, np.float64) + (1.0 - beta1) * Gr
    v = beta2 * np.asarray(v, np.float64) + (1.0 - beta2) * Gr * Gr
    Up = rd(adam_in_basis(m, v, beta1, beta2, eps, step))
    return soap_rotate_back(Up, QL, QR, bf16_operands), m, v, Up


def adam_in_basis(m, v, beta1, beta2, eps, step):
    """U' = (m / (1 - beta1^t)) / (sqrt(v / (1 - beta2^t)) + eps)."""
    return (np.asarray(m, np.float64) / (1.0 - beta1 ** step)) / (
        np.sqrt(np.asarray(v, np.float64) / (1.0 - beta2 ** step)) + eps)


def soap_rotate_back(Up, QL, QR, bf16_operands=False):
    """U = Q_L U' Q_R^T, the cheaper association first."""
    from .bf16 import round_bf16
    rd = (lambda x: round_bf16(np.asarray(x, np.float32)).astype(np.float64)) if bf16_operands else (lambda x: x)
    QL = np.asarray(QL, np.float64)
    QRt = np.swapaxes(np.asarray(QR, np.float64), -1, -2)
    Up = np.asarray(Up, np.float64)
    right_first = Up.shape[-1] > Up.shape[-2]
    return QL @ rd(Up @ QRt) if right_first else rd(QL @ Up) @ QRt


def coupled_newton_one(A, root, epsilon=0.0, tolerance=1e-6, max_iterations=100):
    """Coupled Newton iteration for A^{-1/root}, restated from shampoo.py:277-347.

    X_0 = z^{1/root} I, M_0 = z A with z = (root+1) / (2 ||A||_F); repeat
    Mp = (1 - 1/root) I + M/root ... in the reference's form Mp = alpha M + (1-alpha) I
    with alpha = -1/root; X <- X Mp; M <- Mp^root M; until max|M - I| <= tolerance.
    Returns (X, iterations, error).
    """
    A = np.asarray(A, np.float64)
    n = A.shape[0]
    I = np.eye(n)
    Ar = A + epsilon * I if epsilon != 0.0 else A
    alpha = -1.0 / float(root)
    z = (root + 1.0) / (2.0 * np.linalg.norm(Ar))
    X = z ** (-alpha) * I
    M = z * Ar
    err = np.abs(M - I).max()
    it = 0
    while err > tolerance and it < max_iterations:
        Mp = alpha * M + (1.0 - alpha) * I
        X = X @ Mp
        M = np.linalg.matrix_power(Mp, root) @ M
        err = np.abs(M - I).max()
        it += 1
    return X, it, float(err)


def block_sizes(n: int, max_dim: int) -> list[int]:
    """Split a dimension into blocks of max_dim plus a remainder (1600 -> [1024, 576])."""
    out = [max_dim] * (n // max_dim)
    if n % max_dim:
        out.append(n % max_dim)
    return out


def soap_flops(r: int, c: int) -> float:
    """Algorithmic flops of one SOAP block step: stats 2r^2c + 2rc^2, rotate and rotate back 2 x (2r^2c + 2rc^2)."""
    return 6.0 * r * c * (r + c)
