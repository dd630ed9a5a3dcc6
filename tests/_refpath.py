"""The reference's torch op sequences, restated for running on the GPU under test.

The reference module cannot travel to the GPU machine, so the tests restate its
few torch lines here to obtain "the reference bf16 path on the same device":

* ``ns_torch``          — zeropower_serial / zeropower_batched_oriented,
                          muon_lm_ddp.py:331-426 (bmm in bf16, cuBLAS)
* ``muon_step_torch``   — _momentum_update + zeropower + _apply_update,
                          muon_lm_ddp.py:554-612
"""
from __future__ import annotations

import math

import torch

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315


@torch.no_grad()
def ns_torch(G: torch.Tensor, ns_steps: int, eps: float, orient: bool = True) -> torch.Tensor:
    X = G.to(dtype=torch.bfloat16, copy=True)
    squeeze = X.dim() == 2
    if squeeze:
        X = X[None]
    transposed = orient and X.shape[-2] > X.shape[-1]
    if transposed:
        X = X.transpose(-1, -2)
    norms = X.flatten(1).norm(dim=1).clamp(min=eps)
    X = X / norms[:, None, None]
    for _ in range(ns_steps):
        A = torch.bmm(X, X.transpose(-1, -2))
        A2 = torch.bmm(A, A)
        B = NS_B * A + NS_C * A2
        X = NS_A * X + torch.bmm(B, X)
    if transposed:
        X = X.transpose(-1, -2)
    X = X.contiguous()
    return X[0] if squeeze else X


def adjusted_lr(lr, shape, mode="original"):
    rows, cols = shape
    if mode == "original":
        return lr * math.sqrt(max(1.0, rows / cols))
    if mode == "match_rms_adamw":
        return lr * 0.2 * math.sqrt(max(rows, cols))
    return lr


@torch.no_grad()
def muon_step_torch(params, grads, moms, lr, mu, nesterov, wd, ns_steps, eps, lr_adjust="original"):
    """In-place reference Muon step on lists of bf16 CUDA tensors."""
    for p, g, buf in zip(params, grads, moms):
        buf.mul_(mu).add_(g)
        u = g + mu * buf if nesterov else buf
        o = ns_torch(u, ns_steps, eps, orient=True)
        if wd != 0.0:
            p.mul_(1.0 - lr * wd)
        p.add_(o.to(dtype=p.dtype), alpha=-adjusted_lr(lr, p.shape, lr_adjust))


def batched_coupled_newton_torch(A, root, tolerance=1e-6, max_iterations=100):
    """The reference's batched coupled Newton recurrence (shampoo.py:408-542) as
    plain torch ops in A's dtype and device (fp32 reference numerics on CPU)."""
    B, n, _ = A.shape
    eye = torch.eye(n, device=A.device, dtype=A.dtype).expand(B, n, n)
    alpha = -1.0 / float(root)
    z = (root + 1.0) / (2.0 * A.flatten(1).norm(dim=1))
    X = (z.pow(-alpha)[:, None, None] * eye).contiguous()
    M = (z[:, None, None] * A).contiguous()
    iters = torch.zeros(B, dtype=torch.int32, device=A.device)
    active = (M - eye).abs().flatten(1).amax(dim=1) > tolerance
    for _ in range(max_iterations):
        if not bool(active.any()):
            break
        Mp = alpha * M + (1.0 - alpha) * eye
        Xn = X @ Mp
        P = Mp @ Mp
        if root == 4:
            P = P @ P
        Mn = P @ M
        m3 = active[:, None, None]
        X = torch.where(m3, Xn, X)
        M = torch.where(m3, Mn, M)
        iters = iters + active.to(torch.int32)
        active = (M - eye).abs().flatten(1).amax(dim=1) > tolerance
    return X, iters
