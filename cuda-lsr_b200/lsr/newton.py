"""Coupled Newton inverse roots for Shampoo factors (drop-in for shampoo.py).

Same names, arguments and return values as the reference's
``coupled_newton_one`` (shampoo.py:277-347), ``per_factor_coupled_newton``
(:351-400), ``batched_coupled_newton`` (:408-542) and ``hybrid_coupled_newton``
(:545-595); every one runs the batched sm_100a kernel chain
``lsr_coupled_newton_f32`` (fp32 factors, root 2 or 4).

The kernel keeps an independent convergence mask per factor and computes each
factor's recurrence on its own, so the batched result of a factor equals its
per-factor result. The products run in fp32 FFMA on the CUDA cores (the
reference turns TF32 off, shampoo.py:73-75), as symmetric upper triangles. When
``torch.backends.cuda.matmul.allow_tf32`` is on, they run as 3xTF32 on the
tensor cores until max|M - I| <= 1e-4 and in fp32 FFMA from there (X within
~1e-4 of the fp32 result), and ill-conditioned factors (more than 14 / 13
iterations for root 2 / 4) are recomputed in fp32 FFMA. `iters` counts the
recurrence's iterations, `err` is the final max|M - I|. `hard` of
``hybrid_coupled_newton`` keeps the reference's meaning: iters above the
fallback threshold (15 for root 2, 16 for root 4).
"""
from __future__ import annotations

import torch

from . import _lib

FALLBACK_THRESHOLD = {2: 15, 4: 16}


def _run(A: torch.Tensor, root: int, epsilon: float, tolerance: float, max_iterations: int,
         check_every: int = 4, use_tf32: bool | None = None):
    if not A.is_cuda:
        raise ValueError("coupled Newton: A must be a CUDA tensor (there is no CPU path)")
    if A.dim() != 3 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"coupled Newton: expected [B, n, n], got {tuple(A.shape)}")
    if root not in (2, 4):
        raise ValueError("This benchmark supports root=2 or root=4.")
    Af = A.to(torch.float32).contiguous()
    B, n, _ = Af.shape
    X = torch.empty_like(Af)
    iters = torch.zeros(B, dtype=torch.int32, device=A.device)
    err = torch.zeros(B, dtype=torch.float32, device=A.device)
    redo = torch.zeros(B, dtype=torch.int32, device=A.device)
    if B == 0:
        return X, iters, err, redo.bool()
    lib = _lib.load()
    nb = lib.lsr_coupled_newton_workspace_bytes(B, n)
    if nb == 0:
        raise ValueError(f"coupled Newton: unsupported size B={B}, n={n} (n must be a multiple of 4)")
    ws = _lib.WORKSPACE.get(nb, A.device)
    _lib.check(lib.lsr_coupled_newton_f32(Af.data_ptr(), X.data_ptr(), iters.data_ptr(), err.data_ptr(),
                                          redo.data_ptr(), B, n, root,
                                          float(epsilon), float(tolerance), int(max_iterations), int(check_every),
                                          int(bool(torch.backends.cuda.matmul.allow_tf32 if use_tf32 is None
                                                   else use_tf32)),
                                          ws.data_ptr(), nb, _lib.stream_handle(A.device)),
               "lsr_coupled_newton_f32")
    return X, iters, err, redo.bool()


@torch.no_grad()
def batched_coupled_newton(A, root, epsilon=0.0, tolerance=1e-6, max_iterations=100):
    """A [B, n, n] -> (X [B, n, n], iters int32 [B], err fp32 [B]) (shampoo.py:408-542)."""
    X, iters, err, _ = _run(A, root, epsilon, tolerance, max_iterations)
    return X, iters, err


@torch.no_grad()
def coupled_newton_one(A, root, epsilon=0.0, tolerance=1e-6, max_iterations=100):
    """A [n, n] -> (X [n, n], iterations, final max|M - I|) (shampoo.py:277-347)."""
    X, it, err, _ = _run(A.unsqueeze(0), root, epsilon, tolerance, max_iterations)
    return X[0], int(it[0].item()), float(err[0].item())


@torch.no_grad()
def per_factor_coupled_newton(A, root, epsilon=0.0, tolerance=1e-6, max_iterations=100):
    """Factor-by-factor execution (shampoo.py:351-400): (X, iters, errors)."""
    outs, its, errs = [], [], []
    for b in range(A.shape[0]):
        X, it, err = coupled_newton_one(A[b], root, epsilon, tolerance, max_iterations)
        outs.append(X)
        its.append(it)
        errs.append(err)
    dev = A.device
    return (torch.stack(outs, 0), torch.tensor(its, device=dev, dtype=torch.int32),
            torch.tensor(errs, device=dev, dtype=torch.float32))


@torch.no_grad()
def hybrid_coupled_newton(A, root, epsilon=0.0, tolerance=1e-6, max_iterations=100):
    """(X, iters, hard, err) as shampoo.py:545-595; `hard` marks factors that
    needed more than the fallback threshold of iterations."""
    X, iters, err, _ = _run(A, root, epsilon, tolerance, max_iterations)
    return X, iters, iters > FALLBACK_THRESHOLD[root], err
