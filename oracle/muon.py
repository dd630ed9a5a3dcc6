"""CPU restatement of Muon's Newton–Schulz path (oracle / test infrastructure only).

Follows muon_lm_ddp.py of the reference:

* ``NS_A, NS_B, NS_C``                       muon_lm_ddp.py:297-299
* ``adjusted_muon_lr``                       muon_lm_ddp.py:302-328
* ``zeropower``  (serial + batched forms)     muon_lm_ddp.py:331-426
* ``momentum_update`` (Nesterov)             muon_lm_ddp.py:554-568
* ``apply_update`` (decoupled weight decay)  muon_lm_ddp.py:571-593

Every tensor op of the reference runs in bf16 storage with an fp32
intermediate; this restatement does the same: products are float32 GEMMs of
bf16-valued operands rounded to bf16, and each scalar*tensor and
tensor+tensor is rounded to bf16, in the reference's op order.
"""
from __future__ import annotations

import math

import numpy as np

from .bf16 import round_bf16

NS_A = 3.4445
NS_B = -4.7750
NS_C = 2.0315


def adjusted_muon_lr(lr: float, shape, mode: str) -> float:
    """muon_lm_ddp.py:302-328."""
    rows, cols = shape
    if mode == "original":
        ratio = math.sqrt(max(1.0, rows / cols))
    elif mode == "match_rms_adamw":
        ratio = 0.2 * math.sqrt(max(rows, cols))
    elif mode == "none":
        ratio = 1.0
    else:
        raise ValueError(mode)
    return lr * ratio


def _f32(x: float) -> np.float32:
    return np.float32(x)


def frob_norm_bf16(X: np.ndarray, eps: float) -> np.ndarray:
    """Per-matrix bf16 Frobenius norm clamped at bf16(eps), over the last two axes."""
    ss = np.sum(np.square(X.astype(np.float64)), axis=(-2, -1))
    nrm = round_bf16(np.sqrt(ss.astype(np.float32)))
    e = round_bf16(np.float32(eps))
    return np.maximum(nrm, e)


def ns_iterate(X: np.ndarray, ns_steps: int, a=NS_A, b=NS_B, c=NS_C) -> np.ndarray:
    """The quintic iteration on bf16-valued float32 X [..., m, n] (muon_lm_ddp.py:405-424)."""
    a, b, c = _f32(a), _f32(b), _f32(c)
    for _ in range(ns_steps):
        Xt = np.swapaxes(X, -1, -2)
        A = round_bf16(np.matmul(X, Xt))
        A2 = round_bf16(np.matmul(A, A))
        B = round_bf16(round_bf16(b * A) + round_bf16(c * A2))
        X = round_bf16(round_bf16(a * X) + round_bf16(np.matmul(B, X)))
    return X


def zeropower(G: np.ndarray, ns_steps: int, eps: float, orient: bool = True, a=NS_A, b=NS_B, c=NS_C) -> np.ndarray:
    """Newton–Schulz orthogonalisation of G [..., rows, cols].

    orient=True mirrors zeropower_serial (tall inputs are transposed and the
    result transposed back, muon_lm_ddp.py:346-368); orient=False mirrors
    zeropower_batched_oriented (input used as given, muon_lm_ddp.py:385-426).
    """
    X = round_bf16(np.asarray(G, dtype=np.float32))
    transposed = orient and X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    nrm = frob_norm_bf16(X, eps)
    X = round_bf16(X / nrm[..., None, None])
    X = ns_iterate(X, ns_steps, a, b, c)
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    return X


def momentum_update(buf: np.ndarray, g: np.ndarray, mu: float, nesterov: bool):
    """buf = mu*buf + g ; u = g + mu*buf (Nesterov) — muon_lm_ddp.py:554-568.

    Returns (new_buf, u); both bf16-valued float32.
    """
    mu = _f32(mu)
    buf = round_bf16(round_bf16(mu * buf) + g)
    u = round_bf16(g + round_bf16(mu * buf)) if nesterov else buf
    return buf, u


def apply_update(p: np.ndarray, update: np.ndarray, lr: float, wd: float, lr_adj: float) -> np.ndarray:
    """p *= 1 - lr*wd ; p += -lr_adj * update — muon_lm_ddp.py:571-593."""
    if wd != 0.0:
        p = round_bf16(p * _f32(1.0 - lr * wd))
    return round_bf16(p + _f32(-lr_adj) * update)


def muon_step(params, grads, moms, *, lr: float, mu: float, nesterov: bool, wd: float, ns_steps: int, eps: float,
              lr_adjust: str = "original"):
    """One MuonAdamW.muon_step() over lists of 2-D bf16-valued arrays.

    Returns (new_params, new_moms).
    """
    new_p, new_m = [], []
    for p, g, m in zip(params, grads, moms):
        m2, u = momentum_update(m, g, mu, nesterov)
        o = zeropower(u, ns_steps, eps, orient=True)
        new_p.append(apply_update(p, o, lr, wd, adjusted_muon_lr(lr, p.shape, lr_adjust)))
        new_m.append(m2)
    return new_p, new_m


def ns_flops(m: int, n: int, steps: int = 5) -> float:
    """Dense flop count of `steps` quintic iterations on an oriented m x n matrix (m <= n)."""
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)
