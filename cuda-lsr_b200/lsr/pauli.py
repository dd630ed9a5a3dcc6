"""Pauli-string Hamiltonian apply on B200 (drop-in for pauli.py's encode / native_apply).

* ``encode_pauli_strings(local_ops)``  [S, K] codes 0..3 (I, X, Y, Z) -> (flip, sign, ny_mod4), int32,
                                        pauli.py:159-199
* ``pauli_apply(psi_r, psi_i, flip, sign, ny, coeff, out_r=None, out_i=None)``
      out[r] = Σ_s coeff_s i^{ny_s} (-1)^{popcount((r ^ flip_s) & sign_s)} psi[r ^ flip_s]
* ``native_apply(prob, P, partial_r, partial_i, out_r, out_i, block=256)``  the reference's
      signature (pauli.py:516-578): ``prob`` holds K, S, psi_r / psi_i, flip / sign / ny, coeff;
      P, the partial buffers and block are accepted and not needed (one launch, no partial sums).

The state is complex, kept as separate fp32 real / imaginary arrays of N = 2^K amplitudes, as the
reference keeps it. H is never formed.
"""
from __future__ import annotations

import torch

from . import _lib


def encode_pauli_strings(local_ops: torch.Tensor):
    """local_ops [S, K] int (0 = I, 1 = X, 2 = Y, 3 = Z) -> flip, sign, ny (int32 [S], CPU):
    flip bit k for X or Y on qubit k, sign bit k for Y or Z, ny = number of Y factors mod 4."""
    ops = torch.as_tensor(local_ops).to(torch.int64).cpu()
    if ops.dim() != 2:
        raise ValueError("local_ops must be [S, K]")
    S, K = ops.shape
    if K > 30:
        raise ValueError("at most 30 qubits (int32 masks)")
    bits = torch.ones(K, dtype=torch.int64) << torch.arange(K, dtype=torch.int64)
    flip = (((ops == 1) | (ops == 2)).to(torch.int64) * bits).sum(dim=1)
    sign = (((ops == 2) | (ops == 3)).to(torch.int64) * bits).sum(dim=1)
    ny = (ops == 2).sum(dim=1).remainder(4)
    return flip.to(torch.int32), sign.to(torch.int32), ny.to(torch.int32)


def _vec(t: torch.Tensor, name: str, dtype: torch.dtype, n: int) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (liblsr has no CPU path)")
    if t.dtype != dtype or not t.is_contiguous() or t.numel() != n:
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of {n} entries")
    return t


def pauli_apply(psi_r, psi_i, flip, sign, ny, coeff, out_r=None, out_i=None):
    """H psi for H = Σ_s coeff_s P_s (P_s the Pauli string encoded by flip / sign / ny); returns (out_r, out_i)."""
    N = psi_r.numel()
    if N < 1 or N & (N - 1):
        raise ValueError("the state must have 2^K amplitudes")
    K = N.bit_length() - 1
    S = coeff.numel()
    _vec(psi_r, "psi_r", torch.float32, N)
    _vec(psi_i, "psi_i", torch.float32, N)
    ints = []
    for t, nm in ((flip, "flip"), (sign, "sign"), (ny, "ny")):
        if t.dtype == torch.int64:
            t = t.to(torch.int32)
        ints.append(_vec(t, nm, torch.int32, S))
    _vec(coeff, "coeff", torch.float32, S)
    out_r = torch.empty_like(psi_r) if out_r is None else _vec(out_r, "out_r", torch.float32, N)
    out_i = torch.empty_like(psi_i) if out_i is None else _vec(out_i, "out_i", torch.float32, N)
    for o in (out_r, out_i):
        for src in (psi_r, psi_i):
            if o.data_ptr() == src.data_ptr():
                raise ValueError("out must not alias psi")
    if any(t.device != psi_r.device for t in (psi_i, *ints, coeff, out_r, out_i)):
        raise ValueError("all tensors must be on the same CUDA device")
    lib = _lib.load()
    with _lib.on_device(psi_r.device):
        rc = lib.lsr_pauli_apply_f32(psi_r.data_ptr(), psi_i.data_ptr(), ints[0].data_ptr(), ints[1].data_ptr(),
                                     ints[2].data_ptr(), coeff.data_ptr(), out_r.data_ptr(), out_i.data_ptr(), K, S,
                                     _lib.stream_handle(psi_r.device))
    _lib.check(rc, "lsr_pauli_apply_f32")
    return out_r, out_i


def native_apply(prob, P=None, partial_r=None, partial_i=None, out_r=None, out_i=None, block=256):
    """pauli.py:516-578 signature: writes H psi into out_r / out_i (returns them)."""
    if prob["N"] != 1 << prob["K"] or prob["S"] != prob["coeff"].numel():
        raise ValueError("prob: N must be 2^K and S the number of strings")
    return pauli_apply(prob["psi_r"], prob["psi_i"], prob["flip"], prob["sign"], prob["ny"], prob["coeff"],
                       out_r, out_i)


__all__ = ["encode_pauli_strings", "pauli_apply", "native_apply"]
