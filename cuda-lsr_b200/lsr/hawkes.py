"""Multivariate Hawkes event update on B200 (drop-ins for hft.py's hawkes_dense / hawkes_kron).

* ``hawkes_dense(state, event, decay, Kcol, out)``   out[n] = decay[n] state[n] + Kcol[event[n]]
                                                      (Kcol = K^T, hft.py:539-570)
* ``hawkes_kron(state, event_asset, event_type, decay, KA, KE, out)``
                                                      out[n][j] = decay[n] state[n][j]
                                                                  + KA[j // NE][ea[n]] KE[j % NE][et[n]]
                                                      (K = KA ⊗ KE never formed, hft.py:573-611)

Same arguments, shapes and return value (``out``) as the reference; fp32 state and factors,
int32 events (int64 events are converted). Errors raise before any launch; an event index out
of range is caught on the device (that row becomes NaN, lsr.device_status() reports 110).
"""
from __future__ import annotations

import torch

from . import _lib


def _check(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (liblsr has no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _same_device(*ts: torch.Tensor) -> None:
    if any(t.device != ts[0].device for t in ts[1:]):
        raise ValueError("all tensors must be on the same CUDA device")


def _events(e: torch.Tensor, name: str, n: int) -> torch.Tensor:
    if e.dtype == torch.int64:
        e = e.to(torch.int32)
    _check(e, name, torch.int32)
    if e.shape != (n,):
        raise ValueError(f"{name} must have shape [{n}]")
    return e


def hawkes_dense(state: torch.Tensor, event: torch.Tensor, decay: torch.Tensor, Kcol: torch.Tensor,
                 out: torch.Tensor) -> torch.Tensor:
    """out[n][j] = decay[n] state[n][j] + Kcol[event[n]][j] (hft.py:413-464, 539-570)."""
    for t, nm in ((state, "state"), (decay, "decay"), (Kcol, "Kcol"), (out, "out")):
        _check(t, nm, torch.float32)
    if state.dim() != 2:
        raise ValueError("state must be [N, D]")
    N, D = state.shape
    event = _events(event, "event", N)
    if decay.shape != (N,) or Kcol.shape != (D, D) or out.shape != (N, D):
        raise ValueError(f"decay must be [{N}], Kcol [{D}, {D}] and out [{N}, {D}]")
    _same_device(state, event, decay, Kcol, out)
    lib = _lib.load()
    with _lib.on_device(state.device):
        rc = lib.lsr_hawkes_dense_f32(state.data_ptr(), event.data_ptr(), decay.data_ptr(), Kcol.data_ptr(),
                                      out.data_ptr(), N, D, _lib.stream_handle(state.device))
    _lib.check(rc, "lsr_hawkes_dense_f32")
    return out


def hawkes_kron(state: torch.Tensor, event_asset: torch.Tensor, event_type: torch.Tensor, decay: torch.Tensor,
                KA: torch.Tensor, KE: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[n][j] = decay[n] state[n][j] + KA[j // NE][event_asset[n]] KE[j % NE][event_type[n]]
    (hft.py:468-536, 573-611)."""
    for t, nm in ((state, "state"), (decay, "decay"), (KA, "KA"), (KE, "KE"), (out, "out")):
        _check(t, nm, torch.float32)
    if state.dim() != 2 or KA.dim() != 2 or KE.dim() != 2:
        raise ValueError("state, KA and KE must be 2-D")
    N, D = state.shape
    NA, NE = KA.shape[0], KE.shape[0]
    if KA.shape != (NA, NA) or KE.shape != (NE, NE):
        raise ValueError("KA and KE must be square")
    if D != NA * NE:  # the reference asserts D == NA * NE (hft.py:588)
        raise ValueError(f"state has D = {D}, KA ⊗ KE has {NA * NE}")
    event_asset = _events(event_asset, "event_asset", N)
    event_type = _events(event_type, "event_type", N)
    if decay.shape != (N,) or out.shape != (N, D):
        raise ValueError(f"decay must be [{N}] and out [{N}, {D}]")
    _same_device(state, event_asset, event_type, decay, KA, KE, out)
    lib = _lib.load()
    with _lib.on_device(state.device):
        rc = lib.lsr_hawkes_kron_f32(state.data_ptr(), event_asset.data_ptr(), event_type.data_ptr(),
                                     decay.data_ptr(), KA.data_ptr(), KE.data_ptr(), out.data_ptr(), N, NA, NE,
                                     _lib.stream_handle(state.device))
    _lib.check(rc, "lsr_hawkes_kron_f32")
    return out


__all__ = ["hawkes_dense", "hawkes_kron"]
