"""ctypes binding of liblsr.so (the C ABI declared in include/lsr.h).

The library is built in-tree by ``cuda-lsr_b200/build.py``. There is no
fallback: if the library is missing or the device is not an sm_100 GPU, the
calls raise.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "liblsr.so"

LSR_OK = 0
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}  # LSR_DTYPE_* (include/lsr.h)
_ERRORS = {
    -1: ValueError,
    -2: ValueError,
    -3: RuntimeError,
    -4: RuntimeError,
    -5: RuntimeError,
    -6: RuntimeError,
    -7: ValueError,
    -8: RuntimeError,
}

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p


class MuonGroup(ctypes.Structure):
    """Mirror of ``lsr_muon_group`` (include/lsr.h)."""

    _fields_ = [
        ("rows", c_int),
        ("cols", c_int),
        ("count", c_int),
        ("grad_ptrs", c_void_p),
        ("mom_ptrs", c_void_p),
        ("param_ptrs", c_void_p),
        ("lr", c_float),
    ]


# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "lsr_version": (ctypes.c_char_p, []),
    "lsr_strerror": (ctypes.c_char_p, [c_int]),
    "lsr_device_status": (c_int, [ctypes.POINTER(c_int), c_int]),
    "lsr_launch_count": (ctypes.c_longlong, []),
    "lsr_profile_enable": (c_int, [c_int]),
    "lsr_profile_read": (c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong), c_int, c_int]),
    "lsr_ns_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "lsr_ns_bf16": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_float, c_float, c_void_p,
         c_size_t, c_void_p],
    ),
    "lsr_ns_noalloc_capacity": (c_size_t, []),
    "lsr_ns_bf16_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_float, c_float, c_void_p],
    ),
    "lsr_gemm_bf16": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p]),
    "lsr_gram_update_f32": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_float, c_void_p]),
    "lsr_kron_sum_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "lsr_kron_sum_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lsr_kron_sum_f32": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_kron_apply_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "lsr_kron_apply_bf16": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_kron_apply_f32": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_kron_dense_operator_f32": (
        c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "lsr_kron_dense_apply_workspace_bytes": (c_size_t, [c_int, c_int]),
    "lsr_kron_dense_apply_f32": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_kron_reconstruct_f32": (
        c_int, [ctypes.POINTER(c_void_p), ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_int, c_int, c_void_p,
                c_void_p]),
    "lsr_hawkes_dense_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "lsr_hawkes_kron_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                    c_int, c_int, c_void_p]),
    "lsr_pauli_apply_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_int, c_int, c_void_p]),
    "lsr_soap_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lsr_soap_direction_bf16": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
         c_float, c_float, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_shampoo_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lsr_shampoo_direction_bf16": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_int, c_void_p,
         c_size_t, c_void_p]),
    "lsr_blocks_gather_bf16": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "lsr_blocks_apply_bf16": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_float, c_float, c_void_p]),
    "lsr_blocks_apply_any": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_float, c_float, c_void_p]),
    "lsr_graft_tiles": (c_int, [c_int, c_int]),
    "lsr_shampoo_graft_prepare_bf16": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                c_float, c_int, c_void_p]),
    "lsr_shampoo_graft_scale_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lsr_gemm_f32_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "lsr_gemm_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p, c_size_t,
                             c_void_p]),
    "lsr_qr_workspace_bytes": (c_size_t, [c_int, c_int]),
    "lsr_householder_qr_f32": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_eigenbasis_refresh_workspace_bytes": (c_size_t, [c_int, c_int]),
    "lsr_eigenbasis_refresh_f32": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_coupled_newton_workspace_bytes": (c_size_t, [c_int, c_int]),
    "lsr_coupled_newton_f32": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float, c_int,
                c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lsr_ipc_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    "lsr_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "lsr_ipc_close": (c_int, [c_void_p]),
    "lsr_ipc_free": (c_int, [c_void_p]),
    "lsr_peer_push": (c_int, [c_void_p, c_size_t, ctypes.POINTER(ctypes.c_longlong), c_int, c_int, c_void_p]),
    "lsr_muon_workspace_bytes": (c_size_t, [ctypes.POINTER(MuonGroup), c_int]),
    "lsr_muon_step_bf16": (
        c_int,
        [ctypes.POINTER(MuonGroup), c_int, c_float, c_int, c_float, c_float, c_int, c_float, c_float, c_float,
         c_float, c_void_p, c_size_t, c_void_p],
    ),
    "lsr_muon_orthogonalize_bf16": (
        c_int,
        [ctypes.POINTER(MuonGroup), c_int, c_float, c_int, c_int, c_float, c_float, c_float, c_float,
         ctypes.POINTER(c_void_p), c_void_p, c_size_t, c_void_p],
    ),
    "lsr_muon_orthogonalize_phase_bf16": (
        c_int,
        [ctypes.POINTER(MuonGroup), c_int, c_float, c_int, c_int, c_float, c_float, c_float, c_float,
         ctypes.POINTER(c_void_p), c_int, c_void_p, c_size_t, c_void_p],
    ),
    "lsr_muon_apply_bf16": (
        c_int,
        [ctypes.POINTER(MuonGroup), c_int, ctypes.POINTER(c_void_p), c_float, c_float, c_void_p],
    ),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load liblsr.so (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("LSR_LIBRARY", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"liblsr.so not found at {path}; build it with `python cuda-lsr_b200/build.py` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != LSR_OK:
        msg = load().lsr_strerror(rc).decode()
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg} (liblsr code {rc})")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_get_device = getattr(torch._C, "_cuda_getDevice", None)


def stream_handle(device: torch.device | None = None) -> int:
    """cudaStream_t of torch's current stream on `device` (the current device when None or unindexed)."""
    if _raw_stream is None or _get_device is None:
        return torch.cuda.current_stream(device).cuda_stream
    idx = device.index if device is not None and device.index is not None else _get_device()
    return _raw_stream(idx)


def on_device(device: torch.device | int):
    """Context that makes `device` the current CUDA device; costs nothing when it already is."""
    if isinstance(device, int):
        device = torch.device("cuda", device)
    if device.index is None or (_get_device is not None and device.index == _get_device()):
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def device_status(clear: bool = True) -> int:
    """Device status word (0 = no device-side failure recorded). Synchronizes."""
    code = c_int(0)
    check(load().lsr_device_status(ctypes.byref(code), int(clear)), "lsr_device_status")
    return code.value


PROFILE_KINDS = ("ns_gram", "ns_poly", "ns_update", "orient", "normalize", "apply", "gemm_other", "ew_other",
                 "peer_push")


def launch_count() -> int:
    return int(load().lsr_launch_count())


def profile_enable(on: bool) -> None:
    check(load().lsr_profile_enable(int(on)), "lsr_profile_enable")


def profile_read(reset: bool = True) -> dict:
    """{kind: (total_ms, launches)} of the launches recorded while profiling was on."""
    n = len(PROFILE_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_longlong * n)()
    check(load().lsr_profile_read(ms, cnt, n, int(reset)), "lsr_profile_read")
    return {k: (ms[i], int(cnt[i])) for i, k in enumerate(PROFILE_KINDS)}


class Workspace:
    """Per-device scratch buffer, grown on demand (allocated through torch)."""

    def __init__(self) -> None:
        self._bufs: dict[int, torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            self._bufs.pop(idx, None)
            buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            self._bufs[idx] = buf
        return buf


WORKSPACE = Workspace()


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (liblsr has no CPU path)")
