"""Kronecker operators on B200 (drop-ins for hft_fused.py / hft.py).

* ``kron_sum(A, X, B)``            (A ⊕ B) vec(X) = vec(A X + X B^T), one fused kernel
* ``kron_apply(X, A, B)``          Σ_s A_s X B_s^T  (A [S,m,m] or [m,m], B [S,n,n] or [n,n])
* ``kron_apply_shared_2d(X, A, B)`` A X B^T per snapshot            hft.py:108-140
* ``native_reconstruct(factors, K, out)``  W = Σ_s F_0[s] ⊗ ... ⊗ F_{K-1}[s]   kron_cuda.py:516-583
* ``kron_sum_out(x, at, b, out)``  out[m] = Σ_s A_s x[m] B_s^T with at[s] = A_s^T,
                                   same checks and errors as hft_fused.py:247-319
                                   (sizes generalised beyond [M,64,8] and S in {1,2,4,8})

fp32 inputs run the 3xTF32 tensor-core kernels (fp32-level accuracy); bf16
inputs run the bf16 kernels (fp32 accumulation). Outputs are fp32.
"""
from __future__ import annotations

import torch

from . import _lib


def _check(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if t.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError(f"{name} must be float32 or bfloat16")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _as3(X: torch.Tensor) -> torch.Tensor:
    if X.dim() == 2:
        return X.unsqueeze(0)
    if X.dim() != 3:
        raise RuntimeError("X must be [m, n] or [batch, m, n]")
    return X


def kron_sum(A: torch.Tensor, X: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """(A ⊕ B) vec(X) = vec(A X + X B^T) for X [m, n] or [batch, m, n]; returns fp32."""
    for t, nm in ((A, "A"), (X, "X"), (B, "B")):
        _check(t, nm)
    X3 = _as3(X)
    batch, m, n = X3.shape
    if A.shape != (m, m) or B.shape != (n, n):
        raise RuntimeError(f"A must be [{m},{m}] and B [{n},{n}]")
    if not (A.dtype == X.dtype == B.dtype):
        raise RuntimeError("A, X and B must share a dtype")
    Y = out if out is not None else torch.empty(X3.shape, dtype=torch.float32, device=X.device)
    if Y.dtype != torch.float32 or not Y.is_contiguous() or Y.numel() != X3.numel():
        raise RuntimeError("out must be a contiguous float32 tensor shaped like X")
    lib = _lib.load()
    with _lib.on_device(X.device):
        st = _lib.stream_handle(X.device)
        if X.dtype == torch.bfloat16:
            rc = lib.lsr_kron_sum_bf16(A.data_ptr(), X3.data_ptr(), B.data_ptr(), Y.data_ptr(), batch, m, n, st)
        else:
            nb = lib.lsr_kron_sum_workspace_bytes(batch, m, n, 1)
            ws = _lib.WORKSPACE.get(nb, X.device)
            rc = lib.lsr_kron_sum_f32(A.data_ptr(), X3.data_ptr(), B.data_ptr(), Y.data_ptr(), batch, m, n,
                                      ws.data_ptr(), nb, st)
    _lib.check(rc, "lsr_kron_sum")
    return Y.view(X.shape) if out is None else out


# Dense operators of small fp32 factors, W = sum_s A_s (x) B_s as a tf32 pair, kept per factor
# tensors (identity, version counter, shape): applying the same factors again skips forming W.
_DENSE_CACHE: dict = {}
_DENSE_MAX_MN = 1024


def _dense_operator(A3, B3, a_trans: bool):
    m, n, S = A3.shape[1], B3.shape[1], A3.shape[0]
    key = (A3.data_ptr(), A3._version, B3.data_ptr(), B3._version, a_trans, m, n, S, A3.device.index)
    hit = _DENSE_CACHE.get(key)
    if hit is not None:
        return hit
    if len(_DENSE_CACHE) >= 8:
        _DENSE_CACHE.clear()
    mn = m * n
    Wh = torch.empty(mn, mn, dtype=torch.float32, device=A3.device)
    Wl = torch.empty_like(Wh)
    lib = _lib.load()
    _lib.check(lib.lsr_kron_dense_operator_f32(A3.data_ptr(), int(a_trans), B3.data_ptr(), m, n, S, Wh.data_ptr(),
                                               Wl.data_ptr(), _lib.stream_handle(A3.device)),
               "lsr_kron_dense_operator_f32")
    _DENSE_CACHE[key] = (Wh, Wl, A3, B3)  # the factors are held so their addresses stay theirs
    return _DENSE_CACHE[key]


# Workspace bytes of lsr_kron_apply per (batch, m, n, S, fp32): a function of the sizes only
# (0 selects the small-problem path), looked up once per shape instead of once per call.
_WS_BYTES: dict = {}


def _kron_apply(X3, A3, B3, a_trans: bool, Y) -> None:
    batch, m, n = X3.shape
    S = A3.shape[0]
    f32 = X3.dtype == torch.float32
    lib = _lib.load()
    key = (batch, m, n, S, f32)
    nb = _WS_BYTES.get(key)
    if nb is None:
        nb = lib.lsr_kron_apply_workspace_bytes(batch, m, n, S, int(f32))
        if len(_WS_BYTES) >= 256:
            _WS_BYTES.clear()
        _WS_BYTES[key] = nb
    if f32 and nb == 0:  # small problem: one FFMA launch inside liblsr, no workspace
        dev = X3.device
        with _lib.on_device(dev):
            rc = lib.lsr_kron_apply_f32(A3.data_ptr(), int(a_trans), X3.data_ptr(), B3.data_ptr(), Y.data_ptr(),
                                        batch, m, n, S, None, 0, _lib.stream_handle(dev))
        if rc:
            _lib.check(rc, "lsr_kron_apply")
        return
    if f32 and m * n <= _DENSE_MAX_MN and (m * n) % 4 == 0:
        with _lib.on_device(X3.device):
            Wh, Wl, _, _ = _dense_operator(A3, B3, a_trans)
            nb = lib.lsr_kron_dense_apply_workspace_bytes(batch, m * n)
            ws = _lib.WORKSPACE.get(nb, X3.device)
            _lib.check(lib.lsr_kron_dense_apply_f32(Wh.data_ptr(), Wl.data_ptr(), X3.data_ptr(), Y.data_ptr(), batch,
                                                    m * n, ws.data_ptr(), nb, _lib.stream_handle(X3.device)),
                       "lsr_kron_dense_apply_f32")
        return
    with _lib.on_device(X3.device):
        ws = _lib.WORKSPACE.get(nb, X3.device)
        fn = lib.lsr_kron_apply_f32 if f32 else lib.lsr_kron_apply_bf16
        rc = fn(A3.data_ptr(), int(a_trans), X3.data_ptr(), B3.data_ptr(), Y.data_ptr(), batch, m, n, S,
                ws.data_ptr(), nb, _lib.stream_handle(X3.device))
    _lib.check(rc, "lsr_kron_apply")


def kron_apply(X: torch.Tensor, A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Σ_s A_s X B_s^T for X [m, n] or [batch, m, n]; A [S,m,m] or [m,m], B [S,n,n] or [n,n]; fp32 out."""
    for t, nm in ((A, "A"), (X, "X"), (B, "B")):
        _check(t, nm)
    X3 = _as3(X)
    A3 = A if A.dim() == 3 else A.unsqueeze(0)
    B3 = B if B.dim() == 3 else B.unsqueeze(0)
    batch, m, n = X3.shape
    if A3.shape[1:] != (m, m) or B3.shape[1:] != (n, n) or A3.shape[0] != B3.shape[0]:
        raise RuntimeError("A must be [S,m,m] and B [S,n,n] with the same S")
    if not (A.dtype == X.dtype == B.dtype):
        raise RuntimeError("A, X and B must share a dtype")
    Y = torch.empty(X3.shape, dtype=torch.float32, device=X.device)
    _kron_apply(X3, A3.contiguous(), B3.contiguous(), False, Y)
    return Y.view(X.shape)


def kron_apply_shared_2d(X: torch.Tensor, A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """A X B^T for X [M, na, nf] (hft.py:108-140), without materialising kron(A, B)."""
    return kron_apply(X, A, B)


def kron_sum_out(x: torch.Tensor, at: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> None:
    """out[m] = Σ_s A_s x[m] B_s^T with at[s] = A_s^T (hft_fused.py:247-319 semantics)."""
    for t, nm in ((x, "x"), (at, "at"), (b, "b"), (out, "out")):
        if not t.is_cuda:
            raise RuntimeError(f"{nm} must be CUDA")
        if t.dtype != torch.float32:
            raise RuntimeError(f"{nm} must be float32")
        if not t.is_contiguous():
            raise RuntimeError(f"{nm} must be contiguous")
    if x.dim() != 3:
        raise RuntimeError("x must have shape [M,na,nf]")
    M, na, nf = x.shape
    if at.dim() != 3 or at.shape[1:] != (na, na):
        raise RuntimeError(f"at must have shape [S,{na},{na}]")
    S = at.shape[0]
    if b.dim() != 3 or b.shape != (S, nf, nf):
        raise RuntimeError(f"b must have shape [S,{nf},{nf}]")
    if out.shape != x.shape:
        raise RuntimeError("out must match x shape")
    if S < 1:
        raise RuntimeError(f"Supported S values are >= 1; got {S}")
    _kron_apply(x, at, b, True, out)


def native_reconstruct(factors, K, out=None, block=256):
    """W = Σ_s factors[0][s] ⊗ ... ⊗ factors[K-1][s] (kron_cuda.py:516-583; ``block`` is accepted
    and ignored). factors: K fp32 CUDA tensors [S, r_k, c_k]; out: [Π r_k, Π c_k] fp32 or None."""
    import ctypes
    if len(factors) != K:
        raise ValueError(K)
    if not 1 <= K <= 8:
        raise ValueError(K)
    S = factors[0].shape[0]
    rows, cols = [], []
    for f in factors:
        if not (f.is_cuda and f.dtype == torch.float32 and f.dim() == 3 and f.is_contiguous()) or f.shape[0] != S:
            _check(f, "factor")  # the CUDA / dtype / layout message first, as for any operand
            raise RuntimeError("factors must be float32 [S, r, c] with a common S")
        _, r, c = f.shape
        rows.append(r)
        cols.append(c)
    R = 1
    C = 1
    for r, c in zip(rows, cols):
        R *= r
        C *= c
    if out is None:
        out = torch.empty(R, C, dtype=torch.float32, device=factors[0].device)
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != R * C:
        raise RuntimeError(f"out must be a contiguous float32 tensor with {R}x{C} elements")
    key = (tuple(f.data_ptr() for f in factors), tuple(rows), tuple(cols))
    arrs = _RECON_ARGS.get(key)
    if arrs is None:  # the factor address and shape arrays, built once per factor set
        arrs = ((ctypes.c_void_p * K)(*key[0]), (ctypes.c_int * K)(*rows), (ctypes.c_int * K)(*cols))
        if len(_RECON_ARGS) >= 64:
            _RECON_ARGS.clear()
        _RECON_ARGS[key] = arrs
    lib = _lib.load()
    dev = out.device
    with _lib.on_device(dev):
        rc = lib.lsr_kron_reconstruct_f32(arrs[0], arrs[1], arrs[2], K, S, out.data_ptr(), _lib.stream_handle(dev))
    if rc:
        _lib.check(rc, "lsr_kron_reconstruct_f32")
    return out


# ctypes argument arrays of native_reconstruct per (factor addresses, row counts, column counts).
_RECON_ARGS: dict = {}
