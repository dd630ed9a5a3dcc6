"""GPU: the allocation-free Newton–Schulz entry point.

lsr_ns_bf16_noalloc exists for callers that cannot allocate device memory
themselves (their device memory belongs to another allocator, or they cannot
afford the synchronisation cudaMalloc/cudaFree may cause); it keeps its
scratch in a fixed array inside the library. It runs the same kernels as
lsr_ns_bf16 with a caller workspace, and those kernels are deterministic, so
its output must be bit-identical to lsr_ns_bf16's, call after call, although
every call reuses (and leaves behind) the same scratch contents; a leak of a
previous call's scratch into a later one would break that equality. The
result is also checked against the oracle within the Newton–Schulz tolerance.

This file sorts last so that a failure here comes after every other test has
run; it also passes when run alone in a fresh process.
"""
import pytest
import torch

from oracle import muon as om
from oracle.bf16 import rel_fro

pytestmark = pytest.mark.gpu

TOL = 2e-2  # relative Frobenius tolerance used by the Newton–Schulz parity tests


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def _with_workspace(lib, L, X, rows, cols, orient):
    out = torch.empty_like(X)
    nb = lib.lsr_ns_workspace_bytes(1, rows, cols, orient)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    L.check(lib.lsr_ns_bf16(X.data_ptr(), out.data_ptr(), 1, rows, cols, orient, 5, 3.4445, -4.7750, 2.0315, 1e-7,
                            ws.data_ptr(), nb, L.stream_handle()), "lsr_ns_bf16")
    return out


def _no_alloc(lib, L, X, rows, cols, orient):
    out = torch.empty_like(X)
    L.check(lib.lsr_ns_bf16_noalloc(X.data_ptr(), out.data_ptr(), 1, rows, cols, orient, 5, 3.4445, -4.7750,
                                    2.0315, 1e-7, L.stream_handle()), "lsr_ns_bf16_noalloc")
    return out


def test_noalloc_matches_workspace_entry_point_twice():
    from lsr import _lib as L
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(11)
    cases = [(256, 1024), (1024, 384)]  # a wide then a tall matrix: the second call meets the first's leftovers
    for rows, cols in cases:
        assert lib.lsr_ns_workspace_bytes(1, rows, cols, 1) <= lib.lsr_ns_noalloc_capacity()
        X = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).bfloat16()
        got = _no_alloc(lib, L, X, rows, cols, 1)
        ref = _with_workspace(lib, L, X, rows, cols, 1)
        torch.cuda.synchronize()
        assert got.shape == ref.shape
        assert torch.equal(got, ref), (rows, cols, _rel(got.float(), ref.float()))
        err = rel_fro(got.float().cpu().numpy(), om.zeropower(X.float().cpu().numpy(), 5, 1e-7))
        assert err < TOL, (rows, cols, err)
    assert L.device_status() == 0


def test_noalloc_rejects_problems_beyond_capacity():
    from lsr import _lib as L
    lib = L.load()
    big_rows, big_cols = 4096, 8192
    assert lib.lsr_ns_workspace_bytes(1, big_rows, big_cols, 1) > lib.lsr_ns_noalloc_capacity()
    X = torch.zeros(1, dtype=torch.bfloat16, device="cuda")  # never read: the size check comes first
    rc = lib.lsr_ns_bf16_noalloc(X.data_ptr(), X.data_ptr(), 1, big_rows, big_cols, 1, 5, 3.4445, -4.7750, 2.0315,
                                 1e-7, L.stream_handle())
    assert rc == -7
    assert b"capacity" in lib.lsr_strerror(rc)
