"""GPU (one device): lsr_peer_push stores a byte range at every listed
distance, including the unaligned head and tail of ranges that do not start
or end on a 16-byte boundary, and touches nothing outside the range. The
"peers" are ordinary local buffers here; the kernel only sees addresses."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [2, 14, 30, 4102, 1 << 20, (3 << 20) + 10])
@pytest.mark.parametrize("offset", [0, 2, 6, 14])
@pytest.mark.parametrize("npeers", [1, 3, 7])
def test_push_copies_exact_range(nbytes, offset, npeers):
    from lsr import _lib as L
    lib = L.load()
    size = nbytes + 64
    g = torch.Generator(device="cuda").manual_seed(nbytes + offset + npeers)
    src = torch.randint(0, 256, (size,), dtype=torch.uint8, device="cuda", generator=g)
    dsts = [torch.full((size,), 0xA5, dtype=torch.uint8, device="cuda") for _ in range(npeers)]
    deltas = (ctypes.c_longlong * npeers)(*[d.data_ptr() - src.data_ptr() for d in dsts])
    assert all(v % 16 == 0 for v in deltas)
    L.check(lib.lsr_peer_push(src.data_ptr() + offset, nbytes, deltas, npeers, 0, L.stream_handle()),
            "lsr_peer_push")
    torch.cuda.synchronize()
    for d in dsts:
        assert torch.equal(d[offset:offset + nbytes], src[offset:offset + nbytes])
        assert bool((d[:offset] == 0xA5).all()) and bool((d[offset + nbytes:] == 0xA5).all())
    assert L.device_status() == 0


def test_push_argument_checks():
    from lsr import _lib as L
    lib = L.load()
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    d = (ctypes.c_longlong * 1)(16)
    assert lib.lsr_peer_push(buf.data_ptr(), 3, d, 1, 0, None) == -1      # odd byte count
    assert lib.lsr_peer_push(buf.data_ptr() + 1, 2, d, 1, 0, None) == -1  # odd address
    d8 = (ctypes.c_longlong * 1)(8)
    assert lib.lsr_peer_push(buf.data_ptr(), 2, d8, 1, 0, None) == -1     # distance not a multiple of 16
    assert lib.lsr_peer_push(buf.data_ptr(), 2, d, 16, 0, None) == -1     # more peers than supported
    assert lib.lsr_peer_push(buf.data_ptr(), 0, d, 1, 0, None) == 0       # empty range
