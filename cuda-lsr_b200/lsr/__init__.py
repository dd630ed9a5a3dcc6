"""lsr — B200 (sm_100a) optimizer hot path of cuda-lsr.

Drop-in Python surface over liblsr.so (include/lsr.h):

* ``lsr.muon``  — zeropower_serial / zeropower_batched_oriented /
  zeropower_via_newtonschulz5, MuonAdamW, Muon.

The CUDA library is loaded lazily on the first call; there is no CPU fallback.
"""
from . import _lib
from .muon import (NS_A, NS_B, NS_C, Muon, MuonAdamW, adjusted_muon_lr, zeropower_batched_oriented,
                   zeropower_serial, zeropower_via_newtonschulz5)

__version__ = "0.1.0"


def library_version() -> str:
    return _lib.load().lsr_version().decode()


__all__ = [
    "NS_A", "NS_B", "NS_C", "Muon", "MuonAdamW", "adjusted_muon_lr", "zeropower_batched_oriented",
    "zeropower_serial", "zeropower_via_newtonschulz5", "library_version",
]
