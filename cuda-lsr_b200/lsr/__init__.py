"""lsr — B200 (sm_100a) optimizer hot path of cuda-lsr.

Drop-in Python surface over liblsr.so (include/lsr.h):

* ``lsr.muon``  — zeropower_serial / zeropower_batched_oriented /
  zeropower_via_newtonschulz5, MuonAdamW, Muon.
* ``lsr.kron``, ``lsr.shampoo`` — Kronecker sum / apply, Shampoo / SOAP.
* ``lsr.newton`` — coupled Newton inverse roots (coupled_newton_one,
  per_factor / batched / hybrid_coupled_newton).
* ``lsr.dist``  — ShardedMuon across the GPUs of one node.
* ``lsr.hawkes`` — multivariate Hawkes event update (hawkes_dense / hawkes_kron).
* ``lsr.lm_driver`` — the language-model driver with the reference's command line.

The CUDA library is loaded lazily on the first call; there is no CPU fallback.
"""
from . import _lib
from .muon import (NS_A, NS_B, NS_C, Muon, MuonAdamW, adjusted_muon_lr, zeropower_batched_oriented,
                   zeropower_serial, zeropower_via_newtonschulz5)
from .newton import (batched_coupled_newton, coupled_newton_one, hybrid_coupled_newton,
                     per_factor_coupled_newton)

__version__ = "0.1.0"


def library_version() -> str:
    return _lib.load().lsr_version().decode()


__all__ = [
    "NS_A", "NS_B", "NS_C", "Muon", "MuonAdamW", "adjusted_muon_lr", "zeropower_batched_oriented",
    "zeropower_serial", "zeropower_via_newtonschulz5", "library_version", "batched_coupled_newton",
    "coupled_newton_one", "hybrid_coupled_newton", "per_factor_coupled_newton",
]
