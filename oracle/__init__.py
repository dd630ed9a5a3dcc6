"""CPU oracle for the optimizer hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms of cuda-lsr's
optimizer hot path so that the CUDA kernels of liblsr can be checked against
them. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may import it, and only as the checker; the product
path (the ``lsr`` package) never calls it and fails loudly when the CUDA
library is missing.

Pinning: the Newton–Schulz / Muon restatement is checked against golden
vectors produced by running the reference's own functions
(``muon_lm_ddp.zeropower_serial`` / ``zeropower_batched_oriented`` /
``MuonAdamW``) on CPU, stored in ``tests/golden/`` together with the script
that made them. The Kronecker apply restatement is pinned the same way against
``kron_apply_shared_2d`` (``hft.py:108-140``). The Shampoo / SOAP math lives in
the un-vendored ``distributed_shampoo`` package: that part is
**parity unpinned** (see ``oracle/shampoo.py``).
"""
