"""Stage the reference's own modules for the baselines — TEST INFRASTRUCTURE ONLY.

The reference implements its Muon path in Python / torch (muon_lm_ddp.py:296-696:
adjusted_muon_lr, zeropower_serial, zeropower_batched_oriented, MuonAdamW),
so there is nothing to compile, and its Kronecker-sum kernel
(kron_sum_64x8_kernel, hft_fused.py:89-319) is CUDA source that hft_fused.py
builds itself with torch's load_inline when imported on a GPU machine. The same holds
for kron_cuda.py, hft.py and pauli.py (tiny-factor reconstruction, Hawkes update and Pauli-string
apply: Triton kernels compiled by Triton on the GPU). This recipe copies those five modules, unmodified, from a cuda-lsr checkout into
``oracle/_ref/`` (git-ignored; it travels with the working tree to the machine
that runs the benchmark, where the checkout is absent) and records their
SHA-256 beside them:

    python oracle/stage_reference.py --reference <path of the cuda-lsr checkout>

``bench.py``'s reference arm and its ``cpu_baseline`` leg import the staged
Muon module and time the reference's own ``MuonAdamW.muon_step`` on the host
cores (``cpu_baseline.kind = "reference"``); without it they fall back to the
numpy restatement in ``oracle/muon.py`` (``kind = "port"``). ``bench.py
--workload kron64x8`` imports the staged hft_fused.py to time the reference's
kernel beside liblsr's on the same GPU, and ``--workload kronrec`` imports the staged
kron_cuda.py to time the reference's Triton tiny-factor reconstruction the same way;
``--workload hawkes`` and ``tests/test_gpu_hawkes.py`` run the Triton Hawkes kernels of the staged
hft.py (its function definitions only, ``load_functions``), and ``--workload pauli`` /
``tests/test_gpu_pauli.py`` the Triton Pauli-string kernels of the staged pauli.py. Nothing in the product (the ``lsr``
package) imports them.
"""
from __future__ import annotations

import argparse
import hashlib
import shutil
import sys
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref"
MODULE = "muon_lm_ddp.py"
MODULES = (MODULE, "hft_fused.py", "kron_cuda.py", "hft.py", "pauli.py")


def stage(reference: str | Path) -> Path | None:
    """Copy the reference's muon_lm_ddp.py and hft_fused.py into oracle/_ref/; returns the staged
    Muon module's path (None if the checkout has none)."""
    out = None
    for name in MODULES:
        src = Path(reference) / name
        if not src.is_file():
            continue
        REF_DIR.mkdir(exist_ok=True)
        dst = REF_DIR / name
        shutil.copyfile(src, dst)
        digest = hashlib.sha256(dst.read_bytes()).hexdigest()
        (REF_DIR / (name + ".sha256")).write_text(f"{digest}  {name}\n")
        if name == MODULE:
            out = dst
    return out


def staged_module_path(name: str = MODULE) -> Path | None:
    p = REF_DIR / name
    return p if p.is_file() else None


def load_functions(name: str, functions: list[str], env: dict) -> dict | None:
    """The named top-level function definitions (decorators included) of the staged module `name`,
    executed in `env` without the module's other top-level statements (hft.py runs its benchmarks
    at import, hft.py:821-825). None when the module is not staged."""
    import ast
    path = staged_module_path(name)
    if path is None:
        return None
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in functions]
    missing = set(functions) - {n.name for n in keep}
    if missing:
        raise RuntimeError(f"{name}: functions not found: {sorted(missing)}")
    ns = dict(env)
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(path), "exec"), ns)
    return {k: ns[k] for k in functions}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path of the cuda-lsr checkout")
    args = ap.parse_args(argv)
    out = stage(args.reference)
    if out is None:
        print(f"{MODULE} not found under {args.reference}", file=sys.stderr)
        return 1
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
