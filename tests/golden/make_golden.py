"""Generate the golden fixtures in this directory by running the REFERENCE's own
code on CPU (run where a cuda-lsr checkout is available):

    python tests/golden/make_golden.py --reference <path of the cuda-lsr checkout>

* muon_golden.npz   — muon_lm_ddp.zeropower_serial / zeropower_batched_oriented /
                      MuonAdamW.muon_step (imported unmodified; the module only
                      needs torch at import time).
* kron_golden.npz   — kron_apply_shared_2d of hft.py:108-140 and of
                      hft_fused.py:463-509. Both modules assert CUDA at import,
                      so the two function definitions are extracted from the
                      reference source with ``ast`` and executed on CPU tensors.
* kronrec_golden.npz — batched_kron / vectorized_kron of kron_cuda.py:117-145,
                      :618-629 on K = 5 / 4 / 3 factor sets (same extraction).
* driver_golden.json — the key list of the run summary, the parameter count and
                      the optimizer structure of the reference's recorded GPT-2-XL
                      Muon run (gpt2xl_4gpu_batched.json).
* newton_golden.npz — coupled_newton_one (+ matrix_power_small) of shampoo.py:254-347
                      (same extraction), and batched_coupled_newton (:408-542) on
                      SPD batches built as make_spd_batch (:178-247) builds them
                      (Gram / n, Frobenius norm sqrt(n), ridge 1e-2 with a 15%
                      tail at 1e-5): outputs, per-factor iteration counts and
                      final errors.

Inputs are seeded torch CPU draws; bf16 arrays are stored as uint16 bit
patterns, fp32 arrays as float32. The fixtures hold inputs and outputs, so the
tests never need the reference or torch's RNG to reproduce them.
"""
from __future__ import annotations

import argparse
import ast
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def extract_functions(path: Path, names: list[str], env: dict) -> dict:
    """Execute only the named top-level function definitions of a reference file."""
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in keep}
    if missing:
        raise RuntimeError(f"{path.name}: functions not found: {sorted(missing)}")
    mod = ast.Module(body=keep, type_ignores=[])
    ns = dict(env)
    exec(compile(mod, str(path), "exec"), ns)
    return {k: ns[k] for k in names}


def make_muon(ref: Path) -> dict:
    sys.path.insert(0, str(ref))
    import muon_lm_ddp as M  # noqa: E402  (reference module, unmodified)

    torch.set_num_threads(8)
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(1234)
    # zeropower_serial on wide, tall, square and ragged shapes
    serial_shapes = [(64, 256), (256, 64), (96, 96), (17, 33), (33, 17), (128, 512), (512, 128)]
    for i, (r, c) in enumerate(serial_shapes):
        G = (torch.randn(r, c, generator=g) * 0.02).to(torch.bfloat16)
        Y = M.zeropower_serial(G, ns_steps=5, eps=1e-7)
        out[f"serial{i}_in"] = bits(G)
        out[f"serial{i}_out"] = bits(Y)
    out["serial_shapes"] = np.array(serial_shapes, dtype=np.int64)
    # zeropower_batched_oriented on a [B, m, n] stack
    Xb = (torch.randn(3, 64, 192, generator=g) * 0.02).to(torch.bfloat16)
    Yb = M.zeropower_batched_oriented(Xb, ns_steps=5, eps=1e-7)
    out["batched_in"] = bits(Xb)
    out["batched_out"] = bits(Yb)
    # ns_steps variations
    G = (torch.randn(48, 160, generator=g) * 0.02).to(torch.bfloat16)
    for steps in (0, 1, 3):
        out[f"steps{steps}_out"] = bits(M.zeropower_serial(G, ns_steps=steps, eps=1e-7))
    out["steps_in"] = bits(G)
    # config-1 shape: one wide and one tall 768 x 3072 matrix, N(0, 0.02^2), seed 0
    g0 = torch.Generator().manual_seed(0)
    # (the inputs are regenerated from the seed by the tests; the fixture keeps
    # input checksums to detect an RNG change, plus output checksums and a slice)
    for name, (r, c) in (("cfg1_wide", (768, 3072)), ("cfg1_tall", (3072, 768))):
        G = (torch.randn(r, c, generator=g0) * 0.02).to(torch.bfloat16)
        Y = M.zeropower_serial(G, ns_steps=5, eps=1e-7).float().double()
        Gd = G.float().double()
        out[f"{name}_in_sums"] = np.array([Gd.sum().item(), (Gd * Gd).sum().item()])
        out[f"{name}_out_rows"] = bits(Y[:64])
        out[f"{name}_out_colsum"] = Y.sum(0).numpy()
        out[f"{name}_out_fro"] = np.array([Y.norm().item()])
    # adjusted_muon_lr
    lr_cases = [(0.02, (1600, 4800)), (0.02, (6400, 1600)), (0.02, (1600, 1600)), (0.01, (768, 3072))]
    out["lr_cases"] = np.array([[lr, s[0], s[1]] for lr, s in lr_cases], dtype=np.float64)
    out["lr_original"] = np.array([M.adjusted_muon_lr(lr, s, "original") for lr, s in lr_cases])
    out["lr_match"] = np.array([M.adjusted_muon_lr(lr, s, "match_rms_adamw") for lr, s in lr_cases])
    out["lr_none"] = np.array([M.adjusted_muon_lr(lr, s, "none") for lr, s in lr_cases])
    # MuonAdamW: two muon steps (batched and serial) on a toy parameter set
    shapes = [("h.0.attn.c_attn.weight", (64, 192)), ("h.0.attn.c_proj.weight", (64, 64)),
              ("h.0.mlp.c_fc.weight", (64, 256)), ("h.0.mlp.c_proj.weight", (256, 64)),
              ("h.1.mlp.c_fc.weight", (64, 256)), ("h.1.mlp.c_proj.weight", (256, 64)),
              ("wte.weight", (100, 64)), ("ln_f.bias", (64,))]
    init = {n: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16) for n, s in shapes}
    grads = [{n: (torch.randn(*s, generator=g) * 0.01).to(torch.bfloat16) for n, s in shapes} for _ in range(2)]
    for mode in ("batched", "serial"):
        params = {n: torch.nn.Parameter(t.clone()) for n, t in init.items()}
        opt = M.MuonAdamW(list(params.items()), muon_mode=mode, muon_lr=0.02, muon_momentum=0.95,
                          muon_weight_decay=0.01, muon_nesterov=True, muon_ns_steps=5, muon_eps=1e-7,
                          muon_lr_adjust="original", muon_batch_matrices=8, adam_lr=3e-4,
                          adam_betas=(0.9, 0.95), adam_weight_decay=0.1, rank=0)
        for step in range(2):
            for n, p in params.items():
                p.grad = grads[step][n].clone()
            opt.muon_step()
        for n, p in params.items():
            if p.ndim == 2 and "wte" not in n:
                out[f"muon_{mode}_{n}"] = bits(p.data)
                out[f"muon_{mode}_mom_{n}"] = bits(opt.momentum[p])
        if mode == "batched":
            summ = opt.summary()
            out["summary_muon_count"] = np.array([summ["muon_param_count"], summ["adam_param_count"],
                                                  summ["muon_matrix_count"]])
    for n, t in init.items():
        out[f"muon_init_{n}"] = bits(t)
        for step in range(2):
            out[f"muon_grad{step}_{n}"] = bits(grads[step][n])
    return out


def make_kron(ref: Path) -> dict:
    env = {"torch": torch, "math": math}
    hft = extract_functions(ref / "hft.py", ["kron_apply_shared_2d"], env)
    hff = extract_functions(ref / "hft_fused.py", ["kron_apply_shared_2d"], env)
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(4321)
    # general shared 2-D apply, Y = A X B^T (hft.py:108-140)
    for i, (M_, na, nf) in enumerate([(5, 32, 16), (3, 48, 40), (2, 128, 64)]):
        X = torch.randn(M_, na, nf, generator=g)
        A = torch.randn(na, na, generator=g) / math.sqrt(na)
        B = torch.randn(nf, nf, generator=g) / math.sqrt(nf)
        out[f"apply{i}_X"], out[f"apply{i}_A"], out[f"apply{i}_B"] = X.numpy(), A.numpy(), B.numpy()
        out[f"apply{i}_Y"] = hft["kron_apply_shared_2d"](X, A, B).numpy()
    # Kronecker sum (A (+) B) vec(X) = A X + X B^T via the S=2 term list (A, I), (I, B)
    for i, n in enumerate([32, 64]):
        X = torch.randn(4, n, n, generator=g)
        Mm = torch.randn(n, n, generator=g) / math.sqrt(n)
        A = (Mm + Mm.T) / 2
        Mm = torch.randn(n, n, generator=g) / math.sqrt(n)
        B = (Mm + Mm.T) / 2
        I = torch.eye(n)
        Y = hft["kron_apply_shared_2d"](X, A, I) + hft["kron_apply_shared_2d"](X, I, B)
        out[f"ksum{i}_X"], out[f"ksum{i}_A"], out[f"ksum{i}_B"], out[f"ksum{i}_Y"] = (
            X.numpy(), A.numpy(), B.numpy(), Y.numpy())
    # multi-term sum over S terms with the [M,64,8] shapes of hft_fused.py (torch factored path :655-669)
    for S in (1, 2, 4):
        X = torch.randn(6, 64, 8, generator=g)
        A = torch.randn(S, 64, 64, generator=g) / math.sqrt(64)
        B = torch.randn(S, 8, 8, generator=g) / math.sqrt(8)
        Y = torch.zeros_like(X)
        for s in range(S):
            Y.add_(hff["kron_apply_shared_2d"](X, A[s], B[s]))
        W = torch.zeros(512, 512)
        for s in range(S):
            W.add_(torch.kron(A[s], B[s]))
        out[f"multi{S}_X"], out[f"multi{S}_A"], out[f"multi{S}_B"], out[f"multi{S}_Y"] = (
            X.numpy(), A.numpy(), B.numpy(), Y.numpy())
        out[f"multi{S}_Ydense"] = (X.reshape(6, 512) @ W.T).reshape(6, 64, 8).numpy()
    return out


def make_newton(ref: Path) -> dict:
    env = {"torch": torch, "math": math}
    fns = extract_functions(ref / "shampoo.py", ["matrix_power_small", "coupled_newton_one"], env)
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(999)
    for i, n in enumerate([16, 48]):
        Q, _ = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))
        eig = torch.logspace(-1, 1, n, dtype=torch.float64)
        A = (Q @ torch.diag(eig) @ Q.T).float()
        out[f"newton{i}_A"] = A.numpy()
        for root in (2, 4):
            res = fns["coupled_newton_one"](A, root=root)
            X = res[0] if isinstance(res, tuple) else res
            out[f"newton{i}_root{root}"] = X.numpy()
    # batched, per-factor convergence mask
    env_b = {"torch": torch, "math": math, "DEV": "cpu"}
    fb = extract_functions(ref / "shampoo.py", ["matrix_power_small", "coupled_newton_one", "batched_coupled_newton"],
                           env_b)
    for j, (n, B, roots) in enumerate([(48, 7, (2, 4)), (96, 2, (4,))]):
        g = torch.Generator().manual_seed(2024 + j)
        Xr = torch.randn(B, n, n, generator=g)
        A = Xr @ Xr.transpose(-1, -2) / float(n)
        A = A / A.flatten(1).norm(dim=1).clamp_min(1e-12)[:, None, None] * math.sqrt(n)
        ridge = torch.full((B,), 1e-2)
        ridge[-max(1, int(round(B * 0.15))):] = 1e-5
        A = (A + ridge[:, None, None] * torch.eye(n)).contiguous()
        out[f"nbatch{j}_A"] = A.numpy()
        for root in roots:
            X, iters, err = fb["batched_coupled_newton"](A, root=root)
            out[f"nbatch{j}_root{root}_X"] = X.numpy()
            out[f"nbatch{j}_root{root}_iters"] = iters.numpy()
            out[f"nbatch{j}_root{root}_err"] = err.numpy()
            out[f"nbatch{j}_root{root}_iters_one"] = np.array(
                [fb["coupled_newton_one"](A[b], root=root)[1] for b in range(B)], dtype=np.int32)
    return out


def make_kronrec(ref: Path) -> dict:
    """Tiny-factor Kronecker reconstruction (kron_cuda.py:117-145, :618-629): K = 5 factors of
    shapes [S,1,3], [S,2,4] x 4 and the exactly merged K = 4 / K = 3 sets built with the
    reference's batched_kron; W = vectorized_kron(factors) = sum_s kron(...)."""
    env = {"torch": torch, "math": math}
    fns = extract_functions(ref / "kron_cuda.py", ["batched_kron", "vectorized_kron"], env)
    bk, vk = fns["batched_kron"], fns["vectorized_kron"]
    out: dict[str, np.ndarray] = {}
    for S in (1, 7, 64):
        g = torch.Generator().manual_seed(17 + S)
        f = [0.5 * torch.randn(S, *shape, generator=g) for shape in [(1, 3), (2, 4), (2, 4), (2, 4), (2, 4)]]
        g01 = bk(f[0], f[1])
        g012 = bk(g01, f[2])
        sets = {5: f, 4: [g01, f[2], f[3], f[4]], 3: [g012, f[3], f[4]]}
        for K, fs in sets.items():
            for i, t in enumerate(fs):
                out[f"S{S}_K{K}_f{i}"] = t.numpy()
            out[f"S{S}_K{K}_W"] = vk(fs).numpy()
    return out


def make_driver(ref: Path) -> dict:
    """The run-summary schema and GPT-2-XL optimizer structure of the reference's own recorded
    run (gpt2xl_4gpu_batched.json, written by muon_lm_ddp.py:1539-1634): the summary's key order,
    the model's parameter count and MuonAdamW.summary() (muon_lm_ddp.py:700-745)."""
    import json
    run = json.loads((ref / "gpt2xl_4gpu_batched.json").read_text())
    return {"summary_keys": list(run.keys()), "model_params": run["model_params"],
            "optimizer_structure": run["optimizer_structure"]}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the cuda-lsr checkout")
    ap.add_argument("--only", choices=["muon", "kron", "newton", "kronrec", "driver"], default=None)
    args = ap.parse_args()
    ref = Path(args.reference)
    if args.only in (None, "muon"):
        np.savez_compressed(HERE / "muon_golden.npz", **make_muon(ref))
    if args.only in (None, "kron"):
        np.savez_compressed(HERE / "kron_golden.npz", **make_kron(ref))
    if args.only in (None, "newton"):
        np.savez_compressed(HERE / "newton_golden.npz", **make_newton(ref))
    if args.only in (None, "kronrec"):
        np.savez_compressed(HERE / "kronrec_golden.npz", **make_kronrec(ref))
    if args.only in (None, "driver"):
        import json
        (HERE / "driver_golden.json").write_text(json.dumps(make_driver(ref), indent=1) + "\n")
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
