#!/usr/bin/env python
"""Benchmark: full GPT-2-XL Muon optimizer step on 1..8 B200 GPUs.

Workload (the reference's headline Muon step, muon_lm_ddp.py:615-696, on its
GPT-2-XL parameter set gpt2xl_4gpu_*.json:26-73): 48 layers x {1600x4800,
1600x1600, 1600x6400, 6400x1600} = 192 bf16 matrices (1.4746 B parameters).
One step = Nesterov momentum update + 5-step quintic Newton–Schulz of every
matrix + decoupled weight decay and the lr-adjusted update (lr 0.02, wd 0.01,
momentum 0.95, "original" lr adjust). Gradients / momentum N(0, 0.01^2) and
parameters N(0, 0.02^2), bf16, seeded (seed 4) on the device.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lsr|reference]

N > 1 is launched with torch.distributed.run: the matrices of each shape group
are sharded round-robin over the ranks (ZeRO-1), the orthogonalised updates are
all-gathered with NCCL and applied on every rank (total work fixed: strong
scaling). ``--impl reference`` times the reference's own Muon step
(muon_lm_ddp.MuonAdamW.muon_step, torch on the host cores, the module staged
unmodified in oracle/_ref/ by oracle/stage_reference.py; the numpy
restatement in oracle/muon.py when it is not staged) on a bounded sample, one
of the 48 layers per step, extrapolated to the full step.

Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "cuda-lsr_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

LAYER_SHAPES = [(1600, 4800), (1600, 1600), (1600, 6400), (6400, 1600)]  # c_attn, attn.c_proj, mlp.c_fc, mlp.c_proj
N_LAYERS = 48
NS_STEPS = 5
LR, MU, WD, EPS = 0.02, 0.95, 0.01, 1e-7
METRIC = "GPT-2-XL Muon optimizer step ms at 1/2/4/8 B200; % of dense bf16 TC peak"
BASELINE_MS = 369.40  # gpt2xl_4gpu_batched.json:20 (4x RTX PRO 6000, Muon replicated)
WORKLOAD = ("gpt2-xl muon step: 192 bf16 matrices (48 x {1600x4800, 1600x1600, 1600x6400, 6400x1600}), "
            "nesterov momentum 0.95 + 5 Newton-Schulz steps + apply (lr 0.02, wd 0.01)")


def ns_dense_flops(shape, steps=NS_STEPS) -> float:
    m, n = min(shape), max(shape)
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)


def phase_flops(shapes) -> dict:
    """Dense (algorithmic) flops of one launch of each NS phase over all matrices."""
    out = {"ns_gram": 0.0, "ns_poly": 0.0, "ns_update": 0.0}
    for s in shapes:
        m, n = min(s), max(s)
        out["ns_gram"] += 2.0 * m * m * n
        out["ns_poly"] += 2.0 * m ** 3
        out["ns_update"] += 2.0 * m * m * n
    return out


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                    "hbm_gbs": d["hbm_gbs"], "source": "measured"}
        except Exception:
            pass
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons)}


def physical_gpu(local_rank: int) -> int:
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        toks = [t.strip() for t in cvd.split(",") if t.strip()]
        if local_rank < len(toks) and toks[local_rank].isdigit():
            return int(toks[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# CPU side: oracle restatement of the reference path (bounded sample)
# ---------------------------------------------------------------------------

def cpu_layer_step_ms(seed: int = 4) -> float:
    """Time one layer's Muon step (4 matrices) through the numpy oracle; returns ms."""
    from oracle import muon as om
    from oracle.bf16 import round_bf16
    rng = np.random.default_rng(seed)
    P = [round_bf16(rng.standard_normal(s, dtype=np.float32) * 0.02) for s in LAYER_SHAPES]
    G = [round_bf16(rng.standard_normal(s, dtype=np.float32) * 0.01) for s in LAYER_SHAPES]
    M = [round_bf16(rng.standard_normal(s, dtype=np.float32) * 0.01) for s in LAYER_SHAPES]
    t0 = time.perf_counter()
    om.muon_step(P, G, M, lr=LR, mu=MU, nesterov=True, wd=WD, ns_steps=NS_STEPS, eps=EPS)
    return (time.perf_counter() - t0) * 1e3


def load_reference_module(name: str = "muon_lm_ddp"):
    """The reference's own module `name` as staged in oracle/_ref/ (None when not staged)."""
    from oracle import stage_reference
    path = stage_reference.staged_module_path(name + ".py")
    if path is None:
        return None
    import importlib.util
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class ReferenceLayerStep:
    """One layer's Muon step (c_attn 1600x4800, attn.c_proj 1600x1600, mlp.c_fc 1600x6400,
    mlp.c_proj 6400x1600) through the reference's own MuonAdamW.muon_step on CPU tensors,
    with the benchmark's hyper-parameters (muon_lm_ddp.py:433-696, batched mode, chunks of 8)."""

    def __init__(self, mod, seed: int = 4):
        g = torch.Generator().manual_seed(seed)
        self.params = [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16()) for s in LAYER_SHAPES]
        named = [(f"transformer.h.0.w{i}", p) for i, p in enumerate(self.params)]
        self.opt = mod.MuonAdamW(named, "batched", LR, MU, WD, True, NS_STEPS, EPS, "original", 8, 3e-4,
                                 (0.9, 0.95), 0.0, 0)
        for p in self.params:
            self.opt.momentum[p].copy_((torch.randn(*p.shape, generator=g) * 0.01).bfloat16())
            p.grad = (torch.randn(*p.shape, generator=g) * 0.01).bfloat16()

    def __call__(self) -> float:
        t0 = time.perf_counter()
        self.opt.muon_step()
        return (time.perf_counter() - t0) * 1e3


def cpu_baseline_sampler():
    """(callable returning one layer's step ms, kind, description) for the CPU baseline: the reference's
    own torch code when staged in oracle/_ref/, else the numpy restatement of it."""
    mod = load_reference_module()
    if mod is not None:
        torch.set_num_threads(os.cpu_count() or 1)
        step = ReferenceLayerStep(mod)
        return step, "reference", (f"muon_lm_ddp.MuonAdamW.muon_step (the reference module, unmodified, "
                                   f"torch on {torch.get_num_threads()} CPU threads) on 1 of 48 layers "
                                   f"(4 matrices 1600x4800, 1600x1600, 1600x6400, 6400x1600), extrapolated x48")
    return cpu_layer_step_ms, "port", ("1 of 48 layers (4 matrices 1600x4800, 1600x1600, 1600x6400, 6400x1600), "
                                       "full Muon step (momentum, 5 NS steps, apply) through the numpy "
                                       "restatement of the reference, extrapolated x48")


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    fn, kind, desc = cpu_baseline_sampler()
    cores = torch.get_num_threads() if kind == "reference" else (os.cpu_count() or 1)
    for _ in range(args.warmup):
        fn()
    samples = [fn() for _ in range(args.steps)]
    layer_ms = statistics.median(samples)
    value = layer_ms * N_LAYERS
    sample = f"{desc}; median of {args.steps} one-layer samples"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": round(value / BASELINE_MS, 4), "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.01^2) grads/momentum, N(0,0.02^2) params)",
        "config": {"workload": WORKLOAD, "parallelism": "host cores", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "ms", "cores": cores, "kind": kind, "sample": sample,
                         "extrapolated": {"from": "1 layer of 48", "factor": N_LAYERS,
                                          "layer_ms_median": round(layer_ms, 3),
                                          "timed_wall_s": round(sum(samples) / 1e3, 2)}},
        "e2e": {"value": round(value, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

def make_params(device, layers: int):
    g = torch.Generator(device=device).manual_seed(4)
    shapes = [s for _ in range(layers) for s in LAYER_SHAPES]
    P = [(torch.randn(s, generator=g, device=device) * 0.02).bfloat16() for s in shapes]
    G = [(torch.randn(s, generator=g, device=device) * 0.01).bfloat16() for s in shapes]
    M = [(torch.randn(s, generator=g, device=device) * 0.01).bfloat16() for s in shapes]
    return shapes, P, G, M


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def run_lsr(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    import lsr
    from lsr import _lib
    from lsr.dist import ShardedMuon

    shapes, P, G, M = make_params(dev, args.layers)
    params = [torch.nn.Parameter(p) for p in P]
    named = [(f"h.{i // 4}.w{i % 4}", p) for i, p in enumerate(params)]

    if world == 1:
        opt = lsr.MuonAdamW(named, muon_mode="batched", muon_lr=LR, muon_momentum=MU, muon_weight_decay=WD,
                            muon_nesterov=True, muon_ns_steps=NS_STEPS, muon_eps=EPS, muon_lr_adjust="original",
                            muon_batch_matrices=8, adam_lr=3e-4, adam_betas=(0.9, 0.95), adam_weight_decay=0.0,
                            rank=0)
        for p, m in zip(params, M):
            opt.momentum[p].copy_(m)
        step = opt.muon_step
    else:
        opt = ShardedMuon(params, lr=LR, momentum=MU, nesterov=True, weight_decay=WD, ns_steps=NS_STEPS, eps=EPS,
                          flat_params=True, exchange=args.exchange)
        for Gp in opt.groups:
            for k, j in enumerate(Gp.owned):
                idx = next(i for i, p in enumerate(params) if p is Gp.params[j])
                Gp.momentum[k].copy_(M[idx])
        step = opt.step
    for p, gr in zip(params, G):
        p.grad = gr
    del M

    # ---------------------------------------------------------------- device-timed
    with _nvtx("muon.warmup"):
        for _ in range(args.warmup):
            step()
    barrier(world)
    sampler = ClockSampler(physical_gpu(local_rank))
    sampler.start()
    time.sleep(0.3)
    _lib.profile_enable(True)
    _lib.profile_read(reset=True)
    launches0 = _lib.launch_count()
    barrier(world)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    with _nvtx("muon.steps"):
        for _ in range(args.steps):
            step()
    t_end.record()
    barrier(world)
    launches = _lib.launch_count() - launches0
    _lib.profile_enable(False)
    prof = _lib.profile_read(reset=True)
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    ms = max_over_ranks(ms, world)

    peaks = measured_peaks()
    # dominant kernel: the NS launch kind with the largest total time
    ns_kinds = ("ns_gram", "ns_poly", "ns_update")
    dom = max(ns_kinds, key=lambda k: prof[k][0])
    dom_ms, dom_n = prof[dom]
    my_shapes = shapes if world == 1 else [opt.groups[gi].shape for gi in range(len(opt.groups))
                                           for _ in opt.groups[gi].owned]
    per_launch_flops = phase_flops(my_shapes)[dom]
    if world == 1:
        # one launch per NS step covers every group (<= 4 groups per launch)
        launches_per_step = NS_STEPS * ((len(set(shapes)) + 3) // 4)
        flops_per_launch = per_launch_flops / (launches_per_step // NS_STEPS)
    else:
        flops_per_launch = per_launch_flops / len(opt.groups)  # one launch per group per NS step
    dom_avg_ms = dom_ms / max(dom_n, 1)
    achieved = flops_per_launch / (dom_avg_ms * 1e-3) / 1e12 if dom_n else None
    step_flops = sum(ns_dense_flops(s) for s in shapes)
    traffic = load_traffic(dom)  # bytes of the full 192-matrix launch; scale to this launch's share
    if traffic is not None:
        traffic = round(traffic * flops_per_launch / phase_flops([s for _ in range(N_LAYERS) for s in LAYER_SHAPES])[dom])
    roofline = {
        "bound": "tensor", "kernel": f"gemm_sm100_kernel ({dom})",
        "achieved": round(achieved, 1) if achieved else None,
        "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
        "frac": round(achieved / peaks["bf16_tflops_sustained"], 4) if achieved else None,
        "peak_kind": f"bf16_tflops_sustained ({peaks['source']})",
        "traffic": traffic,
        "dense_flops_per_launch": flops_per_launch, "avg_launch_ms": round(dom_avg_ms, 4),
        "step": {"dense_tflop": round(step_flops / 1e12, 3),
                 "achieved_tflops": round(step_flops / (ms * 1e-3) / 1e12, 1),
                 "per_gpu_frac_of_sustained": round(
                     step_flops / (ms * 1e-3) / 1e12 / world / peaks["bf16_tflops_sustained"], 4),
                 "per_gpu_frac_of_burst": round(step_flops / (ms * 1e-3) / 1e12 / world / peaks["bf16_tflops"], 4)},
        "per_kind_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in prof.items() if v[1]},
    }

    # ---------------------------------------------------------------- end to end (host buffers)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, params, G, step, world, opt)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fn, kind, desc = cpu_baseline_sampler()
        fn()  # warm-up
        layer_ms = statistics.median([fn() for _ in range(3)])
        cores = torch.get_num_threads() if kind == "reference" else (os.cpu_count() or 1)
        cpu = {"value": round(layer_ms * N_LAYERS, 1), "unit": "ms", "cores": cores, "kind": kind,
               "sample": f"{desc}; median of 3"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": round(ms / BASELINE_MS, 4), "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.01^2) grads/momentum, N(0,0.02^2) params, generated on device)",
            "config": {"workload": WORKLOAD, "layers": args.layers, "ns_steps": NS_STEPS,
                       "parallelism": "single gpu" if world == 1 else
                       f"zero1 round-robin shards x{world}, {args.exchange} exchange",
                       "l2": "inputs larger than L2 (8.8 GB params+grads+momentum)"},
            "roofline": roofline, "clocks": clocks, "gpu_launches": int(launches), "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    e2e_invalid = e2e is not None and not e2e.get("valid", True)
    if world > 1:
        import torch.distributed as dist
        opt.close()
        dist.barrier()
        dist.destroy_process_group()
    if e2e_invalid:
        # a wrong host copy must not pass as a timing: the run fails
        raise SystemExit("e2e: the downloaded parameters differ from the device parameters")


def run_e2e(args, params, grads, step, world, opt):
    """Same step through the public API with host buffers: every step uploads its
    gradients from pinned host memory and downloads the updated parameters to
    pinned host memory, inside the timed region.

    Pipelined as a training loop with host-resident gradients would run it:
    the device holds two gradient buffers, so step i+1's upload (copy stream)
    overlaps step i's compute, and the updated parameters are first copied into
    a device snapshot, so step i's download (second copy stream) overlaps step
    i+1's compute. Every step still moves all of its bytes each way; the timed
    region ends when the last download has landed.

    Under ZeRO-1 (world > 1) a rank uploads the gradients of the matrices it
    owns and downloads the updated parameters it owns, so the ranks together
    move every gradient and every parameter across PCIe exactly once per step.
    """
    if world == 1:
        need = list(range(len(params)))
    else:
        need = sorted({next(i for i, p in enumerate(params) if p is Gp.params[j]) for Gp in opt.groups
                       for j in Gp.owned})
    host_g = {i: torch.empty(grads[i].shape, dtype=torch.bfloat16, pin_memory=True) for i in need}
    for i in need:
        host_g[i].copy_(grads[i])
    host_p = [torch.empty(params[i].shape, dtype=torch.bfloat16, pin_memory=True) for i in need]
    h2d = sum(host_g[i].numel() * 2 for i in need)
    d2h = sum(h.numel() * 2 for h in host_p)
    gbuf = [{i: torch.empty_like(grads[i]) for i in need} for _ in range(2)]
    snap = [torch.empty_like(params[i].data) for i in need]
    mine = [params[i] for i in need]
    compute = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    ev_snap, ev_down = torch.cuda.Event(), torch.cuda.Event()
    for e in ev_free:
        e.record(compute)
    ev_down.record(compute)
    state = {"k": 0}

    def upload(k):
        b = k & 1
        up.wait_event(ev_free[b])  # the step that last read this buffer is done
        with torch.cuda.stream(up):
            for i in need:
                gbuf[b][i].copy_(host_g[i], non_blocking=True)
            ev_up[b].record(up)

    def e2e_step():
        k = state["k"]
        b = k & 1
        if k == 0:
            upload(0)
        upload(k + 1)  # next step's gradients, overlapping this step's compute
        compute.wait_event(ev_up[b])
        for i in need:
            params[i].grad = gbuf[b][i]
        step()
        ev_free[b].record(compute)
        compute.wait_event(ev_down)  # the previous download has read the snapshot
        for p, s_ in zip(mine, snap):
            s_.copy_(p.data, non_blocking=True)
        ev_snap.record(compute)
        down.wait_event(ev_snap)
        with torch.cuda.stream(down):
            for s_, h in zip(snap, host_p):
                h.copy_(s_, non_blocking=True)
            ev_down.record(down)
        state["k"] = k + 1

    for _ in range(max(1, min(args.warmup, 2))):
        e2e_step()
    compute.wait_event(ev_down)
    # the first timed step's gradients (uploaded during the last warm-up step) are on the device:
    # the timed region then holds exactly n uploads, n steps and n downloads
    compute.wait_stream(up)
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(1, min(args.steps, 5))
    a.record()
    for _ in range(n):
        e2e_step()
    compute.wait_event(ev_down)  # the last step's parameters are on the host
    compute.wait_stream(up)      # and the prefetched upload has finished too
    b.record()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / n, world)
    # the host copy is the step's result: check it against the device parameters
    matches = all(torch.equal(h, p.data.cpu()) for h, p in zip(host_p, mine))
    return {"value": round(ms, 3) if matches else None, "unit": "ms", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "host_copy_matches_device": bool(matches), "valid": bool(matches),
            "steps": n, "path": "lsr.MuonAdamW.muon_step" if world == 1 else "lsr.dist.ShardedMuon.step",
            "pipelining": "double-buffered device gradients (upload of step i+1 during step i) and a device "
                          "snapshot of the parameters (download of step i during step i+1); two copy streams",
            "copies": "all gradients in, all parameters out" if world == 1 else
                      "per rank: the gradients in and the updated parameters out of the matrices it owns "
                      "(every matrix crosses PCIe once per step across the ranks)"}


def load_traffic(kind: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if present."""
    f = ROOT / "profiles" / "traffic_per_launch.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) == 2 and not line.startswith("#") and parts[0] == kind:
            return float(parts[1])
    return None


# ---------------------------------------------------------------------------
# Per-row workloads (not the headline line): --workload cfg1|cfg2|cfg3|cfg5
# ---------------------------------------------------------------------------

def _nvtx(name):
    """An NVTX push/pop range around a timed phase, so an ncu capture can select that phase's
    kernels (`ncu --nvtx --nvtx-include "<name>/" ...`)."""
    return torch.cuda.nvtx.range(name) if name else contextlib.nullcontext()


def _time_gpu(fn, warmup, iters, flush_bytes=256 << 20, name=None):
    """Mean ms of fn() over `iters` runs, L2 flushed (a buffer larger than L2 is written) before each
    unless flush_bytes is 0. Warm-up and timed runs sit inside the NVTX range `name`."""
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda") if flush_bytes else None
    with _nvtx(name):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            if flush is not None:
                flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            tot += a.elapsed_time(b)
    return tot / iters


def _median_loop_ms(fn, warmup=20, iters=100, repeats=7, name=None):
    """Per-call ms as the reference's microbenchmarks time their kernels (median_ms,
    hft_fused.py:403-432; median_us, kron_cuda.py:91-114): `iters` back-to-back calls between two
    events, median over `repeats`. Host launch cost overlaps the GPU here, so the figure is the
    larger of the two per call. Also returns the host microseconds per call (no synchronisation
    inside the loop)."""
    with _nvtx(name):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        vals, host = [], []
        for _ in range(repeats):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            t0 = time.perf_counter()
            for _ in range(iters):
                fn()
            host.append((time.perf_counter() - t0) * 1e6 / iters)
            b.record()
            b.synchronize()
            vals.append(a.elapsed_time(b) / iters)
    return statistics.median(vals), statistics.median(host)


def _time_cpu(fn, reps=2):
    fn()
    t = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        t.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(t)


def _torch_batched_coupled_newton(A, root, tolerance=1e-6, max_iterations=100):
    """The reference's batched recurrence (shampoo.py:408-542) as plain torch fp32 ops."""
    B, n, _ = A.shape
    eye = torch.eye(n, device=A.device, dtype=A.dtype).expand(B, n, n)
    alpha = -1.0 / float(root)
    z = (root + 1.0) / (2.0 * A.flatten(1).norm(dim=1))
    X = (z.pow(-alpha)[:, None, None] * eye).contiguous()
    M = (z[:, None, None] * A).contiguous()
    active = (M - eye).abs().flatten(1).amax(dim=1) > tolerance
    for _ in range(max_iterations):
        if not bool(active.any()):
            break
        Mp = alpha * M + (1.0 - alpha) * eye
        Xn = X @ Mp
        P = Mp @ Mp
        if root == 4:
            P = P @ P
        Mn = P @ M
        m3 = active[:, None, None]
        X = torch.where(m3, Xn, X)
        M = torch.where(m3, Mn, M)
        active = (M - eye).abs().flatten(1).amax(dim=1) > tolerance
    return X


def run_cfg5_sharded(args, world: int) -> None:
    """The GPT-2-XL SOAP step under ZeRO-1 on `world` GPUs (one process each, NCCL): every rank builds
    the same 192 matrices (seed 5), owns 1/world of the 2016 blocks (greedy by flops), and the
    directions are all-gathered in the reference's default communication dtype (float16). Time per
    step: CUDA events on each rank, max over ranks; total work is fixed (strong scaling)."""
    import torch.distributed as dist
    from lsr import shampoo as SH
    rank, local_rank = int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    g = torch.Generator().manual_seed(5)
    shapes = [s for _ in range(args.layers) for s in LAYER_SHAPES]
    params = [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().to(dev)) for s in shapes]
    for p in params:
        p.grad = (torch.randn(*p.shape, generator=g) * 0.01).bfloat16().to(dev)
    opt = SH.DistributedShampoo(params, lr=0.02, betas=(0.95, 0.95), epsilon=1e-8, weight_decay=0.01,
                                max_preconditioner_dim=1024, precondition_frequency=10 ** 9,
                                start_preconditioning_step=10 ** 9, preconditioner_config=SH.DefaultSOAPConfig,
                                distributed_config=SH.DDPDistributedConfig())
    opt.step()  # builds the block groups
    gq = torch.Generator(device=dev).manual_seed(5 + rank)
    for _, grp, _ in opt._groups:
        if grp is None:
            continue
        n, r, c = grp.stack.shape
        grp.QL = torch.linalg.qr(torch.randn(n, r, r, generator=gq, device=dev))[0].bfloat16().contiguous()
        grp.QR = torch.linalg.qr(torch.randn(n, c, c, generator=gq, device=dev))[0].bfloat16().contiguous()
    for _ in range(args.warmup):
        opt.step()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        opt.step()
    b.record()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
    if rank == 0:
        from oracle import shampoo as osh
        fl = sum(osh.soap_flops(r, c) * len(lst) for (r, c), _, lst in opt._groups)
        peaks = measured_peaks()
        print(json.dumps({"workload": f"cfg5: GPT-2-XL SOAP step, {args.layers} layers, 2016 blocks at 1024, "
                                      f"ZeRO-1 over {world} GPUs, float16 exchange",
                          "value": ms, "unit": "ms", "n_gpus": world, "algorithmic_tflop": fl / 1e12,
                          "tflops": fl / ms / 1e9,
                          "per_gpu_frac_of_sustained": fl / ms / 1e9 / world / peaks["bf16_tflops_sustained"],
                          "steps": args.steps, "warmup": args.warmup, "scaling": "strong"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_workload(args) -> None:
    import lsr
    import lsr.kron as K
    from lsr import shampoo as SH
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        if args.workload != "cfg5":
            raise SystemExit(f"--workload {args.workload} runs on one GPU; cfg5 also runs sharded under torchrun")
        run_cfg5_sharded(args, world)
        return
    torch.cuda.set_device(0)
    peaks = measured_peaks()
    dev = torch.device("cuda", 0)
    lines = []
    w = args.workload
    if w == "cfg1":
        g = torch.Generator().manual_seed(0)
        wide = (torch.randn(12, 768, 3072, generator=g) * 0.02).bfloat16().to(dev)
        tall = (torch.randn(12, 3072, 768, generator=g) * 0.02).bfloat16().to(dev)
        ms = _time_gpu(lambda: (lsr.zeropower_via_newtonschulz5(wide, 5, 1e-7),
                                lsr.zeropower_via_newtonschulz5(tall, 5, 1e-7)), args.warmup, args.steps,
                      name="cfg1")
        fl = 24 * ns_dense_flops((768, 3072))
        from oracle import muon as om
        G1 = wide[0].float().cpu().numpy()
        cpu = _time_cpu(lambda: om.zeropower(G1, 5, 1e-7), 1) * 24
        lines.append({"workload": "cfg1: Newton-Schulz, 12x(768x3072) + 12x(3072x768), 5 steps", "value": ms,
                      "unit": "ms", "dense_tflop": fl / 1e12, "tflops": fl / ms / 1e9,
                      "frac_of_sustained": fl / ms / 1e9 / peaks["bf16_tflops_sustained"],
                      "cpu_ms": cpu, "cpu_sample": "1 matrix via the numpy restatement, x24"})
    elif w == "cfg2":
        g = torch.Generator().manual_seed(1)
        Ms = [torch.randn(1024, 1024, generator=g) / 32.0 for _ in range(2)]
        A, B = [((m + m.T) / 2).contiguous().to(dev) for m in Ms]
        X = torch.randn(64, 1024, 1024, generator=torch.Generator().manual_seed(2)).to(dev)
        fl = 64 * (2.0 * 1024 ** 3 * 2)
        for name, a, x, b, peak in (("fp32 (3xTF32)", A, X, B, peaks["bf16_tflops_sustained"] / 2),
                                    ("bf16", A.bfloat16(), X.bfloat16(), B.bfloat16(),
                                     peaks["bf16_tflops_sustained"])):
            Y = torch.empty(64, 1024, 1024, device=dev)
            ms = _time_gpu(lambda: K.kron_sum(a, x, b, out=Y), args.warmup, args.steps,
                           name="cfg2." + name.split()[0])
            nbytes = x.numel() * x.element_size() + Y.numel() * 4
            line = {"workload": f"cfg2: Kronecker sum (A+B)vec(X), A,B 1024^2, 64 RHS, {name}", "value": ms,
                    "unit": "ms", "algorithmic_gflop": fl / 1e9, "tflops": fl / ms / 1e9,
                    "min_bytes": nbytes, "gbs": nbytes / ms / 1e6}
            if name.startswith("fp32"):
                line["tensor_tflops_3xtf32"] = 3 * fl / ms / 1e9
                line["note"] = "3 tf32 products per fp32 product; tf32 dense peak is half the bf16 peak"
                line["frac_of_tf32_peak_3x"] = 3 * fl / ms / 1e9 / peak
            else:
                line["frac_of_sustained"] = fl / ms / 1e9 / peak
            lines.append(line)
        An, Bn, Xn = A.cpu().numpy(), B.cpu().numpy(), X[:4].cpu().numpy()
        cpu = _time_cpu(lambda: An @ Xn + Xn @ Bn.T, 2) * 16
        lines[0]["cpu_ms"] = cpu
        lines[0]["cpu_sample"] = "4 of 64 right-hand sides, numpy fp32 A@X + X@B.T, x16"
    elif w in ("cfg3", "cfg5"):
        g = torch.Generator().manual_seed(3 if w == "cfg3" else 5)

        gq = torch.Generator(device=dev).manual_seed(3 if w == "cfg3" else 5)

        def orth(n, b):  # seeded random orthogonal bases: QR of N(0, 1)
            return torch.linalg.qr(torch.randn(b, n, n, generator=gq, device=dev))[0].bfloat16().contiguous()
        if w == "cfg3":
            r, c = 1600, 6400
            G = (torch.randn(1, r, c, generator=g) * 0.01).bfloat16().to(dev)
            L = torch.zeros(1, r, r, device=dev)
            R = torch.zeros(1, c, c, device=dev)
            ms_stats = _time_gpu(lambda: (SH.gram_update(G, L, 0, 0.0, 1.0), SH.gram_update(G, R, 1, 0.0, 1.0)),
                                 args.warmup, args.steps, name="cfg3.stats")
            Lr, Rr = orth(r, 1), orth(c, 1)  # stand-ins with the shapes of the precomputed inverse roots
            ms_apply = _time_gpu(lambda: SH.shampoo_direction(G, Lr, Rr), args.warmup, args.steps,
                                 name="cfg3.shampoo")
            m = torch.zeros(1, r, c, device=dev)
            v = torch.zeros(1, r, c, device=dev)
            ms_soap = _time_gpu(lambda: SH.soap_direction(G, None, None, Lr, Rr, m, v, 0.95, 0.95, 1e-8, 1, False),
                                args.warmup, args.steps, name="cfg3.soap")
            f_stats = 2.0 * r * r * c + 2.0 * r * c * c
            for name, ms, fl in (("statistics L=GG^T, R=G^TG", ms_stats, f_stats),
                                 ("Shampoo apply L^-1/4 G R^-1/4", ms_apply, f_stats),
                                 ("SOAP rotate, Adam, rotate back", ms_soap, 2 * f_stats)):
                lines.append({"workload": f"cfg3: 1600x6400, {name}", "value": ms, "unit": "ms",
                              "algorithmic_gflop": fl / 1e9, "tflops": fl / ms / 1e9,
                              "frac_of_sustained": fl / ms / 1e9 / peaks["bf16_tflops_sustained"]})
        else:
            shapes = [s for _ in range(args.layers) for s in LAYER_SHAPES]
            params = [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().to(dev)) for s in shapes]
            for p in params:
                p.grad = (torch.randn(*p.shape, generator=g) * 0.01).bfloat16().to(dev)
            opt = SH.DistributedShampoo(params, lr=0.02, betas=(0.95, 0.95), epsilon=1e-8, weight_decay=0.01,
                                        max_preconditioner_dim=1024, precondition_frequency=10 ** 9,
                                        start_preconditioning_step=10 ** 9,
                                        preconditioner_config=SH.DefaultSOAPConfig)
            opt.step()  # builds the block groups
            for _, grp, _ in opt._groups:
                n, r, c = grp.stack.shape
                grp.QL, grp.QR = orth(r, n), orth(c, n)
            ms = _time_gpu(opt.step, args.warmup, args.steps, name="cfg5.step")
            from lsr import _lib
            _lib.profile_enable(True)
            _lib.profile_read(reset=True)
            opt.step()
            torch.cuda.synchronize()
            _lib.profile_enable(False)
            kinds = {k: round(v[0], 3) for k, v in _lib.profile_read(reset=True).items() if v[1]}
            from oracle import shampoo as osh
            fl = sum(osh.soap_flops(r, c) * len(grp.refs) for (r, c), grp, _ in opt._groups)
            lines.append({"workload": f"cfg5: GPT-2-XL SOAP step, {args.layers} layers, "
                                      f"{sum(len(grp.refs) for _, grp, _ in opt._groups)} blocks at 1024, 1 GPU",
                          "value": ms, "unit": "ms", "algorithmic_tflop": fl / 1e12, "tflops": fl / ms / 1e9,
                          "frac_of_sustained": fl / ms / 1e9 / peaks["bf16_tflops_sustained"],
                          "per_kind_ms_one_step": kinds})
    elif w in ("refresh", "cfg5s"):
        # refresh: the periodic SOAP eigenbasis refresh of the config-5 blocks (every L and R factor,
        # statistics of a few seeded steps): power iteration with Householder QR from the current
        # bases (lsr_eigenbasis_refresh_f32, one iteration, as every refresh after the first), timed
        # beside an fp32 torch.linalg.eigh of a sample of the same factors (extrapolated by count).
        # cfg5s: the Shampoo step (Adam grafting, inverse 4th roots fixed) on the config-5 blocks.
        g = torch.Generator().manual_seed(5)
        shapes = [s for _ in range(args.layers) for s in LAYER_SHAPES]
        params = [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().to(dev)) for s in shapes]
        for p in params:
            p.grad = (torch.randn(*p.shape, generator=g) * 0.01).bfloat16().to(dev)
        soap = w == "refresh"
        opt = SH.DistributedShampoo(params, lr=0.02, betas=(0.95, 0.95), epsilon=1e-8, weight_decay=0.01,
                                    max_preconditioner_dim=1024, precondition_frequency=10 ** 9,
                                    start_preconditioning_step=1 if not soap else 10 ** 9,
                                    preconditioner_config=SH.DefaultSOAPConfig if soap else None,
                                    grafting_config=None if soap else SH.AdamPreconditionerConfig(0.95, 1e-8))
        for _ in range(3):
            opt.step()  # statistics of three steps
        if soap:
            for _, grp, _ in opt._groups:
                opt._refresh(grp, 1e-8)  # first refresh (from the identity basis, first_iterations)
            torch.cuda.synchronize()
            ms = _time_gpu(lambda: [opt._refresh(grp, 1e-8) for _, grp, _ in opt._groups], args.warmup, args.steps,
                           name="refresh")
            nfac = sum(2 * len(grp.refs) for _, grp, _ in opt._groups)
            # eigh of a sample: the first 4 blocks of every shape, both factors, scaled by count
            t_eigh, n_eigh = 0.0, 0
            for (r, c), grp, _ in opt._groups:
                k = min(4, len(grp.refs))
                Ls, Rs = grp.L[:k].clone(), grp.R[:k].clone()
                ms_s = _time_gpu(lambda: (torch.linalg.eigh(Ls), torch.linalg.eigh(Rs)), 1, 1, flush_bytes=0)
                t_eigh += ms_s * len(grp.refs) / k
                n_eigh += 2 * k

            def torch_refresh():  # the same refresh through torch: cuBLAS bmm + cuSOLVER batched QR
                for _, grp, _ in opt._groups:
                    for S_, Q_ in ((grp.L, grp.QLf), (grp.R, grp.QRf)):
                        torch.linalg.qr(torch.bmm(S_, Q_))
            ms_tq = _time_gpu(torch_refresh, 1, 1)
            lines.append({"workload": f"refresh: SOAP eigenbasis refresh of the config-5 blocks ({args.layers} layers, "
                                      f"{nfac} factors of <= 1024^2), one power iteration + Householder QR",
                          "value": ms, "unit": "ms", "torch_eigh_fp32_ms_extrapolated": t_eigh,
                          "eigh_sample_factors": n_eigh, "speedup_vs_eigh": t_eigh / ms,
                          "torch_bmm_qr_fp32_ms": ms_tq, "speedup_vs_torch_qr": ms_tq / ms})
        else:
            gq = torch.Generator(device=dev).manual_seed(5)
            for (r, c), grp, _ in opt._groups:  # stand-ins with the shapes of the inverse roots
                n = len(grp.refs)
                grp.QL = torch.linalg.qr(torch.randn(n, r, r, generator=gq, device=dev))[0].bfloat16().contiguous()
                grp.QR = torch.linalg.qr(torch.randn(n, c, c, generator=gq, device=dev))[0].bfloat16().contiguous()
                grp.have_roots = True
            ms = _time_gpu(opt.step, args.warmup, args.steps, name="cfg5s.step")
            from oracle import shampoo as osh
            # statistics and the two-sided apply: 2 (2 r^2 c + 2 r c^2) = 2/3 of the SOAP count
            fl = sum(osh.soap_flops(r, c) * len(grp.refs) * 2 / 3 for (r, c), grp, _ in opt._groups)
            lines.append({"workload": f"cfg5s: GPT-2-XL Shampoo step with Adam grafting, {args.layers} layers, "
                                      f"{sum(len(grp.refs) for _, grp, _ in opt._groups)} blocks at 1024, 1 GPU",
                          "value": ms, "unit": "ms",
                          "algorithmic_tflop": fl / 1e12, "tflops": fl / ms / 1e9,
                          "frac_of_sustained": fl / ms / 1e9 / peaks["bf16_tflops_sustained"]})
    elif w == "kron64x8":
        # The reference's own Kronecker-sum sweep (hft_fused.py:856-862): x [M, 64, 8], S terms
        # A_s [64,64] / sqrt(64), B_s [8,8] / sqrt(8), at = A^T prepacked, fp32 (TF32 off). Its
        # kron_sum_64x8_kernel (built from the staged hft_fused.py by its own load_inline) and
        # lsr.kron.kron_sum_out run on the same inputs and GPU, both timed with the reference's own
        # method (median_ms: 100 back-to-back calls between two events, median of 7, no L2 flush);
        # results are compared against the fp64 product.
        ref = load_reference_module("hft_fused")
        torch.backends.cuda.matmul.allow_tf32 = False
        for M in (256, 1024, 4096, 16384):
            for S in (1, 2, 4, 8):
                gk = torch.Generator(device=dev).manual_seed(17 + 1000 * M + S)
                X = torch.randn(M, 64, 8, device=dev, generator=gk)
                A = torch.randn(S, 64, 64, device=dev, generator=gk) / 8.0
                B = torch.randn(S, 8, 8, device=dev, generator=gk) / math.sqrt(8)
                AT = A.transpose(1, 2).contiguous()
                Y = torch.empty_like(X)
                Yd = torch.einsum("sik,mkl,sjl->mij", A.double(), X.double(), B.double())

                def ours():
                    K.kron_sum_out(X, AT, B, Y)
                ms, host_us = _median_loop_ms(ours, name=f"kron64x8.M{M}.S{S}")
                err = ((Y.double() - Yd).norm() / Yd.norm()).item()
                line = {"workload": f"kron64x8: x [{M},64,8], S={S}, fp32", "value": ms, "unit": "ms",
                        "host_us_per_call": host_us, "rel_err_vs_fp64": err,
                        "timing": "median of 7 x (100 back-to-back calls between two events)"}
                if ref is not None:
                    Yr = torch.empty_like(X)

                    def theirs():
                        ref.ext.kron_sum_out(X, AT, B, Yr)
                    ms_ref, host_ref = _median_loop_ms(theirs)
                    line.update({"reference_kernel_ms": ms_ref, "reference_host_us_per_call": host_ref,
                                 "speedup_vs_reference_kernel": ms_ref / ms,
                                 "reference_rel_err_vs_fp64": ((Yr.double() - Yd).norm() / Yd.norm()).item()})
                else:
                    line["reference_kernel_ms"] = None
                lines.append(line)
    elif w == "kronrec":
        # The reference's tiny-factor reconstruction sweep (kron_cuda.py:705-1040): W [16, 768] =
        # sum_s F_0[s] x ... x F_{K-1}[s] for the three equivalent factorisations K = 3, 4, 5 of
        # make_equivalent_factors (kron_cuda.py:169-225), S in its default list. Its Triton
        # native_reconstruct (best block of 64..512, as its find_best_native picks) and
        # lsr.kron.native_reconstruct run on the same factors and GPU, both timed with the
        # reference's median_us method (200 back-to-back calls between two events, median of 7).
        ref = load_reference_module("kron_cuda")
        for S in (1, 2, 4, 8, 16, 32, 64, 96, 128, 192, 256):
            if ref is not None:
                reps = ref.make_equivalent_factors(S, seed=17)
            else:  # the same construction: K=5 factors, merged pairwise into the K=4 and K=3 lists
                gk = torch.Generator().manual_seed(17 + S)
                f = [(0.5 * torch.randn(S, *sh, generator=gk)).to(dev)
                     for sh in ((1, 3), (2, 4), (2, 4), (2, 4), (2, 4))]

                def bk(a, b):
                    return torch.einsum("sij,skl->sikjl", a, b).reshape(a.shape[0], a.shape[1] * b.shape[1],
                                                                        a.shape[2] * b.shape[2])
                g01 = bk(f[0], f[1])
                reps = {5: f, 4: [g01] + f[2:], 3: [bk(g01, f[2])] + f[3:]}
            W64 = None
            for Kf in (5, 4, 3):
                fac = reps[Kf]
                out = torch.empty(16, 768, device=dev)
                ms, host_us = _median_loop_ms(lambda: K.native_reconstruct(fac, Kf, out), warmup=10, iters=200,
                                              name=f"kronrec.K{Kf}.S{S}")
                if W64 is None:  # fp64 reference value of W from the K=5 factors
                    t = reps[5][0].double().cpu()
                    for fk in reps[5][1:]:
                        fk = fk.double().cpu()
                        t = torch.einsum("sij,skl->sikjl", t, fk).reshape(S, t.shape[1] * fk.shape[1],
                                                                          t.shape[2] * fk.shape[2])
                    W64 = t.sum(0)
                err = ((out.double().cpu() - W64).norm() / W64.norm()).item()
                line = {"workload": f"kronrec: W 16x768, K={Kf}, S={S}, fp32", "value": ms, "unit": "ms",
                        "host_us_per_call": host_us, "rel_err_vs_fp64": err,
                        "timing": "median of 7 x (200 back-to-back calls between two events)"}
                if ref is not None:
                    outr = torch.empty(16, 768, device=dev)
                    best, _ = ref.find_best_native(fac, Kf, outr)
                    ref.native_reconstruct(fac, Kf, outr, block=best["block"])
                    torch.cuda.synchronize()
                    line.update({"reference_triton_ms": best["us"] / 1e3, "reference_block": best["block"],
                                 "speedup_vs_reference_triton": best["us"] / 1e3 / ms,
                                 "reference_rel_err_vs_fp64": ((outr.double().cpu() - W64).norm()
                                                               / W64.norm()).item()})
                else:
                    line["reference_triton_ms"] = None
                lines.append(line)
    elif w == "hawkes":
        # The reference's Hawkes event-update benchmark (benchmark_hawkes, hft.py:615-800): 128 assets
        # x 8 event types (D = 1024), N in {1024, 8192, 32768} streams, inputs drawn as it draws them.
        # lsr.hawkes and the reference's Triton kernels (function definitions of the staged hft.py)
        # on the same inputs and GPU, both timed with the reference's method (median of 7 x 100
        # back-to-back calls). HBM-bound: 8 bytes per state entry (state in, out out); the 4 MB
        # dense K stays in L2.
        from lsr import hawkes as H
        from oracle import stage_reference
        try:
            import triton
            ref = stage_reference.load_functions(
                "hft.py", ["hawkes_dense_kernel", "hawkes_kron_kernel", "hawkes_dense", "hawkes_kron"],
                {"torch": torch, "triton": triton, "tl": triton.language})
        except ImportError:
            ref = None
        NA, NE = 128, 8
        g = torch.Generator(device=dev).manual_seed(123)
        KA = (torch.rand(NA, NA, device=dev, generator=g) * 0.02).contiguous()
        KE = (torch.rand(NE, NE, device=dev, generator=g) * 0.02).contiguous()
        Kcol = torch.kron(KA, KE).T.contiguous()
        D = NA * NE
        for N in (1024, 8192, 32768):
            state = torch.randn(N, D, device=dev, generator=g)
            ea = torch.randint(0, NA, (N,), device=dev, generator=g, dtype=torch.int32)
            et = torch.randint(0, NE, (N,), device=dev, generator=g, dtype=torch.int32)
            ev = (ea * NE + et).contiguous()
            decay = (0.90 + 0.099 * torch.rand(N, device=dev, generator=g)).contiguous()
            nbytes = 8.0 * N * D
            for kind in ("dense", "kron"):
                out = torch.empty_like(state)
                if kind == "dense":
                    ours = lambda: H.hawkes_dense(state, ev, decay, Kcol, out)  # noqa: E731
                    theirs = (lambda o: ref["hawkes_dense"](state, ev, decay, Kcol, o)) if ref else None
                else:
                    ours = lambda: H.hawkes_kron(state, ea, et, decay, KA, KE, out)  # noqa: E731
                    theirs = (lambda o: ref["hawkes_kron"](state, ea, et, decay, KA, KE, o)) if ref else None
                ms, host_us = _median_loop_ms(ours, name=f"hawkes.{kind}.N{N}")
                line = {"workload": f"hawkes {kind}: N={N} streams, D={D} (128 assets x 8 types), fp32",
                        "value": ms, "unit": "ms", "host_us_per_call": host_us, "gbs": nbytes / ms / 1e6,
                        "frac_of_hbm": nbytes / ms / 1e6 / peaks["hbm_gbs"],
                        "timing": "median of 7 x (100 back-to-back calls between two events)"}
                if theirs is not None:
                    o2 = torch.empty_like(state)
                    ms_ref, _ = _median_loop_ms(lambda: theirs(o2))
                    err = ((out.double() - o2.double()).norm() / o2.double().norm()).item()
                    line.update({"reference_triton_ms": ms_ref, "speedup_vs_reference_triton": ms_ref / ms,
                                 "rel_err_vs_reference": err})
                else:
                    line["reference_triton_ms"] = None
                lines.append(line)
    elif w == "pauli":
        # The reference's Pauli-string Hamiltonian benchmark (pauli.py:1184-1300): K in {8, 12, 16, 20}
        # qubits, S in {64, 256, 1024} strings, cases with 2^K S above 150 M skipped as it skips them;
        # problems drawn by its make_problem. Its native_apply is timed at the partition count its
        # tune_native picks (median_us: 5 repeats of a back-to-back loop); lsr.pauli.native_apply the
        # same way. The state (at most 8 MB) stays in L2: the figure of merit is amplitude reads per
        # second, 8 bytes per (output, string) pair.
        from lsr import pauli as PA
        ref = load_reference_module("pauli")
        for K in (8, 12, 16, 20):
            for S in (64, 256, 1024):
                N = 1 << K
                if N * S > 150_000_000:
                    continue
                if ref is not None:
                    prob = ref.make_problem(K, S)
                else:  # the same draw: seeded ops, coefficients / sqrt(S), a normalised random state
                    gk = torch.Generator().manual_seed(17 + 10007 * K + S)
                    ops = torch.randint(0, 4, (S, K), generator=gk, dtype=torch.int64)
                    flip, sign, ny = PA.encode_pauli_strings(ops)
                    coeff = torch.randn(S, generator=gk) / math.sqrt(S)
                    pr, pi = torch.randn(N, generator=gk), torch.randn(N, generator=gk)
                    nrm = torch.sqrt((pr ** 2).sum() + (pi ** 2).sum())
                    prob = {"K": K, "S": S, "N": N, "flip": flip.to(dev), "sign": sign.to(dev), "ny": ny.to(dev),
                            "coeff": coeff.to(dev), "psi_r": (pr / nrm).to(dev), "psi_i": (pi / nrm).to(dev)}
                out_r, out_i = torch.empty(N, device=dev), torch.empty(N, device=dev)
                iters = 100 if N * S <= 2_000_000 else (30 if N * S <= 20_000_000 else 10)
                ms, host_us = _median_loop_ms(lambda: PA.native_apply(prob, 1, None, None, out_r, out_i),
                                              warmup=3, iters=iters, repeats=5, name=f"pauli.K{K}.S{S}")
                pairs = float(N) * S
                line = {"workload": f"pauli: K={K} qubits (N={N}), S={S} strings, complex fp32", "value": ms,
                        "unit": "ms", "host_us_per_call": host_us, "amplitude_reads_per_s": pairs / ms * 1e3,
                        "timing": f"median of 5 x ({iters} back-to-back calls between two events)"}
                if ref is not None:
                    best, _ = ref.tune_native(prob)
                    want = best["out_r"].double() + 1j * best["out_i"].double()
                    got = out_r.double() + 1j * out_i.double()
                    line.update({"reference_triton_ms": best["us"] / 1e3, "reference_P": best["P"],
                                 "speedup_vs_reference_triton": best["us"] / 1e3 / ms,
                                 "rel_err_vs_reference": ((got - want).abs().norm() / want.abs().norm()).item()})
                else:
                    line["reference_triton_ms"] = None
                lines.append(line)
    elif w == "f1":
        # Batched coupled Newton inverse roots on the reference's full bucket list
        # (shampoo.py:812-840: (n, root, B), seeds 17 + 100 j, tolerance 1e-6,
        # max 100 iterations), SPD factors built as make_spd_batch builds them.
        # Beside ours: the reference's batched op sequence in torch fp32 (TF32
        # off, cuBLAS SGEMM, shampoo.py:408-542) on the same GPU.
        torch.backends.cuda.matmul.allow_tf32 = False
        buckets = [(128, 4, 2), (256, 2, 86), (256, 4, 128), (512, 2, 128), (512, 4, 128)]
        tot_ours = tot_ref = tot_tc = 0.0
        for j, (n, root, B) in enumerate(buckets):
            if args.bucket is not None and j != args.bucket:
                continue
            g = torch.Generator().manual_seed(17 + 100 * j)
            Xr = torch.randn(B, n, n, generator=g)
            A = Xr @ Xr.transpose(-1, -2) / float(n)
            A = A / A.flatten(1).norm(dim=1).clamp_min(1e-12)[:, None, None] * math.sqrt(n)
            ridge = torch.full((B,), 1e-2)
            ridge[-max(1, int(round(B * 0.15))):] = 1e-5
            A = (A + ridge[:, None, None] * torch.eye(n)).contiguous().to(dev)
            _, iters, _ = lsr.batched_coupled_newton(A, root)
            ms = _time_gpu(lambda: lsr.batched_coupled_newton(A, root), args.warmup, args.steps,
                           name=f"f1.n{n}.root{root}")
            ms_ref = _time_gpu(lambda: _torch_batched_coupled_newton(A, root), 1, max(1, args.steps // 2))
            from lsr import newton as NW
            ms_tc = _time_gpu(lambda: NW._run(A, root, 0.0, 1e-6, 100, use_tf32=True), args.warmup, args.steps)
            fl = float(iters.sum().item()) * (3 if root == 2 else 4) * 2.0 * n ** 3
            tot_ours += ms
            tot_ref += ms_ref
            tot_tc += ms_tc
            lines.append({"workload": f"f1: batched coupled Newton n={n} root={root} B={B}", "value": ms,
                          "unit": "ms", "torch_fp32_ms": ms_ref, "speedup_vs_torch_fp32": ms_ref / ms,
                          "tf32_mode_ms": ms_tc,
                          "iters_median": float(iters.float().median().item()), "iters_max": int(iters.max().item()),
                          "algorithmic_tflop": fl / 1e12, "tflops": fl / ms / 1e9})
        if args.bucket is None:
          lines.append({"workload": "f1: all five buckets", "value": tot_ours, "unit": "ms",
                        "torch_fp32_ms": tot_ref, "speedup_vs_torch_fp32": tot_ref / tot_ours, "tf32_mode_ms": tot_tc,
                        "note": "value: fp32 FFMA (the reference's precision); tf32_mode_ms: TF32 allowed"})
    elif w == "muon_torch":
        # The reference's Muon op sequence (muon_lm_ddp.py:554-593, :373-426: momentum,
        # torch.bmm Newton-Schulz per shape group in chunks of 8, apply) on this GPU
        # (cuBLAS), on the same 192-matrix workload: the library baseline on B200.
        shapes, P, G, M = make_params(dev, args.layers)
        del shapes
        a_, b_, c_ = 3.4445, -4.7750, 2.0315

        def ref_step():
            groups = {}
            for i, p in enumerate(P):
                groups.setdefault((min(p.shape), max(p.shape)), []).append(i)
            for _, idx in groups.items():
                for s0 in range(0, len(idx), 8):
                    chunk = idx[s0:s0 + 8]
                    us = []
                    for i in chunk:
                        M[i].mul_(MU).add_(G[i])
                        u = G[i] + MU * M[i]
                        us.append(u.T if u.shape[0] > u.shape[1] else u)
                    X = torch.stack(us).bfloat16()
                    X = X / X.flatten(1).norm(dim=1).clamp(min=EPS)[:, None, None]
                    for _ in range(NS_STEPS):
                        A = torch.bmm(X, X.transpose(-1, -2))
                        B = b_ * A + c_ * torch.bmm(A, A)
                        X = a_ * X + torch.bmm(B, X)
                    for k, i in enumerate(chunk):
                        upd = X[k].T if P[i].shape[0] > P[i].shape[1] else X[k]
                        P[i].mul_(1 - LR * WD)
                        ratio = max(1.0, P[i].shape[0] / P[i].shape[1]) ** 0.5
                        P[i].add_(upd, alpha=-LR * ratio)
        ms = _time_gpu(ref_step, args.warmup, args.steps)
        fl = sum(ns_dense_flops(p.shape) for p in P)
        lines.append({"workload": "reference torch op sequence (cuBLAS bmm, chunks of 8) on the GPT-2-XL Muon step",
                      "value": ms, "unit": "ms", "dense_tflop": fl / 1e12, "tflops": fl / ms / 1e9,
                      "frac_of_sustained": fl / ms / 1e9 / peaks["bf16_tflops_sustained"]})
    for ln in lines:
        ln.update({"steps": args.steps, "warmup": args.warmup, "l2": "flushed (256 MB write) before each run",
                   "peak_kind": peaks["source"], "cores": os.cpu_count() or 1})
        print(json.dumps(ln), flush=True)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["lsr", "reference"], default="lsr")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="GPT-2-XL layers (48 = the full model)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bucket", type=int, default=None, help="f1 workload: run one bucket (0..4) only")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="nccl",
                    help="N>1: parameter exchange (peer-memory push or NCCL all-gather)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["muon", "cfg1", "cfg2", "cfg3", "cfg5", "cfg5s", "refresh", "f1", "muon_torch",
                                           "kronrec", "hawkes", "pauli",
                                           "kron64x8"],
                    default="muon",
                    help="muon = the headline GPT-2-XL Muon step (default); cfgN = per-row workloads")
    args = ap.parse_args(argv)
    if args.workload != "muon" and args.impl == "lsr":
        run_workload(args)
        return 0
    if args.impl == "reference":
        run_reference_arm(args)
        return 0
    run_lsr(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
