"""Muon on B200: drop-in replacements for the Muon pieces of muon_lm_ddp.py.

* ``zeropower_serial(G, ns_steps, eps)``            muon_lm_ddp.py:331-370
* ``zeropower_batched_oriented(X, ns_steps, eps)``  muon_lm_ddp.py:373-426
* ``zeropower_via_newtonschulz5(G, steps, eps)``    the common name of the same map
* ``adjusted_muon_lr(lr, shape, mode)``             muon_lm_ddp.py:302-328
* ``MuonAdamW``                                     muon_lm_ddp.py:433-745
* ``Muon``  — the same step as a ``torch.optim.Optimizer`` (with state_dict).

The Newton–Schulz chain, the momentum / Nesterov update, the normalisation, the
orientation of tall matrices and the update apply all run in liblsr's sm_100a
kernels (tcgen05 GEMMs with TMEM accumulators). There is no CPU path: CPU
tensors raise ``ValueError``.
"""
from __future__ import annotations

import ctypes
import math
from collections import defaultdict

import torch

from . import _lib

NS_A = 3.4445
NS_B = -4.7750
NS_C = 2.0315


def adjusted_muon_lr(lr, shape, mode):
    """Learning rate scaled by the matrix shape (muon_lm_ddp.py:302-328)."""
    rows, cols = shape
    if mode == "original":
        ratio = math.sqrt(max(1.0, rows / cols))
    elif mode == "match_rms_adamw":
        ratio = 0.2 * math.sqrt(max(rows, cols))
    elif mode == "none":
        ratio = 1.0
    else:
        raise ValueError(mode)
    return lr * ratio


def _ns_call(X: torch.Tensor, ns_steps: int, eps: float, orient: bool, coef=(NS_A, NS_B, NS_C)) -> torch.Tensor:
    _lib.require_cuda(X, "input")
    if X.dim() not in (2, 3):
        raise ValueError("Newton-Schulz input must be [rows, cols] or [batch, rows, cols]")
    if ns_steps < 0:
        raise ValueError("ns_steps must be >= 0")
    Xb = X.to(dtype=torch.bfloat16, copy=False).contiguous()
    batch = 1 if Xb.dim() == 2 else Xb.shape[0]
    rows, cols = Xb.shape[-2], Xb.shape[-1]
    out = torch.empty_like(Xb)
    if batch == 0 or Xb.numel() == 0:
        return out
    lib = _lib.load()
    with _lib.on_device(Xb.device):
        ws_bytes = lib.lsr_ns_workspace_bytes(batch, rows, cols, int(orient))
        ws = _lib.WORKSPACE.get(ws_bytes, Xb.device)
        rc = lib.lsr_ns_bf16(Xb.data_ptr(), out.data_ptr(), batch, rows, cols, int(orient), int(ns_steps),
                             float(coef[0]), float(coef[1]), float(coef[2]), float(eps), ws.data_ptr(), ws_bytes,
                             _lib.stream_handle(Xb.device))
    _lib.check(rc, "lsr_ns_bf16")
    return out


@torch.no_grad()
def zeropower_serial(G, ns_steps, eps):
    """Quintic Newton–Schulz of one matrix; tall inputs are transposed and back.

    Same contract as muon_lm_ddp.py:331-370: returns a new bf16 tensor of G's shape.
    """
    if G.dim() != 2:
        raise ValueError("zeropower_serial expects a 2-D tensor")
    return _ns_call(G, ns_steps, eps, orient=True)


@torch.no_grad()
def zeropower_batched_oriented(X, ns_steps, eps):
    """Quintic Newton–Schulz of a stack X [B, m, n] used as given (muon_lm_ddp.py:373-426)."""
    if X.dim() != 3:
        raise ValueError("zeropower_batched_oriented expects [B, m, n]")
    return _ns_call(X, ns_steps, eps, orient=False)


@torch.no_grad()
def zeropower_via_newtonschulz5(G, steps=5, eps=1e-7):
    """Orthogonalise G ([rows, cols] or [B, rows, cols]); tall matrices are transposed and back."""
    return _ns_call(G, steps, eps, orient=True)


# ---------------------------------------------------------------------------
# Step engine shared by MuonAdamW and Muon
# ---------------------------------------------------------------------------

class _PtrCache:
    """Device arrays of data pointers, re-uploaded only when the pointers change."""

    def __init__(self) -> None:
        self._cache: dict[tuple, torch.Tensor] = {}

    def get(self, ptrs: tuple, device: torch.device) -> torch.Tensor:
        key = (device.index, ptrs)
        t = self._cache.get(key)
        if t is None:
            if len(self._cache) > 64:
                self._cache.clear()
            t = torch.tensor(ptrs, dtype=torch.int64).to(device)
            self._cache[key] = t
        return t


class MuonStepEngine:
    """Runs the fused Muon step over (param, grad, momentum, lr_adjusted) entries.

    Entries are grouped by (unoriented shape, adjusted lr); each group is one
    ``lsr_muon_group`` of the C ABI. ``step`` is the single-GPU path;
    ``orthogonalize`` + ``apply`` are its two halves, between which a caller
    may all-gather the oriented updates (lsr.dist).
    """

    def __init__(self) -> None:
        self.ptrs = _PtrCache()

    @staticmethod
    def group_items(items):
        by_shape: dict[tuple, list] = defaultdict(list)
        for it in items:
            by_shape[(tuple(it[0].shape), float(it[3]))].append(it)
        return [(shape, lr, its) for (shape, lr), its in by_shape.items()]

    def make_groups(self, grouped, with_grads=True):
        """ctypes array of lsr_muon_group (+ the pointer tensors that must stay alive)."""
        groups, keep = [], []
        for shape, lr, its in grouped:
            dev = its[0][0].device
            g = _lib.MuonGroup()
            g.rows, g.cols = shape
            g.count = len(its)
            pp = self.ptrs.get(tuple(x[0].data_ptr() for x in its), dev)
            g.param_ptrs = pp.data_ptr()
            keep.append(pp)
            if with_grads:
                gp = self.ptrs.get(tuple(x[1].data_ptr() for x in its), dev)
                mp = self.ptrs.get(tuple(x[2].data_ptr() for x in its), dev)
                g.grad_ptrs, g.mom_ptrs = gp.data_ptr(), mp.data_ptr()
                keep += [gp, mp]
            g.lr = lr
            groups.append(g)
        return (_lib.MuonGroup * len(groups))(*groups), keep

    def step(self, items, *, momentum, nesterov, weight_decay, base_lr, ns_steps, eps, coef=(NS_A, NS_B, NS_C)):
        if not items:
            return
        dev = items[0][0].device
        arr, keep = self.make_groups(self.group_items(items))
        lib = _lib.load()
        with _lib.on_device(dev):
            ws_bytes = lib.lsr_muon_workspace_bytes(arr, len(arr))
            ws = _lib.WORKSPACE.get(ws_bytes, dev)
            rc = lib.lsr_muon_step_bf16(arr, len(arr), float(momentum), int(bool(nesterov)), float(weight_decay),
                                        float(base_lr), int(ns_steps), float(coef[0]), float(coef[1]),
                                        float(coef[2]), float(eps), ws.data_ptr(), ws_bytes,
                                        _lib.stream_handle(dev))
        _lib.check(rc, "lsr_muon_step_bf16")
        del keep

    def orthogonalize(self, grouped, *, momentum, nesterov, ns_steps, eps, coef=(NS_A, NS_B, NS_C), out=None):
        """Momentum update + Newton–Schulz. Returns one bf16 [count, m, n] oriented update per group
        (written into ``out[g]`` when given)."""
        if not grouped:
            return []
        dev = grouped[0][2][0][0].device
        arr, keep = self.make_groups(grouped)
        if out is None:
            out = []
            for (r, c), _, its in grouped:
                out.append(torch.empty(len(its), min(r, c), max(r, c), dtype=torch.bfloat16, device=dev))
        ptrs = (ctypes.c_void_p * len(out))(*[o.data_ptr() for o in out])
        lib = _lib.load()
        with _lib.on_device(dev):
            ws_bytes = lib.lsr_muon_workspace_bytes(arr, len(arr))
            ws = _lib.WORKSPACE.get(ws_bytes, dev)
            rc = lib.lsr_muon_orthogonalize_bf16(arr, len(arr), float(momentum), int(bool(nesterov)), int(ns_steps),
                                                 float(coef[0]), float(coef[1]), float(coef[2]), float(eps), ptrs,
                                                 ws.data_ptr(), ws_bytes, _lib.stream_handle(dev))
        _lib.check(rc, "lsr_muon_orthogonalize_bf16")
        del keep
        return out

    def workspace_bytes(self, grouped) -> int:
        arr, keep = self.make_groups(grouped)
        n = _lib.load().lsr_muon_workspace_bytes(arr, len(arr))
        del keep
        return int(n)

    def orthogonalize_phase(self, grouped, phase, workspace, *, momentum, nesterov, ns_steps, eps,
                            coef=(NS_A, NS_B, NS_C), out):
        """orthogonalize() in two calls sharing `workspace` (uint8 CUDA tensor of at least
        workspace_bytes(grouped)): phase 1 = momentum / orientation / normalisation, phase 2 =
        Newton–Schulz into ``out``."""
        dev = grouped[0][2][0][0].device
        arr, keep = self.make_groups(grouped)
        ptrs = (ctypes.c_void_p * len(out))(*[o.data_ptr() for o in out])
        with _lib.on_device(dev):
            rc = _lib.load().lsr_muon_orthogonalize_phase_bf16(
                arr, len(arr), float(momentum), int(bool(nesterov)), int(ns_steps), float(coef[0]), float(coef[1]),
                float(coef[2]), float(eps), ptrs, int(phase), workspace.data_ptr(), workspace.numel(),
                _lib.stream_handle(dev))
        _lib.check(rc, "lsr_muon_orthogonalize_phase_bf16")
        del keep

    def apply(self, grouped, updates, *, weight_decay, base_lr):
        """p *= 1 - base_lr*wd ; p -= lr_adj * update, for every group (updates oriented [count, m, n])."""
        if not grouped:
            return
        dev = grouped[0][2][0][0].device
        arr, keep = self.make_groups(grouped, with_grads=False)
        for u, (shape, _, its) in zip(updates, grouped):
            if u.dtype != torch.bfloat16 or not u.is_contiguous() or tuple(u.shape) != (
                    len(its), min(shape), max(shape)):
                raise ValueError("updates must be contiguous bf16 [count, min(r,c), max(r,c)] per group")
        ptrs = (ctypes.c_void_p * len(updates))(*[u.data_ptr() for u in updates])
        with _lib.on_device(dev):
            rc = _lib.load().lsr_muon_apply_bf16(arr, len(arr), ptrs, float(weight_decay), float(base_lr),
                                                 _lib.stream_handle(dev))
        _lib.check(rc, "lsr_muon_apply_bf16")
        del keep


def _check_bf16_cuda(p: torch.Tensor, what: str) -> None:
    _lib.require_cuda(p, what)
    if p.dtype != torch.bfloat16:
        raise ValueError(f"{what}: liblsr's Muon step needs bf16 parameters (got {p.dtype})")
    if not p.is_contiguous():
        raise ValueError(f"{what}: parameters must be contiguous")


# ---------------------------------------------------------------------------
# MuonAdamW (drop-in for muon_lm_ddp.MuonAdamW)
# ---------------------------------------------------------------------------

class MuonAdamW:
    """Hybrid optimizer: Muon for 2-D hidden matrices, fused AdamW for the rest.

    Constructor, attributes and methods follow muon_lm_ddp.py:433-745. Both
    ``muon_mode="serial"`` and ``"batched"`` run the same fused liblsr step
    (every matrix of the step in one set of grouped launches); the per-matrix
    arithmetic is that of the reference, so the modes give identical results.
    ``muon_batch_matrices`` is accepted and recorded (it only sized the
    reference's torch.bmm chunks).
    """

    EMBED_LIKE_NAMES = ("wte", "wpe", "embed", "embedding", "lm_head", "output_projection", "word_embeddings",
                        "position_embeddings")

    def __init__(self, named_parameters, muon_mode, muon_lr, muon_momentum, muon_weight_decay, muon_nesterov,
                 muon_ns_steps, muon_eps, muon_lr_adjust, muon_batch_matrices, adam_lr, adam_betas,
                 adam_weight_decay, rank):
        self.muon_mode = muon_mode
        self.muon_lr = muon_lr
        self.muon_momentum = muon_momentum
        self.muon_weight_decay = muon_weight_decay
        self.muon_nesterov = muon_nesterov
        self.muon_ns_steps = muon_ns_steps
        self.muon_eps = muon_eps
        self.muon_lr_adjust = muon_lr_adjust
        self.muon_batch_matrices = muon_batch_matrices
        self.rank = rank

        named_parameters = [(n, p) for n, p in named_parameters if p.requires_grad]
        self.muon_named = []
        self.adam_named = []
        seen = set()
        for name, p in named_parameters:
            if id(p) in seen:  # tied weights
                continue
            seen.add(id(p))
            excluded = any(key in name.lower() for key in self.EMBED_LIKE_NAMES)
            if p.ndim == 2 and not excluded:
                self.muon_named.append((name, p))
            else:
                self.adam_named.append((name, p))

        self.momentum = {p: torch.zeros_like(p, memory_format=torch.preserve_format) for _, p in self.muon_named}

        adam_params = [p for _, p in self.adam_named]
        self.adam = torch.optim.AdamW(adam_params, lr=adam_lr, betas=adam_betas, weight_decay=adam_weight_decay,
                                      fused=True) if adam_params else None

        self.shape_groups = defaultdict(list)
        for name, p in self.muon_named:
            r, c = p.shape
            if r <= c:
                oriented, transpose = (r, c), False
            else:
                oriented, transpose = (c, r), True
            self.shape_groups[oriented].append((name, p, transpose))
        self._engine = MuonStepEngine()

    def zero_grad(self):
        for _, p in self.muon_named:
            p.grad = None
        if self.adam is not None:
            self.adam.zero_grad(set_to_none=True)

    def _items(self):
        items = []
        for name, p in self.muon_named:
            if p.grad is None:
                continue
            _check_bf16_cuda(p, name)
            g = p.grad
            if g.dtype != torch.bfloat16 or not g.is_contiguous():
                g = g.to(torch.bfloat16).contiguous()
            items.append((p, g, self.momentum[p], adjusted_muon_lr(self.muon_lr, p.shape, self.muon_lr_adjust)))
        return items

    @torch.no_grad()
    def muon_step_serial(self):
        self._fused_step()

    @torch.no_grad()
    def muon_step_batched(self):
        self._fused_step()

    @torch.no_grad()
    def _fused_step(self):
        self._engine.step(self._items(), momentum=self.muon_momentum, nesterov=self.muon_nesterov,
                          weight_decay=self.muon_weight_decay, base_lr=self.muon_lr, ns_steps=self.muon_ns_steps,
                          eps=self.muon_eps)

    @torch.no_grad()
    def muon_step(self):
        if self.muon_mode == "serial":
            self.muon_step_serial()
        elif self.muon_mode == "batched":
            self.muon_step_batched()
        else:
            raise ValueError(self.muon_mode)

    def adam_step(self):
        if self.adam is not None:
            self.adam.step()

    def summary(self):
        muon_params = sum(p.numel() for _, p in self.muon_named)
        adam_params = sum(p.numel() for _, p in self.adam_named)
        groups = []
        for shape, items in sorted(self.shape_groups.items()):
            groups.append({
                "oriented_shape": list(shape),
                "count": len(items),
                "matrix_million_elements_each": shape[0] * shape[1] / 1e6,
                "example_names": [x[0] for x in items[:4]],
            })
        return {
            "muon_param_count": muon_params,
            "adam_param_count": adam_params,
            "muon_matrix_count": len(self.muon_named),
            "shape_groups": groups,
        }

    def state_dict(self):
        return {
            "momentum": [self.momentum[p] for _, p in self.muon_named],
            "adam": self.adam.state_dict() if self.adam is not None else None,
        }

    def load_state_dict(self, state):
        for (_, p), buf in zip(self.muon_named, state["momentum"]):
            self.momentum[p].copy_(buf)
        if self.adam is not None and state.get("adam") is not None:
            self.adam.load_state_dict(state["adam"])


# ---------------------------------------------------------------------------
# Muon as a torch.optim.Optimizer
# ---------------------------------------------------------------------------

class Muon(torch.optim.Optimizer):
    """Muon for 2-D bf16 CUDA parameters (same arithmetic as MuonAdamW's Muon half).

    Per-group options: lr, momentum, nesterov, weight_decay, ns_steps, eps,
    lr_adjust ("original" | "match_rms_adamw" | "none"). State per parameter:
    ``momentum_buffer`` (bf16, like the reference).
    """

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.01, ns_steps=5, eps=1e-7,
                 lr_adjust="original"):
        defaults = dict(lr=lr, momentum=momentum, nesterov=nesterov, weight_decay=weight_decay, ns_steps=ns_steps,
                        eps=eps, lr_adjust=lr_adjust)
        super().__init__(params, defaults)
        for group in self.param_groups:
            for p in group["params"]:
                if p.ndim != 2:
                    raise ValueError("Muon only handles 2-D parameters")
        self._engine = MuonStepEngine()

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            items = []
            for p in group["params"]:
                if p.grad is None:
                    continue
                _check_bf16_cuda(p, "Muon parameter")
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                g = p.grad
                if g.dtype != torch.bfloat16 or not g.is_contiguous():
                    g = g.to(torch.bfloat16).contiguous()
                items.append((p, g, st["momentum_buffer"],
                              adjusted_muon_lr(group["lr"], p.shape, group["lr_adjust"])))
            self._engine.step(items, momentum=group["momentum"], nesterov=group["nesterov"],
                              weight_decay=group["weight_decay"], base_lr=group["lr"], ns_steps=group["ns_steps"],
                              eps=group["eps"])
        return loss


__all__ = [
    "NS_A", "NS_B", "NS_C", "adjusted_muon_lr", "zeropower_serial", "zeropower_batched_oriented",
    "zeropower_via_newtonschulz5", "MuonAdamW", "Muon", "MuonStepEngine",
]
