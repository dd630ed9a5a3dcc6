"""Shampoo / SOAP on B200 behind the constructor the reference uses.

The reference builds ``DistributedShampoo(params, lr, betas, epsilon,
weight_decay, max_preconditioner_dim, precondition_frequency,
start_preconditioning_step, weight_decay_type=WeightDecayType.DECOUPLED,
distributed_config=DDPDistributedConfig(...), grafting_config=
AdamPreconditionerConfig(...) | preconditioner_config=DefaultSOAPConfig)``
(shampoo_soap_lm_ddp_zero1.py:312-400) from the third-party
distributed_shampoo package. This module accepts the same arguments and
config objects and runs the preconditioner math in liblsr:

* parameters are cut into blocks of at most ``max_preconditioner_dim`` per
  side (1600 -> 1024 + 576); blocks of equal shape across all parameters are
  stacked and processed by one call per shape (``lsr_blocks_gather_bf16``);
* statistics L, R (fp32, EMA with betas[1]): ``lsr_gram_update_f32``;
* Shampoo direction L^{-1/4} G R^{-1/4}: ``lsr_shampoo_direction_bf16``, with
  Adam grafting (the direction takes the Frobenius norm of the Adam direction,
  per block) and a first-moment filter with betas[0];
* SOAP direction Q_L^T G Q_R -> Adam (m, v in the rotated basis) -> Q_L U' Q_R^T:
  ``lsr_soap_direction_bf16``;
* decoupled weight decay and the update: ``lsr_blocks_apply_bf16``;
* at every multiple of ``precondition_frequency`` from
  ``start_preconditioning_step`` on (the reference's periodic steps) the
  inverse roots / eigenbases are recomputed from L, R (before the first one
  Shampoo uses the grafting direction and SOAP the identity basis): SOAP's
  eigenbases by power iteration with a Householder QR from the current basis
  (``lsr_eigenbasis_refresh_f32``; ``amortized_computation=False`` uses an fp32
  ``torch.linalg.eigh`` instead), Shampoo's inverse 4th roots by the batched
  coupled Newton kernel (``lsr.newton``, the recurrence of shampoo.py:277-542,
  all blocks of one shape in one call; ``root_inverse_method="eigh"`` uses an
  eigendecomposition instead);
* with ``DDPDistributedConfig`` and an initialised process group the blocks
  are owned by ranks (greedy by flops, ZeRO-1: state only for owned blocks),
  directions are all-gathered in ``communication_dtype`` and every rank
  applies them.

Non-matrix parameters (biases, norms) take the grafting Adam step (torch ops).
Matrix parameters must be bf16 CUDA tensors.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


class WeightDecayType(enum.Enum):
    DECOUPLED = "decoupled"
    L2 = "l2"


@dataclass
class AdamPreconditionerConfig:
    beta2: float = 0.999
    epsilon: float = 1e-8


@dataclass
class DDPDistributedConfig:
    # float16, the reference script's default (shampoo_soap_lm_ddp_zero1.py:429-434)
    communication_dtype: torch.dtype = torch.float16
    num_trainers_per_group: int = -1
    communicate_params: bool = False


@dataclass
class EigenvalueCorrectedShampooConfig:
    """SOAP: Adam in the eigenbasis of the Shampoo factors.

    amortized_computation=True (the default, as DefaultSOAPConfig's amortized eigenbasis
    computation): every refresh takes ``max_iterations`` steps of power iteration with a
    Householder QR from the current basis (``first_iterations`` on the first refresh, which
    starts from the identity), on liblsr's kernels (lsr_eigenbasis_refresh_f32).
    amortized_computation=False: an fp32 eigendecomposition per refresh (torch.linalg.eigh)."""
    amortized_computation: bool = True
    max_iterations: int = 1
    first_iterations: int = 4


DefaultSOAPConfig = EigenvalueCorrectedShampooConfig()
DefaultEigenvalueCorrectedShampooConfig = DefaultSOAPConfig


def block_sizes(n: int, max_dim: int) -> list[int]:
    out = [max_dim] * (n // max_dim)
    if n % max_dim:
        out.append(n % max_dim)
    return out


def param_blocks(shape, max_dim):
    """[(r0, c0, r, c)] of a 2-D parameter, row-major block order."""
    rows, cols = shape
    out, r0 = [], 0
    for r in block_sizes(rows, max_dim):
        c0 = 0
        for c in block_sizes(cols, max_dim):
            out.append((r0, c0, r, c))
            c0 += c
        r0 += r
    return out


def assign_owners(costs: list[float], world: int) -> list[int]:
    """Greedy longest-processing-time assignment of blocks to ranks (deterministic)."""
    load = [0.0] * world
    owner = [0] * len(costs)
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += costs[i]
    return owner


class _BlockGroup:
    """All owned blocks of one shape, stacked."""

    def __init__(self, shape, refs, device, soap: bool):
        self.shape = shape
        self.refs = refs  # [(param, r0, c0)]
        r, c = shape
        n = len(refs)
        self.L = torch.zeros(n, r, r, dtype=torch.float32, device=device)
        self.R = torch.zeros(n, c, c, dtype=torch.float32, device=device)
        eye_r = torch.eye(r, device=device, dtype=torch.bfloat16).expand(n, r, r).contiguous()
        eye_c = torch.eye(c, device=device, dtype=torch.bfloat16).expand(n, c, c).contiguous()
        self.QL, self.QR = eye_r, eye_c  # SOAP eigenbases or Shampoo inverse roots (bf16)
        self.QLf = self.QRf = None  # SOAP: fp32 master bases of the amortized refresh
        self.have_roots = False
        self.m = torch.zeros(n, r, c, dtype=torch.float32, device=device)  # SOAP m / Shampoo filtered grad
        self.v = torch.zeros(n, r, c, dtype=torch.float32, device=device)  # SOAP v / grafting v
        self.stack = torch.empty(n, r, c, dtype=torch.bfloat16, device=device)
        self.U = torch.empty(n, r, c, dtype=torch.float32, device=device)
        self._ptr_key = None
        self._grad_key = None
        self.adam_sq = self.u_sq = self.gf = None  # Shampoo grafting buffers, made on first use

    def pointers(self):
        """Device arrays of the blocks' parameter and gradient addresses and row strides,
        rebuilt (a small host-to-device copy) only when a tensor has moved."""
        key = tuple(p.data_ptr() for p, _, _ in self.refs)
        if key != self._ptr_key:
            dev = self.stack.device
            self.data_ptrs = torch.tensor(
                [p.data_ptr() + 2 * (r0 * p.shape[1] + c0) for p, r0, c0 in self.refs], dtype=torch.int64).to(dev)
            self.lds = torch.tensor([p.shape[1] for p, _, _ in self.refs], dtype=torch.int32).to(dev)
            self._ptr_key = key
        gkey = tuple(p.grad.data_ptr() for p, _, _ in self.refs)
        if gkey != self._grad_key:
            self.grad_ptrs = torch.tensor([p.grad.data_ptr() + 2 * (r0 * p.shape[1] + c0) for p, r0, c0 in self.refs],
                                          dtype=torch.int64).to(self.stack.device)
            self._grad_key = gkey
        return self.data_ptrs, self.lds, self.grad_ptrs


class DistributedShampoo(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-2, betas=(0.9, 1.0), epsilon=1e-12, weight_decay=0.0,
                 max_preconditioner_dim=1024, precondition_frequency=1, start_preconditioning_step=-1,
                 weight_decay_type=WeightDecayType.DECOUPLED, distributed_config: Optional[DDPDistributedConfig] = None,
                 grafting_config: Optional[AdamPreconditionerConfig] = None, preconditioner_config=None,
                 eager_nan_check: bool = False, root_inverse_method: str = "coupled_newton", **unused):
        if weight_decay_type != WeightDecayType.DECOUPLED:
            raise ValueError("only WeightDecayType.DECOUPLED is supported")
        if max_preconditioner_dim % 8:
            raise ValueError("max_preconditioner_dim must be a multiple of 8")
        defaults = dict(lr=lr, betas=betas, epsilon=epsilon, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.soap = isinstance(preconditioner_config, EigenvalueCorrectedShampooConfig)
        self.soap_cfg = preconditioner_config if self.soap else None
        if root_inverse_method not in ("eigh", "coupled_newton"):
            raise ValueError(f"root_inverse_method must be 'eigh' or 'coupled_newton', got {root_inverse_method!r}")
        self.root_inverse_method = root_inverse_method
        self.grafting = grafting_config or AdamPreconditionerConfig(beta2=betas[1], epsilon=1e-8)
        self.max_dim = max_preconditioner_dim
        self.freq = max(1, precondition_frequency)
        self.start = start_preconditioning_step if start_preconditioning_step >= 0 else self.freq
        self.dcfg = distributed_config
        self.world = dist.get_world_size() if (distributed_config is not None and dist.is_initialized()) else 1
        self.rank = dist.get_rank() if self.world > 1 else 0
        self.step_count = 0
        self._groups = None
        self._comm_dtype = distributed_config.communication_dtype if distributed_config else torch.float32
        if self._comm_dtype not in _lib.DTYPE_CODES:
            raise ValueError(f"communication_dtype must be float32, bfloat16 or float16, got {self._comm_dtype}")
        self._ex: dict = {}
        self._comm_stream = None
        self._pending_comm = False

    # ------------------------------------------------------------------ setup
    def _matrix_params(self):
        out = []
        for g in self.param_groups:
            for p in g["params"]:
                if p.ndim == 2:
                    out.append((p, g))
        return out

    def _build(self):
        entries = []  # (param, r0, c0, r, c)
        for p, _ in self._matrix_params():
            _lib.require_cuda(p, "parameter")
            if p.dtype != torch.bfloat16 or not p.is_contiguous():
                raise ValueError("matrix parameters must be contiguous bf16 CUDA tensors")
            if p.shape[1] % 8:
                raise ValueError("parameter row length must be a multiple of 8")
            for r0, c0, r, c in param_blocks(p.shape, self.max_dim):
                entries.append((p, r0, c0, r, c))
        costs = [6.0 * r * c * (r + c) for _, _, _, r, c in entries]
        self.owner = assign_owners(costs, self.world)
        by_shape: dict[tuple, list] = {}
        for e, o in zip(entries, self.owner):
            by_shape.setdefault((e[3], e[4]), []).append((e, o))
        self._groups = []
        self._all_blocks = {}
        # largest block shapes first: the exchange left after the last shape's compute is the smallest
        for shape, lst in sorted(by_shape.items(), key=lambda kv: (-kv[0][0] * kv[0][1] * (kv[0][0] + kv[0][1]),
                                                                    kv[0])):
            owned = [(e[0], e[1], e[2]) for e, o in lst if o == self.rank]
            grp = _BlockGroup(shape, owned, entries[0][0].device, self.soap) if owned else None
            self._groups.append((shape, grp, lst))

    # ------------------------------------------------------------------ periodic refresh
    def _refresh(self, grp: _BlockGroup, eps: float):
        r, c = grp.shape
        if self.soap and self.soap_cfg.amortized_computation:
            self._refresh_amortized(grp, eps)
        elif self.soap:
            eye_r = torch.eye(r, device=grp.L.device)
            eye_c = torch.eye(c, device=grp.R.device)
            _, QL = torch.linalg.eigh(grp.L + eps * eye_r)
            _, QR = torch.linalg.eigh(grp.R + eps * eye_c)
            grp.QL, grp.QR = QL.bfloat16().contiguous(), QR.bfloat16().contiguous()
        elif self.root_inverse_method == "coupled_newton":
            from .newton import batched_coupled_newton
            grp.QL = batched_coupled_newton(grp.L, 4, epsilon=eps)[0].bfloat16().contiguous()
            grp.QR = batched_coupled_newton(grp.R, 4, epsilon=eps)[0].bfloat16().contiguous()
        else:
            eye_r = torch.eye(r, device=grp.L.device)
            eye_c = torch.eye(c, device=grp.R.device)

            def root(S, I):
                w, V = torch.linalg.eigh(S + eps * I)
                return (V * w.clamp_min(1e-30).pow(-0.25).unsqueeze(-2)) @ V.transpose(-1, -2)
            grp.QL = root(grp.L, eye_r).bfloat16().contiguous()
            grp.QR = root(grp.R, eye_c).bfloat16().contiguous()
        grp.have_roots = True

    # blocks per refresh call: bounds the transient workspace (the W buffer and the
    # tf32 pairs of the fp32 GEMM, about 6 n^2 fp32 values per block)
    REFRESH_CHUNK = 128

    def _refresh_amortized(self, grp: _BlockGroup, eps: float):
        """Power iteration with Householder QR on liblsr's kernels, from the fp32 master bases
        (identity before the first refresh); bf16 copies for the SOAP chain."""
        lib = _lib.load()
        n = len(grp.refs)
        first = grp.QLf is None
        if first:
            grp.QLf = torch.empty(n, grp.shape[0], grp.shape[0], dtype=torch.float32, device=grp.L.device)
            grp.QRf = torch.empty(n, grp.shape[1], grp.shape[1], dtype=torch.float32, device=grp.R.device)
        iters = self.soap_cfg.first_iterations if first else self.soap_cfg.max_iterations
        st = _lib.stream_handle(grp.L.device)
        for S, Qf, Qb in ((grp.L, grp.QLf, grp.QL), (grp.R, grp.QRf, grp.QR)):
            k = S.shape[-1]
            for b0 in range(0, n, self.REFRESH_CHUNK):
                nb_ = min(self.REFRESH_CHUNK, n - b0)
                nbytes = lib.lsr_eigenbasis_refresh_workspace_bytes(nb_, k)
                ws = _lib.WORKSPACE.get(nbytes, S.device)
                _lib.check(lib.lsr_eigenbasis_refresh_f32(
                    S[b0:b0 + nb_].data_ptr(), Qf[b0:b0 + nb_].data_ptr(), Qb[b0:b0 + nb_].data_ptr(), nb_, k, eps,
                    int(first), max(1, iters), ws.data_ptr(), nbytes, st), "lsr_eigenbasis_refresh_f32")

    def is_refresh_step(self, t: int) -> bool:
        """True when 1-based step t recomputes the roots / eigenbases: from the start step on, at every
        multiple of the frequency (every step when it is 1). This is the schedule the reference times
        as its periodic steps (shampoo_soap_lm_ddp_zero1.py:622-632)."""
        return t >= self.start and (t % self.freq == 0 or self.freq == 1)

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._groups is None:
            self._build()
        self.step_count += 1
        t = self.step_count
        g0 = self.param_groups[0]
        lr, (b1, b2), eps, wd = g0["lr"], g0["betas"], g0["epsilon"], g0["weight_decay"]
        lib = _lib.load()
        precondition = t >= self.start
        refresh = self.is_refresh_step(t)
        for shape, grp, lst in self._groups:
            r, c = shape
            if grp is not None:
                dev = grp.stack.device
                st = _lib.stream_handle(dev)
                pptrs, lds, gptrs = grp.pointers()
                n = len(grp.refs)
                _lib.check(lib.lsr_blocks_gather_bf16(gptrs.data_ptr(), lds.data_ptr(), n, r, c,
                                                      grp.stack.data_ptr(), st), "lsr_blocks_gather_bf16")
                _lib.check(lib.lsr_gram_update_f32(grp.stack.data_ptr(), grp.L.data_ptr(), n, r, c, 0, b2, 1 - b2, st),
                           "lsr_gram_update_f32")
                _lib.check(lib.lsr_gram_update_f32(grp.stack.data_ptr(), grp.R.data_ptr(), n, r, c, 1, b2, 1 - b2, st),
                           "lsr_gram_update_f32")
                if refresh:
                    self._refresh(grp, eps)
                if self.soap:
                    nb = lib.lsr_soap_workspace_bytes(n, r, c)
                    ws = _lib.WORKSPACE.get(nb, dev)
                    _lib.check(lib.lsr_soap_direction_bf16(
                        grp.stack.data_ptr(), None, None, grp.QL.data_ptr(), grp.QR.data_ptr(), grp.m.data_ptr(),
                        grp.v.data_ptr(), grp.U.data_ptr(), n, r, c, b1, b2, self.grafting.epsilon, t, 0,
                        ws.data_ptr(), nb, st), "lsr_soap_direction_bf16")
                else:
                    self._shampoo_direction(grp, n, r, c, b1, t, precondition and grp.have_roots)
            self._exchange_and_apply(shape, grp, lst, lr, wd)
        if self._pending_comm:
            # the send buffers are rewritten by the next step and the parameters read by what follows:
            # the compute stream waits for every exchange and apply of this step
            torch.cuda.current_stream().wait_stream(self._comm_stream)
            self._pending_comm = False
        self._adam_non_matrix(t)
        return loss

    def _shampoo_direction(self, grp, n, r, c, b1, t, precondition):
        """First-moment filter, Adam grafting and (after the first inverse roots) the grafted Shampoo
        direction, all in liblsr: the prepare pass updates m, v and writes the filtered gradient (bf16,
        the apply's operand) and the per-block Adam norms; the apply runs L^-1/4 Gf R^-1/4; the scale
        pass gives each block the Frobenius norm of its Adam direction."""
        lib = _lib.load()
        st = _lib.stream_handle(grp.stack.device)
        tiles = lib.lsr_graft_tiles(r, c)
        if grp.adam_sq is None:
            dev = grp.stack.device
            grp.adam_sq = torch.empty(n, tiles, dtype=torch.float32, device=dev)
            grp.u_sq = torch.empty(n, tiles, dtype=torch.float32, device=dev)
            grp.gf = torch.empty(n, r, c, dtype=torch.bfloat16, device=dev)
        gb2, geps = self.grafting.beta2, self.grafting.epsilon
        _lib.check(lib.lsr_shampoo_graft_prepare_bf16(
            grp.stack.data_ptr(), grp.m.data_ptr() if b1 > 0 else None, grp.v.data_ptr(), grp.gf.data_ptr(),
            None if precondition else grp.U.data_ptr(), grp.adam_sq.data_ptr(), n, r, c, b1, gb2, geps, t, st),
            "lsr_shampoo_graft_prepare_bf16")
        if not precondition:
            return
        nb = lib.lsr_shampoo_workspace_bytes(n, r, c)
        ws = _lib.WORKSPACE.get(nb, grp.stack.device)
        _lib.check(lib.lsr_shampoo_direction_bf16(grp.gf.data_ptr(), None, None, grp.QL.data_ptr(), grp.QR.data_ptr(),
                                                  grp.U.data_ptr(), n, r, c, 0.0, 0, ws.data_ptr(), nb, st),
                   "lsr_shampoo_direction_bf16")
        _lib.check(lib.lsr_shampoo_graft_scale_f32(grp.U.data_ptr(), grp.adam_sq.data_ptr(), grp.u_sq.data_ptr(),
                                                   n, r, c, st), "lsr_shampoo_graft_scale_f32")

    def _exchange_state(self, shape, lst):
        """Persistent ZeRO-1 exchange buffers of one block shape: send [per][r][c] and recv
        [world*per][r][c] in the communication dtype (padding slots stay zero), and the device arrays
        that map every real recv slot to its parameter block (address, row stride, slot index)."""
        st = self._ex.get(shape)
        if st is not None and st["key"] == tuple(e[0].data_ptr() for e, _ in lst):
            return st
        r, c = shape
        dev = lst[0][0][0].device
        counts = [sum(1 for _, o in lst if o == k) for k in range(self.world)]
        per = max(counts)
        refs, slots = [], []
        for k in range(self.world):
            mine = [e for e, o in lst if o == k]
            for j, e in enumerate(mine):
                refs.append(e)
                slots.append(k * per + j)
        st = {
            "key": tuple(e[0].data_ptr() for e, _ in lst),
            "send": torch.zeros(per, r, c, dtype=self._comm_dtype, device=dev),
            "recv": torch.empty(self.world * per, r, c, dtype=self._comm_dtype, device=dev),
            "ptrs": torch.tensor([e[0].data_ptr() + 2 * (e[1] * e[0].shape[1] + e[2]) for e in refs],
                                 dtype=torch.int64).to(dev),
            "lds": torch.tensor([e[0].shape[1] for e in refs], dtype=torch.int32).to(dev),
            "slots": torch.tensor(slots, dtype=torch.int32).to(dev),
            "n": len(refs),
        }
        self._ex[shape] = st
        return st

    def _exchange_and_apply(self, shape, grp, lst, lr, wd):
        lib = _lib.load()
        r, c = shape
        if self.world == 1:
            pptrs, lds, _ = grp.pointers()
            _lib.check(lib.lsr_blocks_apply_bf16(pptrs.data_ptr(), lds.data_ptr(), len(grp.refs), r, c,
                                                 grp.U.data_ptr(), lr, wd, _lib.stream_handle(grp.U.device)),
                       "lsr_blocks_apply_bf16")
            return
        # ZeRO-1: this rank's directions go into the persistent send buffer (in the communication dtype)
        # on the compute stream; the all-gather and the apply of every rank's directions run on the comm
        # stream, overlapped with the next block shape's compute.
        ex = self._exchange_state(shape, lst)
        compute = torch.cuda.current_stream()
        if grp is not None:
            ex["send"][:len(grp.refs)].copy_(grp.U)
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device=compute.device)
        comm = self._comm_stream
        ev = torch.cuda.Event()
        ev.record(compute)
        comm.wait_event(ev)
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(ex["recv"], ex["send"])
            _lib.check(lib.lsr_blocks_apply_any(ex["ptrs"].data_ptr(), ex["lds"].data_ptr(), ex["n"], r, c,
                                                ex["recv"].data_ptr(), _lib.DTYPE_CODES[self._comm_dtype],
                                                ex["slots"].data_ptr(), lr, wd, comm.cuda_stream),
                       "lsr_blocks_apply_any")
        self._pending_comm = True

    def _adam_non_matrix(self, t):
        gb2, geps = self.grafting.beta2, self.grafting.epsilon
        for g in self.param_groups:
            lr, (b1, _), wd = g["lr"], g["betas"], g["weight_decay"]
            for p in g["params"]:
                if p.ndim == 2 or p.grad is None:
                    continue
                st = self.state[p]
                if "exp_avg" not in st:
                    st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                    st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
                gr = p.grad.float()
                st["exp_avg"].mul_(b1).add_(gr, alpha=1 - b1)
                st["exp_avg_sq"].mul_(gb2).addcmul_(gr, gr, value=1 - gb2)
                d = (st["exp_avg"] / (1 - b1 ** t)) / ((st["exp_avg_sq"] / (1 - gb2 ** t)).sqrt() + geps)
                if wd:
                    p.mul_(1 - lr * wd)
                p.add_(d.to(p.dtype), alpha=-lr)


def soap_direction(G, L, R, QL, QR, m, v, beta1, beta2, eps, step, update_stats=True):
    """Functional SOAP direction on a block stack (all CUDA): returns U (fp32); L, R, m, v updated in place."""
    lib = _lib.load()
    n, r, c = G.shape
    U = torch.empty(n, r, c, dtype=torch.float32, device=G.device)
    nb = lib.lsr_soap_workspace_bytes(n, r, c)
    ws = _lib.WORKSPACE.get(nb, G.device)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.check(lib.lsr_soap_direction_bf16(G.data_ptr(), ptr(L), ptr(R), QL.data_ptr(), QR.data_ptr(), m.data_ptr(),
                                           v.data_ptr(), U.data_ptr(), n, r, c, beta1, beta2, eps, step,
                                           int(update_stats), ws.data_ptr(), nb, _lib.stream_handle(G.device)),
               "lsr_soap_direction_bf16")
    return U


def shampoo_direction(G, Lroot, Rroot, L=None, R=None, beta2=0.0, update_stats=False):
    """Functional Shampoo preconditioner apply Lroot G Rroot on a block stack; returns P (fp32)."""
    lib = _lib.load()
    n, r, c = G.shape
    P = torch.empty(n, r, c, dtype=torch.float32, device=G.device)
    nb = lib.lsr_shampoo_workspace_bytes(n, r, c)
    ws = _lib.WORKSPACE.get(nb, G.device)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.check(lib.lsr_shampoo_direction_bf16(G.data_ptr(), ptr(L), ptr(R), Lroot.data_ptr(), Rroot.data_ptr(),
                                              P.data_ptr(), n, r, c, beta2, int(update_stats), ws.data_ptr(), nb,
                                              _lib.stream_handle(G.device)), "lsr_shampoo_direction_bf16")
    return P


def gram_update(G, S, side, beta, alpha):
    """S = beta S + alpha G G^T (side 0) or G^T G (side 1), fp32 S, bf16 G stack."""
    lib = _lib.load()
    n, r, c = G.shape
    _lib.check(lib.lsr_gram_update_f32(G.data_ptr(), S.data_ptr(), n, r, c, side, beta, alpha,
                                       _lib.stream_handle(G.device)), "lsr_gram_update_f32")
    return S


__all__ = ["WeightDecayType", "AdamPreconditionerConfig", "DDPDistributedConfig", "DefaultSOAPConfig",
           "DefaultEigenvalueCorrectedShampooConfig", "EigenvalueCorrectedShampooConfig", "DistributedShampoo",
           "soap_direction", "shampoo_direction", "gram_update", "param_blocks", "assign_owners", "block_sizes"]

