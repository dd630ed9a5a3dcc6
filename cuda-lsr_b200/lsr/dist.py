"""ZeRO-1-style sharded Muon across the GPUs of one node.

Ownership (the distribution of shard_groups): within each group of equally
shaped matrices, matrix j is owned by rank j % world (round-robin, so every
rank owns an equal, flop-balanced share when the group count divides by the
world size; otherwise the last slots are padding). Each rank keeps the
momentum of its own matrices only (ZeRO-1 optimizer-state sharding) and runs
the momentum update and Newton–Schulz for them.

Exchange of the results, per shape group, overlapped with the next group's
Newton–Schulz on the compute stream:

* flat_params with exchange="peer": every group's
  parameters live in one rank-major buffer in CUDA IPC memory; a rank applies
  its own updates and stores its shard straight into every peer's replica
  (lsr_peer_push, a kernel that runs beside the GEMM kernels), then the ranks
  meet at one barrier per step;
* flat_params with exchange="nccl" (the default): the same layout, in-place
  NCCL all-gather;
* flat_params=False: the oriented bf16 updates are all-gathered with NCCL and
  every rank applies all of them to its own parameter storage.

The reference replicates Muon on every DDP rank (muon_lm_ddp.py:615-683); this
module is the sharded replacement. Its host logic (ownership, gather order,
padding) is independent of the CUDA engine, which is injectable for CPU tests.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import _lib
from .muon import NS_A, NS_B, NS_C, MuonStepEngine, adjusted_muon_lr


def owner_of(j: int, world: int) -> int:
    return j % world


def local_count(count: int, world: int) -> int:
    """Slots per rank for a group of `count` matrices (ceil; padding when uneven)."""
    return (count + world - 1) // world


def gathered_order(count: int, world: int) -> list[int | None]:
    """Matrix index held by each slot of the rank-major all-gather buffer (None = padding)."""
    per = local_count(count, world)
    order: list[int | None] = []
    for r in range(world):
        for k in range(per):
            j = k * world + r
            order.append(j if j < count else None)
    return order


class IpcBuffer:
    """`nbytes` of device memory from lsr_ipc_alloc (cudaMalloc + CUDA IPC
    export). ``tensor()`` views it as a uint8 torch tensor that keeps this
    object (and so the memory) alive."""

    def __init__(self, nbytes: int, device: torch.device):
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with _lib.on_device(device):
            _lib.check(lib.lsr_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "lsr_ipc_alloc")
        self.ptr = int(ptr.value)
        self.nbytes = nbytes
        self.device = device
        self.handle = bytes(handle)
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (self.ptr, False),
                                         "version": 3, "strides": None}

    def tensor(self) -> torch.Tensor:
        return torch.as_tensor(self, device=self.device)

    def __del__(self):
        if getattr(self, "ptr", 0):
            try:
                _lib.load().lsr_ipc_free(self.ptr)
            except Exception:
                pass
            self.ptr = 0


class PeerExchange:
    """Replicated flat buffers in CUDA IPC memory, one per shape group.

    Collective setup: every rank allocates the same buffer sizes, the IPC
    handles are exchanged with all_gather_object and each rank maps the
    others' buffers. ``push(i, offset, nbytes, stream)`` stores bytes
    [offset, offset + nbytes) of local buffer i into every peer's buffer i at
    the same offset. ``close()`` (collective) unmaps the peers' buffers."""

    def __init__(self, sizes: list[int], device: torch.device, rank: int, world: int, pg=None):
        lib = _lib.load()
        self.rank, self.world, self.pg = rank, world, pg
        self.bufs = [IpcBuffer(nb, device) for nb in sizes]
        handles: list = [None] * world
        dist.all_gather_object(handles, [b.handle for b in self.bufs], group=pg)
        self.mapped: list[list[int]] = []
        self.deltas = []
        try:
            for i, b in enumerate(self.bufs):
                row = []
                # peers listed from rank + 1 on: at any moment the ranks store into distinct receivers
                for q in [(rank + k) % world for k in range(1, world)]:
                    p = ctypes.c_void_p()
                    with _lib.on_device(device):
                        _lib.check(lib.lsr_ipc_open(handles[q][i], ctypes.byref(p)), "lsr_ipc_open")
                    row.append(int(p.value))
                self.mapped.append(row)
                self.deltas.append((ctypes.c_longlong * max(len(row), 1))(*[pp - b.ptr for pp in row]))
        except Exception:
            self._unmap()
            raise

    def tensor(self, i: int) -> torch.Tensor:
        return self.bufs[i].tensor()

    def push(self, i: int, offset: int, nbytes: int, stream: torch.cuda.Stream) -> None:
        npeers = len(self.mapped[i])
        _lib.check(_lib.load().lsr_peer_push(self.bufs[i].ptr + offset, nbytes, self.deltas[i], npeers, 0,
                                             stream.cuda_stream), "lsr_peer_push")

    def _unmap(self) -> None:
        lib = _lib.load()
        for row in self.mapped:
            for p in row:
                lib.lsr_ipc_close(p)
        self.mapped = []

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.pg)  # nobody stores into a replica any more
        self._unmap()
        dist.barrier(group=self.pg)  # every mapping of every buffer is gone before it may be freed


@dataclass
class ShardGroup:
    shape: tuple
    lr: float
    params: list            # all matrices of the group, in model order
    owned: list = field(default_factory=list)  # indices j owned by this rank
    momentum: list = field(default_factory=list)  # momentum buffers of the owned matrices
    local_buf: torch.Tensor | None = None   # [per, m, n] oriented updates of this rank
    gather_buf: torch.Tensor | None = None  # [world * per, m, n]
    flat_buf: torch.Tensor | None = None    # flat mode: parameters, rank-major [world * per, r, c]
    own_slice: torch.Tensor | None = None   # flat mode: this rank's slots of flat_buf
    ws: torch.Tensor | None = None          # workspace kept between the two orthogonalize phases


class ShardedMuon:
    """Muon step sharded over the ranks of `group` (default: the world).

    params: list of 2-D bf16 CUDA parameters (all ranks pass the same list in
    the same order). Gradients are read from ``p.grad`` of the owned matrices.

    flat_params=True re-homes each shape group's parameters into one
    rank-major buffer (``p.data`` becomes a view of it, like a flat-parameter
    ZeRO layout): each rank then applies only its own updates and the updated
    parameters are all-gathered in place, so no rank applies another rank's
    updates. flat_params=False keeps the caller's storage: the oriented
    updates are all-gathered and every rank applies all of them.
    """

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.01, ns_steps=5, eps=1e-7,
                 lr_adjust="original", process_group=None, engine=None, overlap=True, flat_params=False,
                 exchange="nccl"):
        self.lr, self.mu, self.nesterov, self.wd = lr, momentum, nesterov, weight_decay
        self.ns_steps, self.eps, self.lr_adjust = ns_steps, eps, lr_adjust
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.engine = engine if engine is not None else MuonStepEngine()
        self.overlap = overlap
        by_key: dict[tuple, ShardGroup] = {}
        for p in params:
            if p.ndim != 2:
                raise ValueError("ShardedMuon only handles 2-D parameters")
            key = (tuple(p.shape), adjusted_muon_lr(lr, p.shape, lr_adjust))
            if key not in by_key:
                by_key[key] = ShardGroup(shape=key[0], lr=key[1], params=[])
            by_key[key].params.append(p)
        self.groups = list(by_key.values())
        for G in self.groups:
            G.owned = [j for j in range(len(G.params)) if owner_of(j, self.world) == self.rank]
            G.momentum = [torch.zeros_like(G.params[j]) for j in G.owned]
            per = local_count(len(G.params), self.world)
            m, n = min(G.shape), max(G.shape)
            dev = G.params[0].device
            G.local_buf = torch.zeros(per, m, n, dtype=torch.bfloat16, device=dev)
            G.gather_buf = torch.zeros(self.world * per, m, n, dtype=torch.bfloat16, device=dev) \
                if self.world > 1 else G.local_buf
        on_gpu = all(p.is_cuda for G in self.groups for p in G.params)
        self.comm_stream = torch.cuda.Stream() if (self.world > 1 and on_gpu) else None
        self.flat = bool(flat_params) and self.world > 1
        if exchange not in ("peer", "nccl"):
            raise ValueError(f"exchange must be 'peer' or 'nccl', got {exchange!r}")
        self.peer = None
        if self.flat and on_gpu and exchange == "peer":
            if any(G.params[0].dtype != torch.bfloat16 for G in self.groups):
                raise ValueError("the peer exchange handles bf16 parameters")
            sizes = [local_count(len(G.params), self.world) * self.world * G.params[0].numel() * 2
                     for G in self.groups]
            self.peer = PeerExchange(sizes, self.groups[0].params[0].device, self.rank, self.world, self.pg)
        if self.flat:
            for gi, G in enumerate(self.groups):
                order = gathered_order(len(G.params), self.world)
                p0 = G.params[0]
                shape = (len(order),) + tuple(G.shape)
                if self.peer is not None:
                    G.flat_buf = self.peer.tensor(gi).view(torch.bfloat16).view(shape)
                    G.flat_buf.zero_()
                else:
                    G.flat_buf = torch.zeros(shape, dtype=p0.dtype, device=p0.device)
                for k, j in enumerate(order):
                    if j is not None:
                        G.flat_buf[k].copy_(G.params[j].data)
                        G.params[j].data = G.flat_buf[k]
                per = local_count(len(G.params), self.world)
                G.own_slice = G.flat_buf[self.rank * per:(self.rank + 1) * per]
        # flat mode runs the groups largest first, so that the exchange left
        # after the last group's compute is the smallest one
        self.flat_order = sorted(range(len(self.groups)),
                                 key=lambda gi: -len(self.groups[gi].params) * self.groups[gi].params[0].numel())
        self._bar = torch.zeros(1, dtype=torch.int32, device=self.groups[0].params[0].device) \
            if self.peer is not None else None

    def close(self) -> None:
        """Collective: release the peer mappings (flat mode with the peer exchange)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def state_dict(self):
        return {"momentum": [[b for b in G.momentum] for G in self.groups], "rank": self.rank, "world": self.world}

    def load_state_dict(self, state):
        if state["world"] != self.world or state["rank"] != self.rank:
            raise ValueError("momentum shards were saved with a different world size / rank")
        for G, bufs in zip(self.groups, state["momentum"]):
            for dst, src in zip(G.momentum, bufs):
                dst.copy_(src)

    def _orthogonalize(self, G: ShardGroup, phase: int = 3) -> None:
        """phase 3: momentum + Newton–Schulz; phase 1 / 2: the two halves, sharing G.ws."""
        items = [(G.params[j], G.params[j].grad, G.momentum[k], G.lr) for k, j in enumerate(G.owned)]
        if any(it[1] is None for it in items):
            raise RuntimeError("ShardedMuon: every owned parameter needs a gradient")
        if not items:
            return
        grouped = [(G.shape, G.lr, items)]
        kw = dict(momentum=self.mu, nesterov=self.nesterov, ns_steps=self.ns_steps, eps=self.eps,
                  coef=(NS_A, NS_B, NS_C), out=[G.local_buf[:len(items)]])
        if phase == 3:
            self.engine.orthogonalize(grouped, **kw)
            return
        if G.ws is None:
            G.ws = torch.empty(self.engine.workspace_bytes(grouped) + 256, dtype=torch.uint8,
                               device=items[0][0].device)
        self.engine.orthogonalize_phase(grouped, phase, G.ws, **kw)

    def _apply(self, G: ShardGroup) -> None:
        order = gathered_order(len(G.params), self.world)
        slots = [k for k, j in enumerate(order) if j is not None]
        items = [(G.params[order[k]], None, None, G.lr) for k in slots]
        if len(slots) == len(order):
            upd = G.gather_buf
        else:
            upd = G.gather_buf[torch.tensor(slots, device=G.gather_buf.device)].contiguous()
        self.engine.apply([(G.shape, G.lr, items)], [upd], weight_decay=self.wd, base_lr=self.lr)

    def _apply_own(self, G: ShardGroup) -> None:
        """Flat mode: apply this rank's updates to its own parameters (in the flat buffer)."""
        if not G.owned:
            return
        items = [(G.params[j], None, None, G.lr) for j in G.owned]
        self.engine.apply([(G.shape, G.lr, items)], [G.local_buf[:len(items)]], weight_decay=self.wd,
                          base_lr=self.lr)

    def _exchange(self, gi: int, G: ShardGroup) -> None:
        """Make this rank's updated shard of group gi visible in every rank's flat buffer."""
        if self.peer is not None:
            per = local_count(len(G.params), self.world)
            nbytes = per * G.params[0].numel() * 2
            self.peer.push(gi, self.rank * nbytes, nbytes, torch.cuda.current_stream())
        else:
            dist.all_gather_into_tensor(G.flat_buf, G.own_slice, group=self.pg)

    def _finish_exchange(self) -> None:
        if self.peer is not None:
            dist.all_reduce(self._bar, group=self.pg)  # barrier: every peer's stores into this rank are done

    def _step_flat(self) -> None:
        if self.comm_stream is None or not self.overlap:
            for gi in self.flat_order:
                G = self.groups[gi]
                self._orthogonalize(G)
                self._apply_own(G)
                self._exchange(gi, G)
            self._finish_exchange()
            return
        compute = torch.cuda.current_stream()
        comm = self.comm_stream
        # every group's memory-bound prologue (momentum, orientation, norm) first,
        # while no exchange competes for HBM and SMs
        phased = hasattr(self.engine, "orthogonalize_phase")
        if phased:
            for gi in self.flat_order:
                self._orthogonalize(self.groups[gi], phase=1)
        for gi in self.flat_order:
            G = self.groups[gi]
            self._orthogonalize(G, phase=2 if phased else 3)
            self._apply_own(G)
            ev = torch.cuda.Event()
            ev.record(compute)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                self._exchange(gi, G)
        with torch.cuda.stream(comm):
            self._finish_exchange()
        compute.wait_stream(comm)

    @torch.no_grad()
    def step(self) -> None:
        if self.flat:
            self._step_flat()
            return
        if self.world == 1:
            for G in self.groups:
                self._orthogonalize(G)
                self._apply(G)
            return
        if self.comm_stream is None or not self.overlap:
            for G in self.groups:
                self._orthogonalize(G)
                dist.all_gather_into_tensor(G.gather_buf, G.local_buf, group=self.pg)
                self._apply(G)
            return
        compute = torch.cuda.current_stream()
        comm = self.comm_stream
        for G in self.groups:
            self._orthogonalize(G)
            ev = torch.cuda.Event()
            ev.record(compute)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(G.gather_buf, G.local_buf, group=self.pg)
                self._apply(G)
        compute.wait_stream(comm)
