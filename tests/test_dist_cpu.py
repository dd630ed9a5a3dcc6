"""CPU (gloo) tests of the sharded Muon host logic and of failure handling.

The CUDA engine is replaced by a fake with the same interface that performs
the momentum update and a deterministic per-matrix transform in torch, so the
ownership, gather order, padding and apply order of lsr.dist.ShardedMuon are
checked without a GPU. A failing rank must surface as an error on the other
ranks (short process-group timeout), not as a hang.
"""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class FakeEngine:
    """Muon without Newton–Schulz: u = g + mu*buf, update = 2*u (oriented)."""

    def orthogonalize(self, grouped, *, momentum, nesterov, ns_steps, eps, coef, out):
        for (shape, _, items), o in zip(grouped, out):
            for k, (p, g, m, _) in enumerate(items):
                m.mul_(momentum).add_(g)
                u = g + momentum * m if nesterov else m
                u = u.T if shape[0] > shape[1] else u
                o[k].copy_(2.0 * u)
        return out

    def apply(self, grouped, updates, *, weight_decay, base_lr):
        for (shape, lr, items), upd in zip(grouped, updates):
            for k, (p, _, _, _) in enumerate(items):
                u = upd[k].T if shape[0] > shape[1] else upd[k]
                p.mul_(1 - base_lr * weight_decay).add_(u.to(p.dtype), alpha=-lr)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _make(seed=0):
    g = torch.Generator().manual_seed(seed)
    shapes = [(16, 48)] * 5 + [(64, 16)] * 3 + [(32, 32)] * 4
    P = [torch.randn(*s, generator=g) for s in shapes]
    G = [torch.randn(*s, generator=g) for s in shapes]
    return P, G


def _reference():
    """Single process: every matrix on one rank."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "cuda-lsr_b200"))
    from lsr.dist import ShardedMuon
    P, G = _make()
    params = [torch.nn.Parameter(p.clone()) for p in P]
    opt = ShardedMuon(params, lr=0.1, momentum=0.9, weight_decay=0.01, engine=FakeEngine())
    for _ in range(2):
        for p, g in zip(params, G):
            p.grad = g.clone()
        opt.step()
    return [p.detach().clone() for p in params]


def _worker(rank, world, port, mode, q, flat=False):
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "cuda-lsr_b200"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        from lsr.dist import ShardedMuon
        P, G = _make()
        params = [torch.nn.Parameter(p.clone()) for p in P]
        opt = ShardedMuon(params, lr=0.1, momentum=0.9, weight_decay=0.01, engine=FakeEngine(), flat_params=flat)
        for step in range(2):
            for p, g in zip(params, G):
                p.grad = g.clone()
            if mode == "fail" and rank == 1 and step == 1:
                raise RuntimeError("injected failure on rank 1")
            opt.step()
        # numpy copies: tensors in a queue are shared by file descriptor and vanish with this process
        q.put((rank, "ok", [p.detach().numpy().copy() for p in params],
               [len(Gp.owned) for Gp in opt.groups]))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)[:200], traceback.format_exc()[-300:]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, mode, flat=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q, flat)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, *rest = q.get(timeout=120)
        out[r] = (status, rest)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,flat", [(2, False), (3, False), (2, True), (3, True)])
def test_sharded_matches_single_process(world, flat):
    ref = _reference()
    out = _run(world, "ok", flat)
    for r in range(world):
        status, rest = out[r]
        assert status == "ok", rest
        params, owned = rest
        for a, b in zip(params, ref):
            assert torch.allclose(torch.from_numpy(a), b, atol=1e-6), r
    # every matrix owned exactly once (5, 3, 4 matrices per shape group)
    totals = [sum(out[r][1][1][gi] for r in range(world)) for gi in range(3)]
    assert totals == [5, 3, 4]


def test_rank_failure_surfaces_as_error():
    out = _run(2, "fail")
    assert out[1][0] == "error" and "injected" in out[1][1][0]
    assert out[0][0] == "error"  # the surviving rank's collective fails instead of hanging


def test_gathered_order_and_padding():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "cuda-lsr_b200"))
    from lsr.dist import gathered_order, local_count, owner_of
    assert gathered_order(5, 2) == [0, 2, 4, 1, 3, None]
    assert local_count(48, 8) == 6 and local_count(5, 2) == 3
    assert [owner_of(j, 4) for j in range(6)] == [0, 1, 2, 3, 0, 1]
