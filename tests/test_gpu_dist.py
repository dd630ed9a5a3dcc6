"""GPU (>= 2 devices): the sharded Muon step equals the single-GPU step.

Each rank orthogonalises its round-robin share of every shape group and the
results are exchanged (NCCL all-gather of the updates, NCCL all-gather of the
parameters, or the peer-memory push into every rank's replica); the
per-matrix arithmetic is unchanged, so the parameters after the step must be
bit-identical to the single-GPU lsr_muon_step_bf16 result on every rank.
Skipped when fewer than two GPUs are visible.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(256, 768), (256, 256), (256, 1024), (1024, 256)] * 2
# odd element counts and uneven group sizes: shard offsets that are not
# 16-byte aligned, and padding slots
RAGGED = [(5, 7)] * 3 + [(200, 300)] * 3 + [(72, 40)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(shapes):
    g = torch.Generator().manual_seed(21)
    P = [(torch.randn(*s, generator=g) * 0.02).bfloat16() for s in shapes]
    G = [(torch.randn(*s, generator=g) * 0.01).bfloat16() for s in shapes]
    return P, G


def _worker(rank, world, port, q, flat, exchange, shapes):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "cuda-lsr_b200"))
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from lsr.dist import ShardedMuon
        P, G = _data(shapes)
        params = [torch.nn.Parameter(p.cuda()) for p in P]
        opt = ShardedMuon(params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.01, flat_params=flat,
                          exchange=exchange)
        assert (opt.peer is not None) == (flat and exchange == "peer")
        for step in range(2):
            for p, g in zip(params, G):
                p.grad = g.cuda()
            opt.step()
        torch.cuda.synchronize()
        q.put((rank, [p.detach().float().cpu().numpy() for p in params]))
        opt.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("flat,exchange,shapes", [(False, "nccl", SHAPES), (True, "nccl", SHAPES),
                                                  (True, "peer", SHAPES), (True, "peer", RAGGED)])
def test_sharded_equals_single_gpu(flat, exchange, shapes):
    import lsr
    P, G = _data(shapes)
    params = [torch.nn.Parameter(p.cuda()) for p in P]
    opt = lsr.Muon(params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.01)
    for step in range(2):
        for p, g in zip(params, G):
            p.grad = g.cuda()
        opt.step()
    ref = [p.detach().float().cpu().numpy() for p in params]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, flat, exchange, shapes)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for pr in procs:
        pr.join(timeout=120)
    for r in range(2):
        assert not isinstance(results[r], str), results[r]
        for a, b in zip(results[r], ref):
            assert (a == b).all()
