"""GPU (>= 2 devices): DistributedShampoo with DDPDistributedConfig (ZeRO-1).

Blocks are owned by ranks (greedy by flops); each rank computes the
statistics and directions of its own blocks only, the directions are
all-gathered in fp32 and every rank applies all of them. A block's arithmetic
does not depend on which blocks share its stack, so after the steps every
rank's parameters must equal the single-GPU optimizer's bit for bit for
SOAP. Shampoo's Adam grafting rescales each block by a ratio of Frobenius
norms computed with torch reductions, whose summation order follows the
stack's shape: there the parameters may differ by rounding flips, at most
2 bf16 ulps. Skipped with fewer than two GPUs.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(256, 768), (768, 256), (256, 256), (384, 512)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    g = torch.Generator().manual_seed(31)
    P = [(torch.randn(*s, generator=g) * 0.02).bfloat16() for s in SHAPES]
    G = [[(torch.randn(*s, generator=g) * 0.01).bfloat16() for s in SHAPES] for _ in range(3)]
    return P, G


def _run(params, grads, soap, distributed):
    from lsr.shampoo import DDPDistributedConfig, DefaultSOAPConfig, DistributedShampoo
    kw = dict(lr=0.01, betas=(0.9, 0.95), epsilon=1e-6, weight_decay=0.01, max_preconditioner_dim=256,
              precondition_frequency=2, start_preconditioning_step=2)
    if soap:
        kw["preconditioner_config"] = DefaultSOAPConfig
    if distributed:
        kw["distributed_config"] = DDPDistributedConfig(communication_dtype=torch.float32)
    opt = DistributedShampoo(params, **kw)
    for step_grads in grads:
        for p, gr in zip(params, step_grads):
            p.grad = gr.cuda()
        opt.step()
    torch.cuda.synchronize()
    return opt


def _worker(rank, world, port, q, soap):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "cuda-lsr_b200"))
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        P, G = _data()
        params = [torch.nn.Parameter(p.cuda()) for p in P]
        opt = _run(params, G, soap, True)
        owned = sum(len(grp.refs) for _, grp, _ in opt._groups if grp is not None)
        q.put((rank, [p.detach().float().cpu().numpy() for p in params], owned))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), 0))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("soap", [True, False])
def test_zero1_equals_single_gpu(soap):
    P, G = _data()
    params = [torch.nn.Parameter(p.cuda()) for p in P]
    opt = _run(params, G, soap, False)
    total = sum(len(grp.refs) for _, grp, _ in opt._groups if grp is not None)
    ref = [p.detach().float().cpu().numpy() for p in params]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, soap)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = {}
    for _ in range(2):
        r, out, owned = q.get(timeout=300)
        results[r] = (out, owned)
    for pr in procs:
        pr.join(timeout=120)
    for r in range(2):
        out, _ = results[r]
        assert not isinstance(out, str), out
        for a, b in zip(out, ref):
            if soap:
                assert (a == b).all()
            else:
                ulp = abs(b) * 2.0 ** -7 + 1e-30
                assert bool(((abs(a - b)) <= 2 * ulp).all())
    # every block owned by exactly one rank
    assert results[0][1] + results[1][1] == total and min(results[0][1], results[1][1]) > 0
