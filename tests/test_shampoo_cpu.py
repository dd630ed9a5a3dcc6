"""CPU: host-side schedule and configuration of the DistributedShampoo drop-in (no GPU calls)."""
import torch

from lsr.shampoo import DDPDistributedConfig, DistributedShampoo


def _opt(freq, start):
    p = torch.nn.Parameter(torch.zeros(8, 8, dtype=torch.bfloat16))
    return DistributedShampoo([p], precondition_frequency=freq, start_preconditioning_step=start)


def test_refresh_schedule_is_the_reference_periodic_rule():
    """Roots / eigenbases are recomputed at 1-based steps t >= start with t % freq == 0 (every step
    when freq is 1): the steps shampoo_soap_lm_ddp_zero1.py:622-632 times as periodic. With a start
    that is not a multiple of the frequency the first refresh waits for the next multiple."""
    o = _opt(10, 5)
    assert [t for t in range(1, 41) if o.is_refresh_step(t)] == [10, 20, 30, 40]
    o = _opt(2, 3)
    assert [t for t in range(1, 11) if o.is_refresh_step(t)] == [4, 6, 8, 10]
    o = _opt(5, 5)  # the reference script's defaults
    assert [t for t in range(1, 21) if o.is_refresh_step(t)] == [5, 10, 15, 20]
    o = _opt(1, 3)
    assert [t for t in range(1, 6) if o.is_refresh_step(t)] == [3, 4, 5]


def test_communication_dtype_defaults_to_reference_float16():
    assert DDPDistributedConfig().communication_dtype == torch.float16
