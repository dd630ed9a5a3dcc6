"""CPU: the language-model driver's command line and optimizer structure against the reference.

The golden file holds the run-summary keys, parameter count and optimizer structure of the
reference's own recorded GPT-2-XL Muon run (gpt2xl_4gpu_batched.json; tests/golden/make_golden.py).
GPT-2-XL is built on the meta device (no memory, no weights) from the driver's built-in config.
"""
import json
from pathlib import Path

import torch

GOLD = json.loads((Path(__file__).parent / "golden" / "driver_golden.json").read_text())


def test_gpt2xl_optimizer_structure_matches_reference_run():
    import lsr
    from lsr.lm_driver import model_config
    from transformers import AutoModelForCausalLM
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(model_config("openai-community/gpt2-xl", ""))
    assert sum(p.numel() for p in model.parameters()) == GOLD["model_params"]
    opt = lsr.MuonAdamW(list(model.named_parameters()), "batched", 1e-3, 0.95, 0.01, True, 5, 1e-7, "original", 8,
                        1e-4, (0.9, 0.95), 0.01, 0)
    assert json.loads(json.dumps(opt.summary())) == GOLD["optimizer_structure"]


def test_cli_flags_and_defaults_follow_the_reference():
    """muon_lm_ddp.py:905-1103: same flags, same defaults (--muon-mode required)."""
    from lsr.lm_driver import build_parser
    a = build_parser().parse_args(["--muon-mode", "batched"])
    assert (a.model_id, a.init, a.muon_batch_matrices, a.muon_lr, a.muon_momentum, a.muon_weight_decay,
            a.muon_ns_steps, a.muon_eps, a.muon_lr_adjust) == \
        ("openai-community/gpt2-xl", "pretrained", 8, 1e-3, 0.95, 0.01, 5, 1e-7, "original")
    assert (a.adam_lr, a.adam_weight_decay, a.adam_beta1, a.adam_beta2) == (1e-4, 0.01, 0.9, 0.95)
    assert (a.steps, a.warmup_steps, a.seq_len, a.micro_batch, a.grad_accum, a.seed) == (40, 10, 512, 1, 1, 17)
    assert a.gradient_checkpointing and a.output == "muon_run.json" and a.ddp_bucket_cap_mb == 100
    assert a.train_token_cache == "./cache/wikitext103_train_5m.pt" and a.train_cache_tokens == 5_000_000


def test_deterministic_batch_order():
    """Blocks taken in the reference's order (muon_lm_ddp.py:245-289)."""
    from lsr.lm_driver import deterministic_batch
    tok = torch.arange(1000, dtype=torch.int32)
    x = deterministic_batch(tok, optimizer_step=3, micro_step=1, rank=1, world_size=2, micro_batch=2, seq_len=10,
                            grad_accum=2, device="cpu")
    first = (3 * 2 + 1) * 2 * 2 + 1 * 2
    assert x.tolist() == [list(range(10 * first, 10 * first + 10)), list(range(10 * first + 10, 10 * first + 20))]
