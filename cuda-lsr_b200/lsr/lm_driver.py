"""Language-model benchmark driver with liblsr's Muon: the command line and the run summary of
muon_lm_ddp.py (its ``main``, muon_lm_ddp.py:902-1688), so a run here and a run of the reference
are compared key for key (``median_muon_ms`` against gpt2xl_4gpu_*.json).

    python -m lsr.lm_driver --muon-mode batched --init random --steps 40 --warmup-steps 10 \\
        --seq-len 512 --micro-batch 1 --grad-accum 2 --output gpt2xl_1gpu_batched.json
    torchrun --nproc-per-node N -m lsr.lm_driver ...          (DDP, one process per GPU)

Same flags and defaults as the reference, same per-step CUDA-event timing (step, optimizer,
Muon and AdamW intervals, max over ranks), same summary keys in the same order. What differs, and
is recorded in the summary's extra ``"lsr"`` entry:

* the optimizer is ``lsr.MuonAdamW`` (the whole Muon step in liblsr's kernels); with
  ``--muon-sharded`` and more than one rank the Muon matrices are sharded ZeRO-1 style
  (``lsr.dist.ShardedMuon``, flat parameters) instead of replicated on every rank;
* the model is built from its configuration (transformers GPT-2 classes; the GPT-2 family's
  configurations are built in, so no download is needed) — ``--init random`` as the
  reference's ``--init random`` (muon_lm_ddp.py:791-802); ``--init pretrained`` loads weights
  from a local ``--model-id`` directory only;
* the token stream comes from ``--train-token-cache`` when that file exists (the reference's
  cache format, a 1-D token tensor); otherwise it is seeded synthetic tokens, uniform over the
  vocabulary, with the cache's length, and the summary says so.
* ``--config-overrides key=value,...`` changes fields of the model configuration (small
  models for tests).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

# GPT-2 family configurations (n_embd, n_layer, n_head), vocabulary 50257, 1024 positions.
GPT2_FAMILY = {
    "gpt2": (768, 12, 12),
    "gpt2-medium": (1024, 24, 16),
    "gpt2-large": (1280, 36, 20),
    "gpt2-xl": (1600, 48, 25),
}


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model-id", type=str, default="openai-community/gpt2-xl")
    p.add_argument("--init", choices=["pretrained", "random"], default="pretrained")
    p.add_argument("--muon-mode", choices=["serial", "batched"], required=True)
    p.add_argument("--muon-batch-matrices", type=int, default=8)
    p.add_argument("--muon-lr", type=float, default=1e-3)
    p.add_argument("--muon-momentum", type=float, default=0.95)
    p.add_argument("--muon-weight-decay", type=float, default=0.01)
    p.add_argument("--muon-ns-steps", type=int, default=5)
    p.add_argument("--muon-eps", type=float, default=1e-7)
    p.add_argument("--muon-lr-adjust", choices=["original", "match_rms_adamw", "none"], default="original")
    p.add_argument("--adam-lr", type=float, default=1e-4)
    p.add_argument("--adam-weight-decay", type=float, default=0.01)
    p.add_argument("--adam-beta1", type=float, default=0.9)
    p.add_argument("--adam-beta2", type=float, default=0.95)
    p.add_argument("--steps", type=int, default=40)
    p.add_argument("--warmup-steps", type=int, default=10)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--micro-batch", type=int, default=1)
    p.add_argument("--grad-accum", type=int, default=1)
    p.add_argument("--seed", type=int, default=17)
    p.add_argument("--gradient-checkpointing", action=argparse.BooleanOptionalAction, default=True)
    p.add_argument("--train-token-cache", type=str, default="./cache/wikitext103_train_5m.pt")
    p.add_argument("--val-token-cache", type=str, default="./cache/wikitext103_val_1m.pt")
    p.add_argument("--train-cache-tokens", type=int, default=5_000_000)
    p.add_argument("--val-cache-tokens", type=int, default=1_000_000)
    p.add_argument("--eval-every", type=int, default=0, help="0 disables periodic validation")
    p.add_argument("--eval-batches", type=int, default=8)
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--ddp-bucket-cap-mb", type=int, default=100)
    p.add_argument("--output", type=str, default="muon_run.json")
    # additions (not in the reference)
    p.add_argument("--muon-sharded", action="store_true",
                   help="shard the Muon matrices over the ranks (ZeRO-1) instead of replicating the step")
    p.add_argument("--config-overrides", type=str, default="",
                   help="comma-separated key=value changes to the model configuration")
    return p


def model_config(model_id: str, overrides: str):
    from transformers import AutoConfig, GPT2Config
    key = model_id.split("/")[-1]
    if key in GPT2_FAMILY:
        e, l, h = GPT2_FAMILY[key]
        cfg = GPT2Config(n_embd=e, n_layer=l, n_head=h, n_positions=1024, vocab_size=50257)
    elif Path(model_id).is_dir():
        cfg = AutoConfig.from_pretrained(model_id)
    else:
        raise ValueError(f"unknown model {model_id!r}: use a GPT-2 family id or a local configuration directory")
    for kv in filter(None, overrides.split(",")):
        k, v = kv.split("=", 1)
        old = getattr(cfg, k)
        setattr(cfg, k, type(old)(v) if old is not None else int(v))
    return cfg


def load_model(args, device):
    """The model as muon_lm_ddp.load_model_and_tokenizer builds it (:755-826): bf16, use_cache off,
    optional gradient checkpointing, train mode."""
    from transformers import AutoModelForCausalLM
    if args.init == "pretrained":
        if not Path(args.model_id).is_dir():
            raise RuntimeError("--init pretrained needs a local model directory as --model-id "
                               "(no download here); use --init random for the random-init benchmark")
        model = AutoModelForCausalLM.from_pretrained(args.model_id, dtype=torch.bfloat16)
    else:
        model = AutoModelForCausalLM.from_config(model_config(args.model_id, args.config_overrides))
        model = model.to(dtype=torch.bfloat16)
    model.config.use_cache = False
    if args.gradient_checkpointing:
        try:
            model.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})
        except TypeError:
            model.gradient_checkpointing_enable()
    model.to(device)
    model.train()
    return model


def token_stream(path: str, max_tokens: int, vocab: int, seed: int):
    """(tokens, source): the reference's token cache when present, else seeded synthetic tokens."""
    if Path(path).is_file():
        t = torch.load(path, map_location="cpu")
        return t[:max_tokens].to(torch.int32), f"token cache {path}"
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (max_tokens,), generator=g, dtype=torch.int32), \
        f"synthetic: {max_tokens} tokens uniform over the {vocab}-token vocabulary, seed {seed}"


def deterministic_batch(tokens, optimizer_step, micro_step, rank, world_size, micro_batch, seq_len, grad_accum,
                        device):
    """Sequential seq_len blocks, the order muon_lm_ddp.deterministic_batch (:245-289) takes them."""
    nblocks = tokens.numel() // seq_len
    first = (optimizer_step * grad_accum + micro_step) * world_size * micro_batch + rank * micro_batch
    rows = [tokens[((first + b) % nblocks) * seq_len:((first + b) % nblocks + 1) * seq_len].to(torch.long)
            for b in range(micro_batch)]
    return torch.stack(rows, 0).to(device, non_blocking=True)


def _max(x: float, device, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _mean(x: float, device, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item()) / world


class _ShardedMuonAdamW:
    """--muon-sharded: lsr.dist.ShardedMuon for the Muon matrices, fused AdamW for the rest; the
    split, lr adjustment and summary of lsr.MuonAdamW."""

    def __init__(self, base, world):
        from .dist import ShardedMuon
        self.base = base
        self.muon = ShardedMuon([p for _, p in base.muon_named], lr=base.muon_lr, momentum=base.muon_momentum,
                                nesterov=base.muon_nesterov, weight_decay=base.muon_weight_decay,
                                ns_steps=base.muon_ns_steps, eps=base.muon_eps, lr_adjust=base.muon_lr_adjust,
                                flat_params=True)
        base.momentum.clear()  # the shards own the momentum now

    def summary(self):
        return self.base.summary()

    def muon_step(self):
        self.muon.step()

    def adam_step(self):
        self.base.adam_step()

    def zero_grad(self):
        self.base.zero_grad()

    def close(self):
        self.muon.close()


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if args.muon_batch_matrices < 1:
        raise ValueError("--muon-batch-matrices must be >= 1")
    from . import MuonAdamW

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", device_id=device)
    torch.manual_seed(args.seed)
    torch.cuda.manual_seed_all(args.seed)
    torch.set_float32_matmul_precision("highest")
    torch.backends.cuda.matmul.allow_tf32 = False

    model = load_model(args, device)
    total_params = sum(p.numel() for p in model.parameters())
    vocab = model.config.vocab_size
    train_tokens, data_source = token_stream(args.train_token_cache, args.train_cache_tokens, vocab, args.seed)
    if rank == 0:
        print(f"model {args.model_id} ({args.init}), {total_params / 1e9:.3f} B params, world {world}; data: "
              f"{data_source}", flush=True)

    optimizer = MuonAdamW(
        named_parameters=list(model.named_parameters()), muon_mode=args.muon_mode, muon_lr=args.muon_lr,
        muon_momentum=args.muon_momentum, muon_weight_decay=args.muon_weight_decay, muon_nesterov=True,
        muon_ns_steps=args.muon_ns_steps, muon_eps=args.muon_eps, muon_lr_adjust=args.muon_lr_adjust,
        muon_batch_matrices=args.muon_batch_matrices, adam_lr=args.adam_lr,
        adam_betas=(args.adam_beta1, args.adam_beta2), adam_weight_decay=args.adam_weight_decay, rank=rank)
    if args.muon_sharded and world > 1:
        optimizer = _ShardedMuonAdamW(optimizer, world)
    opt_summary = optimizer.summary()

    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP
        ddp_model = DDP(model, device_ids=[local_rank], output_device=local_rank, broadcast_buffers=False,
                        gradient_as_bucket_view=True, bucket_cap_mb=args.ddp_bucket_cap_mb,
                        find_unused_parameters=False)
    else:
        ddp_model = model
    global_tokens_per_step = world * args.micro_batch * args.seq_len * args.grad_accum

    step_ms_values, muon_ms_values, adam_ms_values, optimizer_ms_values, losses = [], [], [], [], []
    optimizer.zero_grad()
    for step in range(args.steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        total_loss = 0.0
        for micro in range(args.grad_accum):
            x = deterministic_batch(train_tokens, step, micro, rank, world, args.micro_batch, args.seq_len,
                                    args.grad_accum, device)
            sync_ctx = (contextlib.nullcontext() if world == 1 or micro == args.grad_accum - 1
                        else ddp_model.no_sync())
            with sync_ctx:
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    loss = ddp_model(input_ids=x, labels=x, use_cache=False).loss / args.grad_accum
                loss.backward()
            total_loss += float(loss.detach())
        ev[1].record()
        optimizer.muon_step()
        ev[2].record()
        optimizer.adam_step()
        ev[3].record()
        optimizer.zero_grad()
        ev[3].synchronize()
        step_ms = _max(ev[0].elapsed_time(ev[3]), device, world)
        muon_ms = _max(ev[1].elapsed_time(ev[2]), device, world)
        adam_ms = _max(ev[2].elapsed_time(ev[3]), device, world)
        opt_ms = _max(ev[1].elapsed_time(ev[3]), device, world)
        loss_mean = _mean(total_loss, device, world)
        measured = step >= args.warmup_steps
        if measured:
            step_ms_values.append(step_ms)
            muon_ms_values.append(muon_ms)
            adam_ms_values.append(adam_ms)
            optimizer_ms_values.append(opt_ms)
            losses.append(loss_mean)
        if rank == 0 and (step % args.log_every == 0 or step == args.steps - 1):
            print(f"[{'MEASURE' if measured else 'WARMUP'}] step={step:03d} loss={loss_mean:.5f} "
                  f"step={step_ms:.1f}ms opt={opt_ms:.1f}ms muon={muon_ms:.1f}ms adam={adam_ms:.1f}ms "
                  f"tok/s={global_tokens_per_step / (step_ms / 1000.0):,.0f}", flush=True)
    if not step_ms_values:
        raise RuntimeError("No measured steps. Set --steps > --warmup-steps.")
    peak_gb = _max(torch.cuda.max_memory_allocated(device) / 1024 ** 3, device, world)
    summary = {
        "model_id": args.model_id,
        "init": args.init,
        "world_size": world,
        "gpu": torch.cuda.get_device_name(local_rank),
        "model_params": total_params,
        "muon_mode": args.muon_mode,
        "muon_batch_matrices": args.muon_batch_matrices,
        "muon_lr": args.muon_lr,
        "muon_lr_adjust": args.muon_lr_adjust,
        "muon_ns_steps": args.muon_ns_steps,
        "adam_lr": args.adam_lr,
        "seq_len": args.seq_len,
        "micro_batch": args.micro_batch,
        "grad_accum": args.grad_accum,
        "global_tokens_per_step": global_tokens_per_step,
        "steps": args.steps,
        "warmup_steps": args.warmup_steps,
        "median_step_ms": statistics.median(step_ms_values),
        "median_optimizer_ms": statistics.median(optimizer_ms_values),
        "median_muon_ms": statistics.median(muon_ms_values),
        "median_adam_ms": statistics.median(adam_ms_values),
        "median_tokens_per_second": global_tokens_per_step / (statistics.median(step_ms_values) / 1000.0),
        "mean_measured_loss": sum(losses) / len(losses),
        "final_measured_loss": losses[-1],
        "peak_allocated_gb": peak_gb,
        "optimizer_structure": opt_summary,
        "lsr": {"optimizer": "lsr.MuonAdamW" + (" + lsr.dist.ShardedMuon" if args.muon_sharded and world > 1
                                                 else ""),
                "data": data_source, "config_overrides": args.config_overrides},
    }
    if rank == 0:
        for key in ("median_step_ms", "median_optimizer_ms", "median_muon_ms", "median_adam_ms",
                    "median_tokens_per_second", "mean_measured_loss", "final_measured_loss", "peak_allocated_gb"):
            print(f"{key:28s}: {summary[key]}")
        out = Path(args.output)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps(summary, indent=2))
        print(f"wrote: {out}", flush=True)
    if hasattr(optimizer, "close"):
        optimizer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
