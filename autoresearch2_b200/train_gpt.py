"""Data-parallel training run of the GPT harness (gpt.py) on synthetic tokens.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m autoresearch2_b200.train_gpt [--dense] [--check] [--batch 32] ...
"""
import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from . import bitsparse as bs
from .gpt import GPT, GPTConfig, TrainStep, flops_per_token, synthetic_batch


def main(argv=None):
    """Train the harness on synthetic tokens and print one JSON line.

    One process per GPU (torchrun; 127.0.0.1 rendezvous): each rank holds the
    whole model (same seed), trains on its own batch (seed + rank), and
    torch's DistributedDataParallel averages the gradients over NCCL.  Timed
    with CUDA events over --steps steps after --warmup, max over ranks;
    tokens/s is for the whole job.  --check: after the steps, every rank's
    parameters must be bit-identical (exit status 1 otherwise)."""
    ap = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=32, help="sequences per GPU")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--width", type=int, default=768)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--hidden", type=int, default=3072)
    ap.add_argument("--vocab", type=int, default=50304)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--dense", action="store_true", help="dense torch MLPs instead of the sparse FFN")
    ap.add_argument("--check", action="store_true")
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    cfg = GPTConfig(n_layer=args.layers, n_head=args.heads, n_embd=args.width, ffn_hidden=args.hidden,
                    vocab=args.vocab, seq_len=args.seq)
    model = GPT(cfg, sparse=not args.dense, device=device)
    net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local]) if world > 1 else model
    idx, tgt = synthetic_batch(cfg, args.batch, device, seed=rank)
    step = TrainStep(net, idx, tgt)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        loss = step()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / args.steps
    ok = True
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
        if args.check:
            flat = torch.cat([p.detach().reshape(-1).float() for p in model.parameters()])
            ref = flat.clone()
            dist.broadcast(ref, 0)
            same = torch.tensor([int(torch.equal(flat, ref))], device=device)
            dist.all_reduce(same, op=dist.ReduceOp.MIN)
            ok = bool(same.item())
    bs.check_status(device)
    tokens = world * args.batch * cfg.seq_len
    if rank == 0:
        print(json.dumps({"harness": "gpt", "mlp": "dense" if args.dense else "sparse_relu2", "n_gpus": world,
                          "tokens_per_s": round(tokens / (ms / 1e3), 1), "ms_per_step": round(ms, 3),
                          "tokens_per_step": tokens, "flops_per_token": flops_per_token(cfg),
                          "loss": round(float(loss), 4), "params_identical": ok if args.check else None}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
