"""Headline benchmark: 29B MMDiT 720p training throughput in latent tokens/s (pretraining, FSDP, no CP).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

One rank per GPU.  Every rank trains the 29B architecture of config/pretrain_29B_720p.yaml (random
init, bf16 compute, exact fp32 masters, Muon + AdamW, global-norm clipping at 1.0, full activation
checkpointing) on its own synthetic packed batch: 5 clips x (21 x 44 x 80 Wan-2.2 latents -> 18,480
patch tokens + 512 text tokens of dim 4096) = 94,960 joint tokens within the 110,576 budget.
Weights are sharded over the N ranks (FSDP-style); when one replica's optimizer state does not fit
the GPUs, master low halves and optimizer state are streamed from pinned host memory.

Timing: W untimed steps, then K steps between barrier + synchronize; CUDA events on the launching
stream; the max over ranks.  ``value`` is the device time of forward+backward+optimizer per step;
``e2e`` is the same K steps measured around the public ``StepRunner`` call including the host->device
copy of the step's inputs from pinned memory and the device->host read of loss and grad norm.
Per-step activations (several GB) exceed the 126 MB L2, so no extra flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "29B MMDiT 720p train latent tokens/s (1/2/4/8 B200, max over ranks); s/video @50 steps"
WORKLOAD_METRICS = {
    "longctx": "29B MMDiT long-context (one 121-frame 720p clip, Ulysses CP) train latent tokens/s",
    "sft": "29B MMDiT SFT mixed image+video packing (CP=2) train latent tokens/s",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--config", default=os.path.join(ROOT, "config", "pretrain_29B_720p.yaml"))
    ap.add_argument("--layers", type=int, default=None, help="development only: fewer joint blocks (invalid result)")
    ap.add_argument("--clips", type=int, default=5)
    ap.add_argument("--frames", type=int, default=21)
    ap.add_argument("--offload", default="auto")
    ap.add_argument("--workload", default="pretrain", choices=("pretrain", "longctx", "sft"),
                    help="pretrain: the headline (5 x 5 s clips per GPU, FSDP); longctx: one 121-frame 720p "
                         "clip (~107k tokens) with Ulysses CP over all ranks; sft: mixed images + videos of "
                         "random lengths filling the SFT budget, CP=2")
    ap.add_argument("--cp", type=int, default=None, help="context-parallel size (longctx: all ranks, sft: 2)")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the small-model check of the fused peer-memory paths against NCCL (N > 1)")
    return ap.parse_args()


REF_DIR = os.path.join(ROOT, "baseline", "_ref")
# The reference's own entry modules on the training path (train.py builds the transformer, FA4
# attention, quack GEMMs and the patched Muon from these), imported in this order.
REF_MODULES = ("pan.models.transformers.pan_transformer", "pan.utils.flash_attention",
               "pan.models.transformers.modules.mlp_ops", "pan.optim.patch_muon")


def reference_arm(args):
    """Runs the unmodified reference from baseline/_ref through its own modules when they import;
    otherwise prints why not (the import error itself), as one JSON line."""
    line = {"impl": "reference", "metric": METRIC}
    if not os.path.isdir(os.path.join(REF_DIR, "pan")):
        line["unavailable"] = ("baseline/_ref holds no reference source: pip refuses to install it (the project has "
                               "no setup.py or pyproject.toml)")
        print(json.dumps(line), flush=True)
        return
    import importlib
    import sys
    sys.path.insert(0, REF_DIR)
    for mod in REF_MODULES:
        try:
            importlib.import_module(mod)
        except Exception as err:  # the reference's hard dependencies are absent from this image
            line["unavailable"] = f"importing the reference's {mod} fails: {type(err).__name__}: {err}"[:400]
            print(json.dumps(line), flush=True)
            return
    line["unavailable"] = ("the reference's modules import, but its trainer needs its pinned stack (torch 2.12, "
                           "flash-attn 4, quack >= 0.6.3) to run the 29B step")
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist
    import yaml
    from pan2_b200.data.synthetic import (batch_bytes, batch_to_device, pin_batch, sft_mix_items,
                                          synthetic_items_batch, synthetic_packed_batch)
    from pan2_b200.models.transformer import translate_architecture_config
    from pan2_b200.ops._ext import start_launch_count, stop_launch_count, ext
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.training.step import StepRunner
    from pan2_b200.optim.lr import lr_lambda_from_config
    from pan2_b200.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if args.workload == "longctx":
        cp = args.cp or world
    elif args.workload == "sft":
        cp = args.cp or (2 if world % 2 == 0 else 1)
    else:
        cp = 1
    if world % cp:
        raise SystemExit(f"--cp {cp} does not divide {world} ranks")
    layout = None
    if world > 1 and cp > 1:
        from pan2_b200.parallel.layout import init_parallel_layout
        layout = init_parallel_layout(cp=cp, backend="cpu:gloo,cuda:nccl", timeout_s=900)
        group = layout.shard_group
    elif world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=device)
        group = dist.group.WORLD

    parity = None
    if world > 1 and not args.no_parity:
        # every fused collective path against its NCCL baseline on a small model, before the timed job
        from pan2_b200.utils.parity import fused_path_parity
        parity = fused_path_parity(device, group, rank, layout, cp)

    with open(args.config) as f:
        cfg = yaml.safe_load(f)
    arch = translate_architecture_config(cfg["model"]["transformer_config_overrides"])
    arch["zero_init_modulation"] = bool(cfg["model"].get("zero_init_modulation", True))
    valid = True
    if args.layers is not None:
        arch["num_layers"] = args.layers
        valid = args.layers == 44
    tr = cfg["training"]
    optim = OptimConfig(lr=float(tr["learning_rate"]), weight_decay=float(tr.get("weight_decay", 0.05)),
                        use_muon=bool(tr.get("use_muon", True)), max_grad_norm=float(tr["max_grad_norm"]))

    # 704x1280 frames -> 44x80 latents; 21 latent frames per 5 s clip; 512 text tokens per clip
    rope = dict(rope_axes=tuple(arch["rope_axes_dim"]), rope_theta=float(arch["rope_theta"]),
                rope_scale=(float(arch["rope_temporal_scale"]), 1.0, 1.0))
    dp_rank = rank // cp
    data = cfg["data"]
    if args.workload == "pretrain":
        batch = synthetic_packed_batch(args.clips, (args.frames, 44, 80), 512, seed=1234 + rank, pin=True, **rope)
    else:
        if args.workload == "longctx":  # 121 latent frames (~20 s) of 704x1280 in one sequence
            items = [((121, 44, 80), True)]
        else:
            items = sft_mix_items(int(data["packed_video_token_budget"]), int(data["packed_joint_token_budget"]),
                                  int(data["packed_dataloader_max_num_seq"]), 512, seed=1234 + dp_rank)
        batch = synthetic_items_batch(items, [512] * len(items), seed=1234 + dp_rank, **rope)
    meta = batch["packed_seq_params"]
    assert meta.n_active <= int(data["packed_joint_token_budget"])
    latent_tokens = meta.n_video  # per cp group

    t0 = time.time()
    # activation reserve: with one rank the block checkpoints live in idle gradient buffers
    reserve_gb = float(os.environ.get("PAN_ACT_RESERVE_GB", "40" if world == 1 else "72"))
    engine = TrainEngine(arch, device, group=group, seed=42, optim=optim, offload=args.offload,
                         activation_bytes_estimate=int(reserve_gb * 1e9))
    if cp > 1:
        # every cp rank trains its strided shard of the cp group's sequence
        from pan2_b200.data.cp_batch import broadcast_and_split
        engine.set_context_parallel(layout.cp_group, cp, layout.cp_rank)
        src = batch_to_device(batch, device) if layout.cp_rank == 0 else None
        shard, _ = broadcast_and_split(src, None, layout, device)
        torch.cuda.synchronize()
        batch = pin_batch({k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in shard.items()})
    elif args.workload != "pretrain":
        batch = pin_batch(batch)
    init_s = time.time() - t0
    runner = StepRunner(engine, lr_lambda=lr_lambda_from_config(tr))

    for _ in range(args.warmup):
        runner.train_step(batch)
    engine.flush_updates()  # the timed region holds exactly K optimizer updates
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    sampler = ClockSampler()  # sampled by the rank that prints (every GPU of this node is queried)
    if rank == 0:
        sampler.start()
    start_launch_count()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for k in range(args.steps):
        ev[k][0].record()
        dev_batch = batch_to_device(batch, device, non_blocking=True)
        ev[k][1].record()
        metrics = runner.device_step(dev_batch)
        if k == args.steps - 1:
            # deferred optimizer updates (one rank) finish inside the timed region: the last step's
            # update is waited for here, the earlier ones by the next step's forward
            engine.flush_updates()
        ev[k][2].record()
    torch.cuda.synchronize()
    launches = stop_launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop(gpus=list(range(world))) if rank == 0 else None

    total_ms = ev[0][0].elapsed_time(ev[-1][2])
    compute_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    t = torch.tensor([total_ms, compute_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, compute_ms = t.tolist()
    ms_step = compute_ms / args.steps
    e2e_ms = total_ms / args.steps
    tokens_global = latent_tokens * (world // cp)
    err = ext().error_flag(True)
    if rank == 0:
        h2d = batch_bytes(batch)
        out = {
            "metric": WORKLOAD_METRICS.get(args.workload, METRIC),
            "value": tokens_global / (ms_step / 1e3),
            "unit": "latent tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong" if args.workload == "longctx" else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random Wan-2.2-shaped latents, random 4096-d text embeddings, random-init 29B weights)",
            "config": {
                "model": f"PAN2 MMDiT {engine.total_params / 1e9:.2f}B ({arch['num_layers']} layers)",
                "global_batch": (args.clips if args.workload == "pretrain" else meta.num_samples) * (world // cp),
                "seq_len": meta.joint_packed_length,
                "latent_tokens_per_gpu": latent_tokens * (world // cp) // world,
                "joint_tokens_per_gpu": meta.n_active * (world // cp) // world,
                "parallelism": f"fsdp{world}" + (f"+cp{cp}" if cp > 1 else "") + ("+host-offload" if engine.offload else ""),
                "workload": args.workload,
                "optimizer": "Muon+AdamW, clip 1.0",
                "activation_checkpointing": "every block",
                "l2": "per-step working set (GBs) larger than L2; no extra flush",
                "valid_full_config": valid,
            },
            "e2e": {"value": tokens_global / (e2e_ms / 1e3), "unit": "latent tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8,
                    "api": "pan2_b200.training.step.StepRunner (inputs copied from pinned host memory)"},
            "gpu_launches": launches["total"],
            "parity_fused_vs_nccl": parity,
            "clocks": clocks,
            "loss": metrics["loss"],
            "grad_norm": metrics["grad_norm"],
            "init_s": init_s,
            "device_error_flag": err,
            "peak_mem_gb": torch.cuda.max_memory_allocated(device) / 1e9,
            "allocator": {k: torch.cuda.memory_stats(device).get(k) for k in
                          ("num_alloc_retries", "num_device_alloc", "num_device_free")},
            "act_reserve_gb": reserve_gb,
            "last_step_phases_ms": runner.phase_times(),
            "host_pinned_gb": engine.host_bytes_planned / 1e9,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
