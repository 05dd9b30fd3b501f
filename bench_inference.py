"""Inference benchmark: seconds per video for 50-step sampling of the 29B MMDiT (720p i2v, CFG, SP).

    python bench_inference.py [--gpus N] [--steps 50] [--warmup 3]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench_inference.py --gpus N

One 720p clip: 81 frames at 704x1280 -> a 21x44x80 Wan-2.2 latent -> 18,480 patch tokens; image-to-video
(first latent frame from a random "reference" latent), classifier-free guidance (negative + positive
prompt, 512 random 4096-d caption embeddings each), random-init 29B weights in bf16, Ulysses sequence
parallel over the N GPUs.  W untimed sampler steps warm up; then one full video of K steps is timed
with CUDA events on the launching stream (max over ranks), through the public
``PanVideoPipeline.__call__``, including the host->device copy of the noise and embeddings and the
device->host read of the final latent.  The 58 GB of weights read every step dwarf the 126 MB L2.
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

METRIC = "29B 720p 50-step sampling s/video (CFG, i2v, sequence parallel)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--config", default=os.path.join(ROOT, "config", "pretrain_29B_720p.yaml"))
    ap.add_argument("--frames", type=int, default=81)
    ap.add_argument("--height", type=int, default=704)
    ap.add_argument("--width", type=int, default=1280)
    ap.add_argument("--text_len", type=int, default=512)
    ap.add_argument("--layers", type=int, default=None, help="development only: fewer joint blocks (invalid result)")
    return ap.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        from bench import reference_arm  # the same import attempt of the unmodified reference
        import bench
        bench.METRIC = METRIC
        bench.REF_MODULES = ("pan.pipelines.pan_video_pipeline",) + bench.REF_MODULES
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist
    import yaml
    from pan2_b200.models.transformer import ARCH_DEFAULTS, translate_architecture_config
    from pan2_b200.ops._ext import ext, start_launch_count, stop_launch_count
    from pan2_b200.parallel.layout import init_parallel_layout
    from pan2_b200.pipelines.video import PanVideoPipeline, build_inference_model
    from pan2_b200.utils.clocks import ClockSampler

    L = init_parallel_layout(cp=args.gpus, timeout_s=900)
    world, rank = L.world_size, L.rank
    local = int(os.environ.get("LOCAL_RANK", 0))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    with open(args.config) as f:
        cfg = yaml.safe_load(f)
    arch = dict(ARCH_DEFAULTS)
    arch.update(translate_architecture_config(cfg["model"]["transformer_config_overrides"]))
    valid = args.layers is None
    if args.layers is not None:
        arch["num_layers"] = args.layers
    t0 = time.time()
    model = build_inference_model(arch, device, dtype=torch.bfloat16, seed=0)
    n_params = sum(p.numel() for p in model.parameters())
    pipe = PanVideoPipeline(model, device=device, sp_group=L.cp_group if world > 1 else None)
    init_s = time.time() - t0
    g = torch.Generator().manual_seed(1)
    pos = [torch.randn(args.text_len, 4096, generator=g).to(torch.bfloat16).pin_memory()]
    neg = [torch.randn(args.text_len, 4096, generator=g).to(torch.bfloat16).pin_memory()]
    ref = torch.randn(48, 1, args.height // 16, args.width // 16, generator=g).pin_memory()
    kw = dict(prompt_embeds=pos, negative_prompt_embeds=neg, reference_latents=ref, video_length=args.frames,
              video_height=args.height, video_width=args.width, guidance_scale=5.0, flow_shift=5.0, seed=42,
              output_type="latent")
    pipe(num_inference_steps=args.warmup, **kw)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler()  # sampled by the rank that prints
    if rank == 0:
        sampler.start()
    start_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    out = pipe(num_inference_steps=args.steps, time_steps=True, **kw)
    lat = out.latents.cpu()
    e1.record()
    torch.cuda.synchronize()
    launches = stop_launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop(gpus=list(range(world))) if rank == 0 else None
    total_ms = e0.elapsed_time(e1)
    steps_ms = sum(out.step_ms)
    t = torch.tensor([total_ms, steps_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, steps_ms = t.tolist()
    err = ext().error_flag(True)
    if rank == 0:
        tokens = (args.frames - 1) // 4 + 1
        tokens *= (args.height // 32) * (args.width // 32)
        res = {
            "metric": METRIC, "value": steps_ms / 1e3, "unit": "s/video", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": steps_ms / args.steps, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random 4096-d caption embeddings, random first-frame latent, random-init 29B weights)",
            "config": {"model": f"PAN2 MMDiT {n_params / 1e9:.2f}B ({arch['num_layers']} layers)",
                       "global_batch": 1, "seq_len": 2 * (tokens + args.text_len), "video_tokens": tokens,
                       "parallelism": f"ulysses-sp{world}", "guidance": "CFG 5.0 (2 packed samples), i2v",
                       "l2": "58 GB of weights read per step; no extra flush", "valid_full_config": valid},
            "e2e": {"value": total_ms / 1e3, "unit": "s/video",
                    "h2d_bytes_per_step": (pos[0].numel() + neg[0].numel()) * 2 // args.steps,
                    "d2h_bytes_per_step": lat.numel() * 4 // args.steps,
                    "api": "pan2_b200.pipelines.PanVideoPipeline.__call__"},
            "gpu_launches": launches["total"], "clocks": clocks, "init_s": init_s, "device_error_flag": err,
            "step_ms_first_last": [out.step_ms[0], out.step_ms[-1]],
            "peak_mem_gb": torch.cuda.max_memory_allocated(device) / 1e9,
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
