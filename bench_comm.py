"""Fused peer-memory collectives against their NCCL baselines, as fractions of the NVLink roofline.

    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench_comm.py \
        [--path gather|adaln|reduce|muon|ulysses|all] [--iters K] [--warmup W]

One rank per GPU of one node (N = 2, 4 or 8).  The units are the 29B model's (one joint block of
config/pretrain_29B_720p.yaml plus the root unit), built by the training engine itself, so every
number times the code path a training step runs:

* ``gather`` (path a): one block's FSDP parameter all-gather fused with the shard -> natural-layout
  unpack (``peer_gather``: each rank pulls its peers' bf16 ``hi`` rows out of symmetric memory)
  against NCCL ``all_gather_into_tensor`` followed by the unpack copies;
* ``adaln`` (path a, fused into the consuming op): the forward's AdaLN modulation of one block,
  ``a [5, H] @ W^T + b`` with ``W [6H, H]`` read row by row from the owning peers inside the
  projection kernel (``peer_gemv``, ``PAN_PEER_ADALN=1``), against gathering ``W`` (``peer_gather`` of
  that slot) and projecting the local copy with the GEMM;
* ``reduce`` (path b): one block's gradient reduce-scatter fused with the bf16 -> fp32 cast
  (device barrier + ``peer_reduce``) against the pack-with-cast copies + NCCL ``reduce_scatter_tensor``;
* ``muon`` (path d): the optimizer step with the distributed Muon exchange through peer memory
  (``PAN_PEER_MUON=1``) against the NCCL all-to-all version;
* ``ulysses`` (path c): forward + backward of one block with Ulysses context parallelism over all N
  ranks, the all-to-alls folded into ``qkv_post`` / attention (``PAN_CP_FUSED=1``) against NCCL
  all-to-alls (``PAN_CP_FUSED=0``), on one 5 s 720p clip (18,480 + 512 tokens).

Roofline (gather, adaln, reduce): the bytes that must cross NVLink into each GPU divided by the measured
peer-copy bandwidth, 770 GB/s per direction (900 nominal); the compute of these two paths (an
unpack, a cast and a sum) is far below its memory time, so the link time is the bound.  For muon
and ulysses the line reports the A/B step times and the link time of the exchanged bytes.

Timing: W untimed repetitions, then K repetitions between a barrier and a synchronize, CUDA events
on the launching stream, the max over ranks.  The operands (1.3 GB per block) exceed the 126 MB L2.
Rank 0 prints one JSON line per path.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LINK_GBS = 770.0  # measured peer copy, per direction per GPU


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--path", default="all", choices=("gather", "adaln", "reduce", "muon", "ulysses", "all"))
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default=os.path.join(ROOT, "config", "pretrain_29B_720p.yaml"))
    return ap.parse_args()


def _arch(config: str) -> dict:
    import yaml
    from pan2_b200.models.transformer import translate_architecture_config
    with open(config) as f:
        cfg = yaml.safe_load(f)
    arch = translate_architecture_config(cfg["model"]["transformer_config_overrides"])
    arch["zero_init_modulation"] = False
    arch["num_layers"] = 1
    return arch


def _timed(fn, iters: int, warmup: int, device) -> float:
    """Milliseconds per call: CUDA events on the current stream, max over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1) / iters], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _emit(rank: int, rec: dict) -> None:
    if rank == 0:
        print(json.dumps(rec), flush=True)


def bench_gather_reduce(args, arch, device, rank, world, paths):
    import torch
    import torch.distributed as dist
    from pan2_b200.ops._ext import ext
    from pan2_b200.parallel.sharded import pack_rows, unpack_rows
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    os.environ["PAN_PEER_COMM"] = "1"
    os.environ["PAN_PEER_ADALN"] = "1" if "adaln" in paths else "0"
    eng = TrainEngine(arch, device, group=dist.group.WORLD, seed=3, optim=OptimConfig(lr=1e-4), offload="off")
    sh = eng.sharded
    if not eng.peer_comm:
        _emit(rank, {"path": "gather/reduce", "unavailable": "peer memory is not available on this node"})
        return
    u = sh.units[0]  # one joint block
    grp = dist.group.WORLD
    bf, f32 = torch.bfloat16, torch.float32
    sh.hi_mem.barrier(0)  # every rank's hi shards are in place before any peer reads them
    if "gather" in paths:
        full_p = torch.empty(u.numel_full, dtype=bf, device=device)
        full_n = torch.empty(u.numel_full, dtype=bf, device=device)
        packed = torch.empty(world * u.numel_shard, dtype=bf, device=device)

        def peer():
            sh.gather_plans[u.index].run(sh.hi_mem, full_p)

        def nccl():
            dist.all_gather_into_tensor(packed, u.hi, group=grp)
            pk = packed.view(world, u.numel_shard)
            for s in u.slots:
                unpack_rows(pk, s, u.slot_full(full_n, s), world)

        t_peer = _timed(peer, args.iters, args.warmup, device)
        t_nccl = _timed(nccl, args.iters, args.warmup, device)
        link_bytes = (world - 1) / world * u.numel_full * 2
        roof_ms = link_bytes / (LINK_GBS * 1e9) * 1e3
        _emit(rank, {"path": "a: FSDP all-gather + unpack (peer_gather)", "n_gpus": world,
                     "unit": "blocks.0", "unit_bytes": u.numel_full * 2, "link_bytes_per_gpu": int(link_bytes),
                     "peer_ms": round(t_peer, 4), "nccl_ms": round(t_nccl, 4),
                     "roofline_ms": round(roof_ms, 4), "peer_of_roofline": round(roof_ms / t_peer, 3),
                     "nccl_of_roofline": round(roof_ms / t_nccl, 3), "equal": bool(torch.equal(full_p, full_n))})
    if "adaln" in paths and u.index in sh.adaln:
        from pan2_b200.ops.gemm import linear
        from pan2_b200.parallel.symm import GatherPlan
        proj, bias_slot = sh.adaln[u.index]
        w = proj.slot
        full = torch.empty(u.numel_full, dtype=bf, device=device)
        sh.gather_plans[u.index].run(sh.hi_mem, full)  # bias (and, for the reference result, W)
        bias = u.slot_full(full, bias_slot)
        from types import SimpleNamespace
        hi_off = proj.w_off - w.shard_off  # the unit's element offset in the hi buffer
        w_plan = GatherPlan(SimpleNamespace(slots=[w]), world, hi_off, device)  # gathers W alone
        gen = torch.Generator(device=device).manual_seed(5)
        a = torch.randn(5, w.cols, generator=gen, device=device).to(bf)
        y_p = torch.empty(5, w.rows, dtype=bf, device=device)

        def fused():
            proj.run(sh.hi_mem, a, bias, y_p)

        def gathered():
            w_plan.run(sh.hi_mem, full)
            return linear(a, u.slot_full(full, w), bias)

        t_fused = _timed(fused, args.iters, args.warmup, device)
        t_gath = _timed(gathered, args.iters, args.warmup, device)
        y_g = gathered()
        rel = ((y_p.float() - y_g.float()).abs().max() / y_g.float().abs().max().clamp_min(1e-30)).item()
        w_bytes = w.rows * w.cols * 2
        link_bytes = (world - 1) / world * w_bytes
        roof_ms = link_bytes / (LINK_GBS * 1e9) * 1e3
        _emit(rank, {"path": "a: AdaLN projection reading the weight from the peers (peer_gemv)", "n_gpus": world,
                     "unit": "blocks.0.modulation.linear", "weight_shape": [w.rows, w.cols], "weight_bytes": w_bytes,
                     "link_bytes_per_gpu": int(link_bytes), "fused_ms": round(t_fused, 4),
                     "gather_then_gemm_ms": round(t_gath, 4), "roofline_ms": round(roof_ms, 4),
                     "fused_of_roofline": round(roof_ms / t_fused, 3),
                     "gather_then_gemm_of_roofline": round(roof_ms / t_gath, 3), "max_rel_diff": rel})
    if "reduce" in paths:
        slot = 1
        g = sh.grad_mem.view(slot * sh.slot_elems * 2, u.numel_full, bf)
        gen = torch.Generator(device=device).manual_seed(100 + rank)
        g.copy_(torch.randn(u.numel_full, generator=gen, device=device, dtype=f32).to(bf))
        out_p = torch.empty(u.numel_shard, dtype=f32, device=device)
        out_n = torch.empty(u.numel_shard, dtype=f32, device=device)
        packed32 = torch.zeros(world * u.numel_shard, dtype=f32, device=device)

        def peer():
            sh.grad_mem.barrier(2)  # every rank's gradient is complete (part of the real cost)
            sh.reduce_plans[u.index].run(sh.slot_ptrs[slot], out_p)

        def nccl():
            pk = packed32.view(world, u.numel_shard)
            for s in u.slots:
                pack_rows(pk, s, u.slot_full(g, s), world)
            dist.reduce_scatter_tensor(out_n, packed32, op=dist.ReduceOp.SUM, group=grp)

        t_peer = _timed(peer, args.iters, args.warmup, device)
        t_nccl = _timed(nccl, args.iters, args.warmup, device)
        link_bytes = (world - 1) * u.numel_shard * 2
        roof_ms = link_bytes / (LINK_GBS * 1e9) * 1e3
        rel = ((out_p - out_n).abs().max() / out_n.abs().max().clamp_min(1e-30)).item()
        _emit(rank, {"path": "b: FSDP reduce-scatter + fp32 cast (peer_reduce)", "n_gpus": world,
                     "unit": "blocks.0", "unit_bytes": u.numel_full * 2, "link_bytes_per_gpu": int(link_bytes),
                     "peer_ms": round(t_peer, 4), "nccl_ms": round(t_nccl, 4),
                     "roofline_ms": round(roof_ms, 4), "peer_of_roofline": round(roof_ms / t_peer, 3),
                     "nccl_of_roofline": round(roof_ms / t_nccl, 3), "max_rel_diff": rel})
    torch.cuda.synchronize(device)
    dist.barrier()  # no rank frees symmetric memory while a peer may still read it
    assert ext().error_flag(True) == 0, "a device barrier gave up waiting"
    del eng


def bench_muon(args, arch, device, rank, world):
    import torch
    import torch.distributed as dist
    from pan2_b200.data.synthetic import batch_to_device, synthetic_packed_batch
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    rope = dict(rope_axes=tuple(arch["rope_axes_dim"]), rope_theta=float(arch["rope_theta"]),
                rope_scale=(float(arch["rope_temporal_scale"]), 1.0, 1.0))
    batch = batch_to_device(synthetic_packed_batch(1, (3, 44, 80), 512, seed=7 + rank, **rope), device)
    times = {}
    os.environ["PAN_PEER_COMM"] = "1"
    for mode in ("1", "0"):
        os.environ["PAN_PEER_MUON"] = mode
        eng = TrainEngine(arch, device, group=dist.group.WORLD, seed=3, optim=OptimConfig(lr=1e-4), offload="off")
        ms = []
        for it in range(args.warmup + args.iters):
            eng.forward_backward(batch)
            eng.grad_norm()
            torch.cuda.synchronize(device)
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            eng.optimizer_step()
            e1.record()
            torch.cuda.synchronize(device)
            if it >= args.warmup:
                ms.append(e0.elapsed_time(e1))
        t = torch.tensor([sum(ms) / len(ms)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times[mode] = float(t.item())
        del eng
        torch.cuda.synchronize(device)
        dist.barrier()
        torch.cuda.empty_cache()
    _emit(rank, {"path": "d: distributed Muon (peer exchange vs NCCL all-to-all), optimizer step of 1 block + root",
                 "n_gpus": world, "peer_ms": round(times["1"], 3), "nccl_ms": round(times["0"], 3)})


def bench_ulysses(args, arch, device, rank, world):
    import torch
    import torch.distributed as dist
    from pan2_b200.data.cp_batch import broadcast_and_split
    from pan2_b200.data.synthetic import batch_to_device, synthetic_packed_batch
    from pan2_b200.parallel.layout import init_parallel_layout
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    if arch["num_attention_heads"] % world:
        _emit(rank, {"path": "c", "unavailable": f"{arch['num_attention_heads']} heads over {world} ranks"})
        return
    L = init_parallel_layout(cp=world, backend="cpu:gloo,cuda:nccl", timeout_s=300)
    rope = dict(rope_axes=tuple(arch["rope_axes_dim"]), rope_theta=float(arch["rope_theta"]),
                rope_scale=(float(arch["rope_temporal_scale"]), 1.0, 1.0))
    times = {}
    for mode in ("1", "0"):
        os.environ["PAN_CP_FUSED"] = mode
        eng = TrainEngine(arch, device, group=L.shard_group, seed=3, optim=OptimConfig(lr=1e-4), offload="off")
        eng.set_context_parallel(L.cp_group, world, L.cp_rank)
        src = None
        if L.cp_rank == 0:
            src = batch_to_device(synthetic_packed_batch(1, (21, 44, 80), 512, seed=5, **rope), device)
        batch, _ = broadcast_and_split(src, None, L, device)
        times[mode] = _timed(lambda: eng.forward_backward(batch), args.iters, args.warmup, device)
        del eng
        torch.cuda.synchronize(device)
        dist.barrier()
        torch.cuda.empty_cache()
    S, hidden = 18480 + 512, arch["hidden_size"]
    # per block forward + backward: q, k, v and dO leave, o, dq, dk, dv come back: 8 exchanges of
    # (world - 1) / world of this rank's rows
    link_bytes = 8 * (world - 1) / world * (S / world) * hidden * 2
    _emit(rank, {"path": "c: Ulysses CP all-to-alls folded into qkv_post / attention, fwd+bwd of 1 block + root",
                 "n_gpus": world, "tokens": S, "fused_ms": round(times["1"], 3), "nccl_ms": round(times["0"], 3),
                 "link_bytes_per_gpu_per_block": int(link_bytes),
                 "link_ms_per_block": round(link_bytes / (LINK_GBS * 1e9) * 1e3, 4)})


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world < 2:
        print(json.dumps({"path": args.path, "unavailable": "run with torchrun on 2 or more GPUs of one node"}))
        return
    import torch
    import torch.distributed as dist
    rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", os.environ["RANK"]))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    arch = _arch(args.config)
    paths = ("gather", "adaln", "reduce", "muon", "ulysses") if args.path == "all" else (args.path,)
    from pan2_b200.parallel.layout import init_process_group
    init_process_group(300.0, "cpu:gloo,cuda:nccl")
    try:
        if "gather" in paths or "reduce" in paths or "adaln" in paths:
            bench_gather_reduce(args, arch, device, rank, world, paths)
        if "muon" in paths:
            bench_muon(args, arch, device, rank, world)
        if "ulysses" in paths:
            bench_ulysses(args, arch, device, rank, world)
    finally:
        torch.cuda.synchronize(device)
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
