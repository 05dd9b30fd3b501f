"""Sharded engine across 2 or 4 gloo ranks == the same engine on 1 rank (CPU).

Both ranks train on the same batch, so the global mean loss and its gradient equal the single-rank
ones; after one optimizer step (AdamW for 1-D/modulation tensors, Muon with local chunked NS for QKV
and owner-rank all-to-all NS for the other matrices) the gathered fp32 masters must match.

AdamW's first step is ``lr * g / (|g| + eps)``: with a tiny ``eps`` it moves every element by about
``lr * sign(g)``, so an element whose gradient is a near-cancellation (rounding noise of the CPU's
multi-threaded reductions, which differ from run to run) can flip sign and move by ``2 lr``.  The
test therefore uses ``eps = 1e-3``, where the first step is proportional to the gradient below that
size, and compares the update, not the sign of rounding noise."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tiny import TINY_ARCH, tiny_batch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _step(world, rank, port, out_q, hsdp_local=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    replicate = None
    if world > 1 and hsdp_local:
        # HSDP: shards within groups of `hsdp_local` ranks (one "node"), replicated across them
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_WORLD_SIZE=str(hsdp_local))
        from pan2_b200.parallel.layout import init_parallel_layout
        L = init_parallel_layout(cp=1, hybrid_shard=True, backend="gloo", timeout_s=120)
        assert L.shard_size == hsdp_local and L.replicate_size == world // hsdp_local
        group, replicate = L.shard_group, L.replicate_group
    elif world > 1:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        group = dist.group.WORLD
    else:
        group = None
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    arch = dict(TINY_ARCH)
    eng = TrainEngine(arch, torch.device("cpu"), group=group, seed=11,
                      optim=OptimConfig(lr=1e-2, weight_decay=0.1, max_grad_norm=0.5, adamw_eps=1e-3),
                      offload="off", replicate_group=replicate)
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**arch)
    batch, _ = tiny_batch(shape_model, seed=7)
    loss = eng.forward_backward(batch)
    norm = eng.grad_norm().clone()
    eng.optimizer_step()
    sd = eng.sharded.full_state_dict()
    if rank == 0:
        import tempfile
        path = os.path.join(tempfile.mkdtemp(), "sd.pt")
        torch.save((float(loss), norm.tolist(), sd), path)
        out_q.put(path)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _run(world, hsdp_local=0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_step, args=(world, r, port, q, hsdp_local)) for r in range(world)]
    for p in procs:
        p.start()
    path = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return torch.load(path)


@pytest.mark.timeout(900)
@pytest.mark.parametrize("world,hsdp_local", [(2, 0), (4, 0), (4, 2)], ids=["fsdp2", "fsdp4", "hsdp2x2"])
def test_multi_rank_step_matches_one_rank(world, hsdp_local):
    loss1, norm1, sd1 = _run(1)
    loss2, norm2, sd2 = _run(world, hsdp_local)
    assert abs(loss1 - loss2) < 1e-5 * abs(loss1) + 1e-6, (loss1, loss2)
    assert abs(norm1[0] - norm2[0]) < 1e-3 * norm1[0], (norm1, norm2)
    worst = (0.0, "")
    for k in sd1:
        a, b = sd1[k].float(), sd2[k].float()
        d = (a - b).abs().max().item() / (a.abs().max().item() + 1e-8)
        worst = max(worst, (d, k))
    assert worst[0] < 2e-3, worst


def test_checkpointing_modes_give_the_same_gradients():
    """Recompute (default), recompute with the kept attention forward, and no recompute."""
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    arch = dict(TINY_ARCH)
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**arch)
    batch, _ = tiny_batch(shape_model, seed=7)
    res = {}
    for mode in ((True, False), (True, True), (False, False)):
        eng = TrainEngine(arch, torch.device("cpu"), seed=11, optim=OptimConfig(lr=1e-2), offload="off")
        eng.set_activation_checkpointing(*mode)
        loss = eng.forward_backward(batch)
        assert not eng._kept_attn  # every kept attention output was consumed by its backward
        res[mode] = (float(loss), [u.full_grad.float().clone() for u in eng.sharded.units])
    base_loss, base = res[(True, False)]
    for mode in ((True, True), (False, False)):
        loss, grads = res[mode]
        assert loss == base_loss
        for a, b in zip(grads, base):  # bf16 gradient buffers: equal within a few ulps
            assert (a - b).abs().max().item() <= 1e-2 * b.abs().max().item() + 1e-7, mode
    eng = TrainEngine(arch, torch.device("cpu"), seed=11, offload="off")
    eng.set_activation_checkpointing(True, True)
    with pytest.raises(ValueError, match="context parallelism"):
        eng.set_context_parallel(None, 2, 0)
