"""Ulysses context parallelism with the all-to-alls folded into qkv_post / attention (peer memory)
against the NCCL all-to-all path, on 2 B200s of one node: same loss, same gradients."""
import os

import pytest
import torch

from test_comm_gpu import _spawn, gpu_world

pytestmark = pytest.mark.gpu

ARCH = dict(patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=512, num_attention_heads=4,
            num_layers=2, mlp_ratio=8.0, context_mlp_ratio=4.0, rope_axes_dim=(32, 48, 48), rope_theta=256,
            rope_temporal_scale=16 / 24, text_embed_dim=4096, zero_init_modulation=False)


def _cp_step(rank, world, port, path):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    from pan2_b200.data.cp_batch import broadcast_and_split
    from pan2_b200.data.synthetic import batch_to_device, synthetic_packed_batch
    from pan2_b200.ops._ext import ext
    from pan2_b200.parallel.layout import init_parallel_layout
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    L = init_parallel_layout(cp=world, backend="cpu:gloo,cuda:nccl", timeout_s=120)
    dev = torch.device("cuda", rank)
    out = {}
    for mode in ("0", "1"):
        os.environ["PAN_CP_FUSED"] = mode
        eng = TrainEngine(ARCH, dev, group=L.shard_group, seed=11, optim=OptimConfig(lr=1e-3), offload="off")
        eng.set_context_parallel(L.cp_group, world, L.cp_rank)
        src = None
        if L.cp_rank == 0:
            src = batch_to_device(synthetic_packed_batch(3, (3, 16, 16), 40, rope_axes=(32, 48, 48), seed=5), dev)
        batch, _ = broadcast_and_split(src, None, L, dev)
        loss = eng.forward_backward(batch)
        grads = [u.grad_shard.float().clone() for u in eng.sharded.units]
        norm = eng.grad_norm().clone()
        eng.optimizer_step()
        loss2 = eng.forward_backward(batch)
        torch.cuda.synchronize()
        out[mode] = dict(loss=loss.item(), loss2=loss2.item(), norm=norm.tolist(), grads=[g.cpu() for g in grads],
                         err=ext().error_flag(True))
        del eng
        torch.cuda.empty_cache()
    if rank == 0:
        torch.save(out, path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one node")
def test_fused_ulysses_matches_nccl_all_to_all(tmp_path):
    r = _spawn(_cp_step, gpu_world(), str(tmp_path / "cp.pt"))
    a, b = r["0"], r["1"]
    assert a["err"] == 0 and b["err"] == 0
    assert abs(a["loss"] - b["loss"]) < 1e-6 * abs(a["loss"]) + 1e-7, (a["loss"], b["loss"])
    assert abs(a["norm"][0] - b["norm"][0]) < 1e-2 * a["norm"][0], (a["norm"], b["norm"])
    for ga, gb in zip(a["grads"], b["grads"]):
        assert (ga - gb).abs().max().item() <= 2e-2 * (ga.abs().max().item() + 1e-12)
    assert abs(a["loss2"] - b["loss2"]) < 1e-2 * abs(a["loss2"])
