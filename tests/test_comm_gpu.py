"""Peer-memory collectives on 2+ B200s of one node: the fused gather / reduce-scatter engine path
equals the NCCL path, the forward's peer AdaLN projection equals the gathered-weight projection, and
a barrier whose peer never arrives returns with an error code.  The projection kernel's arithmetic
is also checked on one GPU, with the "peers" being local buffers."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ARCH = dict(patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=512, num_attention_heads=4,
            num_layers=2, mlp_ratio=8.0, context_mlp_ratio=4.0, rope_axes_dim=(32, 48, 48), rope_theta=256,
            rope_temporal_scale=16 / 24, text_embed_dim=4096, zero_init_modulation=False)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("cpu:gloo,cuda:nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    return dist


def _engine_step(rank, world, port, path):
    dist = _init(rank, world, port)
    from pan2_b200.data.synthetic import batch_to_device, synthetic_packed_batch
    from pan2_b200.ops._ext import ext
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    out = {}
    for mode in ("0", "1", "adaln"):
        os.environ["PAN_PEER_COMM"] = "0" if mode == "0" else "1"
        os.environ["PAN_PEER_ADALN"] = "1" if mode == "adaln" else "0"
        eng = TrainEngine(ARCH, torch.device("cuda", rank), group=dist.group.WORLD, seed=7,
                          optim=OptimConfig(lr=1e-3), offload="off")
        assert eng.peer_comm == (mode != "0")
        assert bool(eng.sharded.adaln) == (mode == "adaln")
        batch = batch_to_device(synthetic_packed_batch(2, (3, 16, 16), 40, rope_axes=(32, 48, 48), seed=rank), "cuda")
        hi0 = [u.hi.float().clone() for u in eng.sharded.units]
        loss = eng.forward_backward(batch)
        grads = [u.grad_shard.clone() for u in eng.sharded.units]
        norm = eng.grad_norm().clone()
        eng.optimizer_step()
        delta = [(u.hi.float() - h0).cpu() for u, h0 in zip(eng.sharded.units, hi0)]
        loss2 = eng.forward_backward(batch)  # second step: exercises the barriers and the gradient ring again
        torch.cuda.synchronize()
        out[mode] = dict(loss=loss.item(), loss2=loss2.item(), norm=norm.tolist(), grads=[g.cpu() for g in grads],
                         hi=[u.hi.float().cpu() for u in eng.sharded.units], delta=delta,
                         err=ext().error_flag(True))
        del eng
        torch.cuda.empty_cache()
    if rank == 0:
        torch.save(out, path)
    dist.barrier()
    dist.destroy_process_group()


def _barrier_timeout(rank, world, port, path):
    dist = _init(rank, world, port)
    from pan2_b200.ops._ext import ext
    from pan2_b200.parallel.symm import PeerMemory
    pm = PeerMemory(4096, dist.group.WORLD, torch.device("cuda", rank))
    pm.barrier(3, timeout_ms=2000)  # both ranks: passes
    torch.cuda.synchronize()
    ok_first = ext().error_flag(True) == 0
    if rank == 0:
        pm.barrier(4, timeout_ms=500)  # rank 1 never arrives on this channel
        torch.cuda.synchronize()
        err = ext().error_flag(True)
        torch.save(dict(ok_first=ok_first, err=err), path)
    dist.barrier()
    dist.destroy_process_group()


def gpu_world() -> int:
    """Ranks for the multi-GPU tests: 2, or ``PAN_TEST_WORLD`` (capped by the visible GPUs)."""
    return max(2, min(torch.cuda.device_count(), int(os.environ.get("PAN_TEST_WORLD", "2"))))


def _spawn(fn, world, path):
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=fn, args=(r, world, port, path)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=600)
        assert p.exitcode == 0
    return torch.load(path)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one node")
def test_peer_memory_engine_matches_nccl(tmp_path):
    r = _spawn(_engine_step, gpu_world(), str(tmp_path / "r.pt"))
    a, b = r["0"], r["1"]
    assert a["err"] == 0 and b["err"] == 0
    assert abs(a["loss"] - b["loss"]) < 1e-6 * abs(a["loss"]) + 1e-7
    assert abs(a["norm"][0] - b["norm"][0]) < 1e-4 * a["norm"][0]
    for ga, gb in zip(a["grads"], b["grads"]):
        assert (ga - gb).abs().max().item() <= 1e-5 * (ga.abs().max().item() + 1e-12)
    for ha, hb in zip(a["hi"], b["hi"]):
        assert (ha - hb).abs().max().item() <= 1e-2 * (ha.abs().max().item() + 1e-12)
    # the optimizer's change of every parameter (Muon over peer memory vs NCCL all-to-all, AdamW)
    for da, db in zip(a["delta"], b["delta"]):
        assert (da - db).abs().max().item() <= 5e-2 * (da.abs().max().item() + 1e-12)
    assert abs(a["loss2"] - b["loss2"]) < 1e-3 * abs(a["loss2"])
    # the forward's modulation rows from the peer projection (accumulation order differs from the GEMM)
    c = r["adaln"]
    assert c["err"] == 0
    assert abs(c["loss"] - b["loss"]) < 1e-3 * abs(b["loss"])
    for gb, gc in zip(b["grads"], c["grads"]):
        assert (gb - gc).abs().max().item() <= 3e-2 * (gb.abs().max().item() + 1e-12)
    assert abs(c["loss2"] - b["loss2"]) < 2e-3 * abs(b["loss2"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one node")
def test_barrier_times_out_with_error_code(tmp_path):
    r = _spawn(_barrier_timeout, 2, str(tmp_path / "b.pt"))
    assert r["ok_first"]
    assert r["err"] == 101  # rank 0 gave up waiting for peer 1


@pytest.mark.parametrize("k,N,K,ranks", [(5, 3072, 512, 2), (8, 1000, 256, 3), (1, 30720, 5120, 8)])
def test_peer_projection_kernel_matches_fp32(k, N, K, ranks):
    """y = a W^T + b with W's row shards in separate buffers (as on separate ranks) at an offset."""
    from pan2_b200.ops._ext import ext
    torch.manual_seed(k * N)
    W = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    a = torch.randn(k, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, device="cuda").to(torch.bfloat16)
    rows = -(-N // ranks)
    off = 8 * 37
    bufs = []
    for r in range(ranks):
        buf = torch.zeros(off + rows * K, device="cuda", dtype=torch.bfloat16)
        part = W[r * rows:(r + 1) * rows]
        buf[off:off + part.numel()] = part.reshape(-1)
        bufs.append(buf)
    peers = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device="cuda")
    y = torch.empty(k, N, device="cuda", dtype=torch.bfloat16)
    ext().peer_gemv(peers, off, rows, a, b, y)
    ref = a.float() @ W.float().t() + b.float()
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    y2 = torch.empty_like(y)
    ext().peer_gemv(peers, off, rows, a, None, y2)
    assert (y2.float() - (ref - b.float())).abs().max().item() <= 1e-2 * ref.abs().max().item()
