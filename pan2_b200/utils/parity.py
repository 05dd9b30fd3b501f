"""Multi-GPU correctness check of the fused peer-memory paths against their NCCL baselines.

Runs inside an already initialised job (every rank calls it) on a small model of the real block
structure (2 joint blocks, 4 heads of 128, or as many as context parallelism needs): one training
step with each path switched on
and off, the others held fixed, and reports the largest relative differences:

* ``fsdp_peer``: parameter gather + gradient reduce-scatter over peer memory (``PAN_PEER_COMM``)
  against NCCL all-gather / reduce-scatter -- loss, gradient shards, update;
* ``muon_peer``: distributed Muon's exchange over peer memory (``PAN_PEER_MUON``) against the NCCL
  all-to-all -- the optimizer's change of every parameter;
* ``adaln_peer``: the forward's AdaLN modulation projected straight from the peers' weight shards
  (``PAN_PEER_ADALN``) against the gathered weight -- loss, gradient shards, and the update as a
  relative RMS (the projection rounds differently from the GEMM, so AdamW's sign-like first step
  flips a few noise-level elements);
* ``cp_fused`` (context-parallel jobs): Ulysses all-to-alls folded into the kernels
  (``PAN_CP_FUSED``) against NCCL ``all_to_all_single`` -- loss and gradient shards.

Differences are max |a - b| / max |a| over all tensors (fp32 reduction order differs between the
paths, so small nonzero values are expected), except the ``_rms`` entries (||a - b|| / ||a||).
"""
from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Dict, Optional

import torch

SMALL_ARCH = dict(patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=512, num_attention_heads=4,
                  num_layers=2, mlp_ratio=8.0, context_mlp_ratio=4.0, rope_axes_dim=(32, 48, 48), rope_theta=256,
                  rope_temporal_scale=16 / 24, text_embed_dim=4096, zero_init_modulation=False)


@contextmanager
def _env(**kv):
    old = {k: os.environ.get(k) for k in kv}
    os.environ.update({k: str(v) for k, v in kv.items()})
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _rel(a, b) -> float:
    num = max(float((x.float() - y.float()).abs().max()) for x, y in zip(a, b))
    den = max(float(x.float().abs().max()) for x in a)
    return num / (den + 1e-30)


def _rel_rms(a, b) -> float:
    """||a - b|| / ||a|| over all tensors.  For an optimizer update after inputs that differ by
    rounding: AdamW's first step is about lr * sign(g), so a few elements whose gradients are pure
    rounding noise change by up to 2 lr (a max-norm of 1-2), while the update as a whole agrees."""
    num = sum(float((x.float() - y.float()).pow(2).sum()) for x, y in zip(a, b))
    den = sum(float(x.float().pow(2).sum()) for x in a)
    return (num / (den + 1e-30)) ** 0.5


def small_arch(cp: int = 1) -> dict:
    """The small model, with as many 128-wide heads as Ulysses needs (a multiple of ``cp``, at least 4)."""
    heads = -(-max(4, cp) // cp) * cp
    return dict(SMALL_ARCH, num_attention_heads=heads, hidden_size=heads * 128)


def _one_step(device, group, rank: int, layout=None, cp: int = 1) -> Dict:
    from ..data.synthetic import batch_to_device, synthetic_packed_batch
    from ..ops._ext import ext
    from ..training.engine import OptimConfig, TrainEngine
    eng = TrainEngine(small_arch(cp), device, group=group, seed=7, optim=OptimConfig(lr=1e-3), offload="off")
    if cp > 1:
        from ..data.cp_batch import broadcast_and_split
        eng.set_context_parallel(layout.cp_group, cp, layout.cp_rank)
        src = None
        if layout.cp_rank == 0:
            src = batch_to_device(synthetic_packed_batch(3, (3, 16, 16), 40, rope_axes=(32, 48, 48), seed=5), device)
        batch, _ = broadcast_and_split(src, None, layout, device)
    else:
        batch = batch_to_device(synthetic_packed_batch(2, (3, 16, 16), 40, rope_axes=(32, 48, 48), seed=rank), device)
    hi0 = [u.hi.float().clone() for u in eng.sharded.units]
    loss = eng.forward_backward(batch)
    grads = [u.grad_shard.float().clone() for u in eng.sharded.units]
    eng.grad_norm()
    eng.optimizer_step()
    delta = [u.hi.float() - h for u, h in zip(eng.sharded.units, hi0)]
    torch.cuda.synchronize(device)
    out = dict(loss=torch.tensor([float(loss)]), grads=grads, delta=delta, err=int(ext().error_flag(True)),
               peer=bool(eng.peer_comm), adaln=bool(eng.sharded.adaln))
    del eng
    torch.cuda.empty_cache()
    return out


def fused_path_parity(device, group, rank: int, layout=None, cp: int = 1) -> Dict[str, Optional[float]]:
    """Every rank calls this; returns the same dict of max relative differences on every rank."""
    import torch.distributed as dist
    res: Dict[str, Optional[float]] = {}
    if cp == 1:
        with _env(PAN_PEER_COMM=1, PAN_PEER_MUON=1, PAN_PEER_ADALN=0):
            peer = _one_step(device, group, rank)
        with _env(PAN_PEER_COMM=0, PAN_PEER_ADALN=0):
            base = _one_step(device, group, rank)
        with _env(PAN_PEER_COMM=1, PAN_PEER_MUON=0, PAN_PEER_ADALN=0):
            muon_nccl = _one_step(device, group, rank)
        with _env(PAN_PEER_COMM=1, PAN_PEER_MUON=1, PAN_PEER_ADALN=1):
            adaln = _one_step(device, group, rank)
        res["fsdp_peer_active"] = float(peer["peer"])
        res["fsdp_peer_loss"] = _rel([peer["loss"]], [base["loss"]])
        res["fsdp_peer_grads"] = _rel(peer["grads"], base["grads"])
        res["fsdp_peer_update"] = _rel(peer["delta"], base["delta"])
        res["muon_peer_update"] = _rel(peer["delta"], muon_nccl["delta"])
        res["adaln_peer_active"] = float(adaln["adaln"])
        res["adaln_peer_loss"] = _rel([adaln["loss"]], [peer["loss"]])
        res["adaln_peer_grads"] = _rel(adaln["grads"], peer["grads"])
        res["adaln_peer_update_rms"] = _rel_rms(adaln["delta"], peer["delta"])
        errs = peer["err"] | base["err"] | muon_nccl["err"] | adaln["err"]
    else:
        with _env(PAN_CP_FUSED=1):
            fused = _one_step(device, group, rank, layout, cp)
        with _env(PAN_CP_FUSED=0):
            base = _one_step(device, group, rank, layout, cp)
        res["cp_fused_loss"] = _rel([fused["loss"]], [base["loss"]])
        res["cp_fused_grads"] = _rel(fused["grads"], base["grads"])
        res["cp_fused_update"] = _rel(fused["delta"], base["delta"])
        errs = fused["err"] | base["err"]
    # the largest difference over ranks, agreed on every rank
    keys = sorted(res)
    t = torch.tensor([res[k] for k in keys] + [float(errs)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out = {k: float(v) for k, v in zip(keys, t.tolist()[:-1])}
    out["device_error_flag"] = int(t[-1].item())
    return out
