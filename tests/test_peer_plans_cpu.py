"""Host-side plans behind the peer-memory kernels, checked on CPU for 2, 4 and 8 ranks: the fused
gather plan rebuilds every parameter from the ranks' shards, the fused reduce-scatter plan gives
each rank the sum of its rows over all ranks, and the distributed-Muon exchange layout keeps every
buffer disjoint and aligned.  The kernels run these run lists element for element."""
import pytest
import torch

from pan2_b200.parallel.sharded import build_unit
from pan2_b200.parallel.symm import GatherPlan, ReducePlan
from pan2_b200.training.engine import muon_exchange_layout
from tiny import tiny_model


def _unit(world):
    model = tiny_model()
    return build_unit(0, "blocks.0", model.blocks[0], world, prefix="blocks.0.")


def _shards(unit, full, world):
    out = []
    for r in range(world):
        sh = torch.zeros(unit.numel_shard)
        for s in unit.slots:
            a = min(s.rows, r * s.shard_rows)
            b = min(s.rows, a + s.shard_rows)
            if b > a:
                sh[s.shard_off:s.shard_off + (b - a) * s.cols] = full[s.full_off + a * s.cols:s.full_off + b * s.cols]
        out.append(sh)
    return out


def _runs(plan):
    return [tuple(int(x) for x in row) for row in plan.segs.tolist()]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gather_plan_rebuilds_full_weights(world):
    unit = _unit(world)
    full = torch.randn(unit.numel_full)
    shards = _shards(unit, full, world)
    plan = GatherPlan(unit, world, 0, "cpu")
    out = torch.full((unit.numel_full,), float("nan"))
    for (src, dst, n), peer in zip(_runs(plan), plan.seg_peer.tolist()):
        out[dst:dst + n] = shards[peer][src:src + n]
    for s in unit.slots:
        seg = slice(s.full_off, s.full_off + s.rows * s.cols)
        assert torch.equal(out[seg], full[seg]), s.name


@pytest.mark.parametrize("world", [2, 4, 8])
def test_reduce_plan_sums_owned_rows(world):
    unit = _unit(world)
    grads = [torch.randn(unit.numel_full) for _ in range(world)]
    total = sum(grads)
    for rank in range(world):
        plan = ReducePlan(unit, rank, world, "cpu")
        out = torch.zeros(unit.numel_shard)
        for src, dst, n in _runs(plan):
            out[dst:dst + n] = sum(g[src:src + n] for g in grads)
        expect = _shards(unit, total, world)[rank]
        assert torch.allclose(out, expect, atol=1e-5), rank


@pytest.mark.parametrize("world", [2, 4, 8])
def test_muon_exchange_layout_disjoint_and_aligned(world):
    unit = _unit(world)
    remote = [s for s in unit.slots if s.kind == "muon"]
    assert remote
    lay = muon_exchange_layout(remote, world)
    spans = []
    for s, off in zip(remote, lay["xoff"]):
        assert off % 256 == 0
        spans.append((off, off + s.shard_rows * s.cols * 2))
    spans.sort()
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:])) and spans[-1][1] <= lay["x_bytes"]
    for owner in range(world):
        mine = sorted((lay["roff"][j], lay["roff"][j] + s.rows_pad * s.cols * 2)
                      for j, s in enumerate(remote) if j % world == owner)
        assert all(a[1] <= b[0] for a, b in zip(mine, mine[1:]))
        assert not mine or mine[-1][1] <= lay["r_bytes"]
    for j, s in enumerate(remote):
        for r in range(world):  # every rank's slice of an owner's result is a 16-byte aligned address
            assert (lay["roff"][j] + r * s.shard_rows * s.cols * 2) % 16 == 0
