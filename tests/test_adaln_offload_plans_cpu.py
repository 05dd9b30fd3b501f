"""Host-side plans of the peer-memory paths and the offload placement (CPU).

* the forward-only gather plan leaves exactly the AdaLN weight's run out, and the peer projection's
  row / offset arithmetic addresses that weight's shard rows;
* the engine's estimate of the root unit's offloadable bytes bounds what the root really allocates,
  so the budget set aside for it covers it;
* the grouped GEMM helpers zero exactly the rows outside the groups;
* the packed caption layout handles empty batches and captions of whole chunks;
* the host arena of the offloaded state hands out 256-byte aligned, zeroed views, declines what does
  not fit (the caller falls back to pinned blocks), unregisters on release, and hands out nothing
  when the driver refuses the registration (a stand-in for the CUDA runtime calls; no GPU here).
"""
import pytest
import torch

from tiny import TINY_ARCH


def _block_unit(world):
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    from pan2_b200.parallel.sharded import build_unit
    torch.manual_seed(0)
    model = PanVideoDiffusionTransformer(**TINY_ARCH)
    blk = model.blocks[0]
    return blk, build_unit(0, "blocks.0", blk, world, "blocks.0.")


def _runs(plan):
    segs = plan.segs.tolist()
    return [tuple(s) for s in segs[:len(plan.prefix)]], plan.seg_peer.tolist()


def test_forward_gather_plan_skips_only_the_adaln_weight():
    from pan2_b200.parallel.symm import GatherPlan, PeerProjection
    world, hi_off = 2, 1024
    blk, u = _block_unit(world)
    w = next(s for s in u.slots if s.module is blk.modulation.linear and s.attr == "weight")
    full, _ = _runs(GatherPlan(u, world, hi_off, "cpu"))
    part, _ = _runs(GatherPlan(u, world, hi_off, "cpu", skip=[w]))
    # the weight's rank slices are the runs whose destination lies inside its natural-layout range
    inside = [r for r in full if w.full_off <= r[1] < w.full_off + w.numel]
    assert len(inside) == world
    assert sorted(part) == sorted(r for r in full if r not in inside)
    assert sum(r[2] for r in inside) == w.numel
    proj = PeerProjection(w, hi_off)
    # row n lives on rank n // shard_rows at element w_off + (n - rank * shard_rows) * cols
    for n in (0, w.shard_rows - 1, w.shard_rows, w.rows - 1):
        r = n // w.shard_rows
        src = proj.w_off + (n - r * w.shard_rows) * w.cols
        run = next(x for x in inside if x[1] == w.full_off + r * w.shard_rows * w.cols)
        assert src == run[0] + (n - r * w.shard_rows) * w.cols


def test_peer_projection_rejects_unaligned_rows():
    from pan2_b200.parallel.symm import PeerProjection
    blk, u = _block_unit(2)
    w = next(s for s in u.slots if s.module is blk.modulation.linear and s.attr == "weight")
    with pytest.raises(ValueError, match="16-byte aligned"):
        PeerProjection(w, 3)


def test_root_reserve_bounds_the_root_state():
    from pan2_b200.training.engine import OptimConfig, TrainEngine
    eng = TrainEngine(dict(TINY_ARCH), torch.device("cpu"), seed=1, optim=OptimConfig(lr=1e-3), offload="off")
    root = eng.sharded.units[-1]
    actual = root.lo.numel() * root.lo.element_size() + sum(
        t.numel() * t.element_size() for t in root.state.values() if t is not None)
    with torch.device("meta"):
        from pan2_b200.models.transformer import PanVideoDiffusionTransformer
        m = PanVideoDiffusionTransformer(**TINY_ARCH)
    est = eng._offloadable_bytes([(n, tuple(p.shape)) for n, p in m.named_parameters()
                                  if not n.startswith("blocks.")])
    assert actual <= est <= actual + (2 << 20)


def test_rows_outside_the_groups_are_zeroed():
    from pan2_b200.ops.gemm import _rows_outside_zeroed
    t = torch.full((10, 3), 7.0)
    _rows_outside_zeroed(t, [2, 5, 8])
    assert t[:2].abs().sum() == 0 and t[8:].abs().sum() == 0
    assert (t[2:8] == 7).all()
    t = torch.full((4, 2), 1.0)
    _rows_outside_zeroed(t, [0, 4])
    assert (t == 1).all()


def test_packed_caption_layout_edges():
    from pan2_b200.models.qwen_packed import _layout
    lay = _layout([64, 128, 1], 64, "cpu")
    assert lay.n_chunks == 1 + 2 + 1
    assert int(lay.grid_valid.sum()) == 64 + 128 + 1
    assert [t.tolist() for t in lay.by_ordinal] == [[0, 1, 3], [2]]
    assert [t.tolist() for t in lay.seg_of_ordinal] == [[0, 1, 2], [1]]
    assert lay.pos.tolist()[:3] == [0, 1, 2] and lay.pos.tolist()[64] == 0
    empty = _layout([], 64, "cpu")
    assert empty.n_chunks == 0 and empty.grid_valid.numel() == 0


class _FakeCudart:
    """Stand-in for the driver's host registration (no GPU here): records the calls."""

    def __init__(self, rc=0):
        self.rc, self.registered, self.unregistered = rc, [], []

    def cudaHostRegister(self, ptr, size, flags):
        self.registered.append((ptr, size))
        return self.rc

    def cudaHostUnregister(self, ptr):
        self.unregistered.append(ptr)
        return 0


def test_host_arena_carves_aligned_zeroed_views(monkeypatch):
    import gc
    from pan2_b200.training import engine as E
    fake = _FakeCudart()
    monkeypatch.setattr(E.torch.cuda, "cudart", lambda: fake)
    arena = E._HostArena(1 << 16)
    assert arena.registered and fake.registered == [(arena.buf.data_ptr(), 1 << 16)]
    arena.buf.fill_(7)
    a = arena.take(10, torch.int16)
    b = arena.take(100, torch.float32)
    assert a.dtype == torch.int16 and b.dtype == torch.float32
    assert (a.data_ptr() - arena.buf.data_ptr()) % 256 == 0 and (b.data_ptr() - arena.buf.data_ptr()) % 256 == 0
    assert b.data_ptr() >= a.data_ptr() + 20
    assert a.abs().sum() == 0 and b.abs().sum() == 0
    assert arena.take(1 << 16, torch.uint8) is None  # does not fit: the caller falls back
    ptr = arena.buf.data_ptr()
    del arena
    gc.collect()
    assert fake.unregistered == [ptr]


def test_host_arena_refused_registration_hands_out_nothing(monkeypatch):
    from pan2_b200.training import engine as E
    fake = _FakeCudart(rc=1)
    monkeypatch.setattr(E.torch.cuda, "cudart", lambda: fake)
    arena = E._HostArena(4096)
    assert not arena.registered and arena.buf is None
    assert arena.take(4, torch.float32) is None
