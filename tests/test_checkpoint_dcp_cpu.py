"""Checkpoints as torch distributed checkpoints (CPU, gloo ranks).

Two ranks write ``transformer/`` and ``optimizer/`` of a tiny model as DCP folders, each its own
``Shard(0)`` rows.  The folder is then read (a) whole, the way the reference's converter reads a
trainer checkpoint (``dcp.load`` of full tensors without a process group), and equals the gathered
state dict; (b) by a one-rank engine and by a three-rank engine's row ranges, which reproduce the
weights and optimizer state; (c) by the reference converter's own ``load_native`` when
``PAN2_REFERENCE_DIR`` points at the reference source (skipped otherwise).
"""
import importlib.util
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


def _engine(group):
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    return TrainEngine(dict(TINY_ARCH), torch.device("cpu"), group=group, seed=3,
                       optim=OptimConfig(lr=1e-2, weight_decay=0.1, max_grad_norm=0.5), offload="off")


def _train_and_save(world, rank, port, root, out_q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    from pan2_b200.checkpoint.io import save_engine
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    eng = _engine(dist.group.WORLD)
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**TINY_ARCH)
    batch, _ = tiny_batch(shape_model, seed=9)
    eng.forward_backward(batch)
    eng.grad_norm()
    eng.optimizer_step()
    save_engine(eng, root)
    sd = eng.sharded.full_state_dict()
    if rank == 0:
        torch.save(sd, os.path.join(root, "expected.pt"))
        out_q.put("done")
    dist.barrier()
    dist.destroy_process_group()


@pytest.fixture(scope="module")
def saved(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("ckpt"))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_train_and_save, args=(2, r, port, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    assert q.get(timeout=600) == "done"
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return root, torch.load(os.path.join(root, "expected.pt"))


def test_folder_is_a_dcp_checkpoint_with_whole_tensors(saved):
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.metadata import TensorStorageMetadata
    root, expected = saved
    folder = os.path.join(root, "transformer")
    assert os.path.exists(os.path.join(folder, ".metadata"))
    reader = dcp.FileSystemReader(folder)
    md = reader.read_metadata()
    sd = {k: torch.empty(m.size, dtype=m.properties.dtype) for k, m in md.state_dict_metadata.items()
          if isinstance(m, TensorStorageMetadata)}
    dcp.load(sd, storage_reader=reader, no_dist=True)
    assert set(sd) == set(expected)
    for k, v in expected.items():
        assert torch.equal(sd[k], v.float().reshape(sd[k].shape)), k
    opt = dcp.FileSystemReader(os.path.join(root, "optimizer")).read_metadata()
    assert any(k.endswith(".momentum_buffer") for k in opt.state_dict_metadata)
    assert any(k.endswith(".exp_avg_sq") for k in opt.state_dict_metadata)


def test_reload_on_one_rank_restores_weights_and_state(saved):
    from pan2_b200.checkpoint.io import load_engine
    root, expected = saved
    eng = _engine(None)
    load_engine(eng, root)
    got = eng.sharded.full_state_dict()
    for k, v in expected.items():
        assert torch.equal(got[k].float(), v.float()), k
    assert eng.step_count == 1
    assert any(float(b.abs().sum()) > 0 for u in eng.sharded.units for b in u.state.values() if b is not None)


def test_row_ranges_of_three_ranks_cover_every_tensor(saved):
    """What each of three loading ranks would request, assembled, equals the saved tensors."""
    from pan2_b200.checkpoint.dcp_rows import load_row_chunks, tensor_specs
    from pan2_b200.checkpoint.io import rows_owned
    root, expected = saved
    folder = os.path.join(root, "transformer")
    specs = tensor_specs(folder)
    for name, (shape, _) in specs.items():
        parts = []
        for r in range(3):
            a, b = rows_owned(shape[0], 3, r)
            dest = {name: (a, torch.empty((b - a,) + tuple(shape[1:])))}
            load_row_chunks(folder, dest)
            parts.append(dest[name][1])
        assert torch.equal(torch.cat(parts), expected[name].float().reshape(shape)), name


def test_reference_converter_reads_the_checkpoint(saved):
    ref = os.environ.get("PAN2_REFERENCE_DIR")
    if not ref:
        pytest.skip("PAN2_REFERENCE_DIR is not set")
    spec = importlib.util.spec_from_file_location("ref_convert", os.path.join(ref, "scripts", "convert_checkpoint.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    root, expected = saved
    sd = mod.load_native(os.path.join(root, "transformer"))
    assert set(sd) == set(expected)
    for k, v in expected.items():
        assert torch.equal(sd[k], v.float().reshape(sd[k].shape)), k
