"""Trainer on CPU (tiny model, sample data): checkpoint resume is exact, non-finite updates are skipped,
anomalies roll back to the latest checkpoint, the heartbeat fires, checkpoints reshard."""
import json
import os
import socket
import threading
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pan2_b200.data.items import HashCaptionCodec
from pan2_b200.data.make_sample_data import write_sample_data
from pan2_b200.training.fault import AnomalyDetector, FaultInjector, Heartbeat, InjectedFault

TINY_OVERRIDES = dict(hidden_size=256, num_attention_heads=4, num_layers=2, rope_axes_dim=[16, 24, 24],
                      text_embed_dim=64)


@pytest.fixture(scope="module")
def data_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("trainer_data")
    write_sample_data(str(d), num_videos=6, num_images=4, latent_frames=3, height=8, width=12,
                      image_grids=((8, 8), (6, 10)))
    return d


def _cfg(data_dir, out, **over):
    from pan2_b200.config.training import parse_training_config
    argv = ["--transformer_config_overrides", json.dumps(TINY_OVERRIDES),
            "--packed_dataloader_meta_csv_path", str(data_dir / "videos.csv"),
            "--image_tar_path", str(data_dir / "images.tar"), "--image_sample_prob", "0.3",
            "--packed_joint_token_budget", "300", "--packed_video_token_budget", "260",
            "--packed_caption_token_budget", "200", "--packed_joint_segment_limit", "300",
            "--packed_caption_segment_limit", "100", "--packed_dataloader_max_num_seq", "3",
            "--packed_dataloader_num_buffers", "2", "--packed_dataloader_num_workers", "2",
            "--video_height", "128", "--video_width", "192",
            "--output_dir", str(out), "--learning_rate", "1e-3", "--warmup_steps", "2", "--log_interval", "1",
            "--text_encoder", "hash", "--optimizer_offload", "off", "--profile_step", "-1",
            "--anomaly_detection_warmup_steps", "1000"]
    for k, v in over.items():
        argv += [f"--{k}", str(v)]
    return parse_training_config(argv)


def _train(cfg):
    from pan2_b200.training.trainer import Trainer
    tr = Trainer(cfg, codec=HashCaptionCodec(embed_dim=64))
    hist = tr.train()
    return tr, hist


@pytest.mark.timeout(900)
def test_resume_is_exact(data_dir, tmp_path):
    _, full = _train(_cfg(data_dir, tmp_path / "a", max_steps=4, save_interval=2))
    _train(_cfg(data_dir, tmp_path / "b", max_steps=2, save_interval=2))
    assert os.path.exists(tmp_path / "b" / "checkpoint-2" / "COMPLETE")
    assert os.path.exists(tmp_path / "b" / "checkpoint-2" / "dataloader" / "0.json")
    assert os.path.exists(tmp_path / "b" / "save_logging" / "checkpoint_2.txt")
    tr, rest = _train(_cfg(data_dir, tmp_path / "b", max_steps=4, save_interval=2))
    assert [h["step"] for h in rest] == [2, 3]
    for a, b in zip(full[2:], rest):
        assert a["loss"] == pytest.approx(b["loss"], rel=1e-6, abs=1e-7), (a, b)
        assert a["grad_norm"] == pytest.approx(b["grad_norm"], rel=1e-5), (a, b)
        assert a["lr"] == b["lr"]


@pytest.mark.timeout(900)
def test_skip_then_recover_and_retention(data_dir, tmp_path):
    cfg = _cfg(data_dir, tmp_path / "c", max_steps=5, save_interval=2, save_total_limit=1,
               fault_injection="nan_loss@3", max_consecutive_skipped_steps=0)
    tr, hist = _train(cfg)
    steps = [h["step"] for h in hist]
    assert hist[steps.index(3)]["step_skipped"]
    assert tr.total_skipped == 1 and tr.recoveries == 1
    assert steps == [0, 1, 2, 3, 2, 3, 4]  # rolled back to checkpoint-2 after the anomaly at step 3
    kept = sorted(d for d in os.listdir(tmp_path / "c") if d.startswith("checkpoint-"))
    assert kept == ["checkpoint-5"]


@pytest.mark.timeout(600)
def test_skip_without_recovery_when_budget_allows(data_dir, tmp_path):
    cfg = _cfg(data_dir, tmp_path / "d", max_steps=3, save_interval=100, fault_injection="nan_loss@1",
               max_consecutive_skipped_steps=5)
    tr, hist = _train(cfg)
    assert [h["step_skipped"] for h in hist] == [False, True, False]
    assert tr.recoveries == 0


@pytest.mark.timeout(600)
def test_injected_exception_surfaces(data_dir, tmp_path):
    cfg = _cfg(data_dir, tmp_path / "e", max_steps=3, save_interval=100, fault_injection="raise@1")
    with pytest.raises(InjectedFault):
        _train(cfg)


@pytest.mark.timeout(900)
def test_corrupt_latest_checkpoint_falls_back(data_dir, tmp_path):
    _train(_cfg(data_dir, tmp_path / "f", max_steps=4, save_interval=2))
    tdir = tmp_path / "f" / "checkpoint-4" / "transformer"
    shards = [f for f in os.listdir(tdir) if f.endswith(".distcp")]
    assert shards
    for f in shards:
        with open(tdir / f, "wb") as fh:
            fh.write(b"not a checkpoint file")
    tr, rest = _train(_cfg(data_dir, tmp_path / "f", max_steps=5, save_interval=100))
    assert [h["step"] for h in rest] == [2, 3, 4]  # resumed from checkpoint-2



def test_checkpoint_retention_counts_complete_folders_only(tmp_path):
    from pan2_b200.checkpoint import io as ckpt
    out = tmp_path / "r"

    def folder(step, complete):
        d = out / f"checkpoint-{step}"
        d.mkdir(parents=True)
        if complete:
            ckpt.mark_complete(str(d), step)
        return d
    folder(1, True)
    folder(2, False)  # interrupted save older than the newest complete one: garbage
    folder(3, True)
    folder(9, False)  # interrupted save of a run that was later rolled back to step 3
    folder(5, True)   # the save that just finished
    removed = ckpt.cleanup_old(str(out), keep=1)
    assert sorted(os.path.basename(d) for d in removed) == ["checkpoint-1", "checkpoint-2", "checkpoint-3"]
    assert sorted(os.listdir(out)) == ["checkpoint-5", "checkpoint-9"]
    # a rewrite drops the marker first, so an interrupted rewrite reads as incomplete
    ckpt.clear_complete(str(out / "checkpoint-5"))
    assert not ckpt.is_complete(str(out / "checkpoint-5"))
    ckpt.clear_complete(str(out / "checkpoint-5"))  # no marker: nothing to do


@pytest.mark.timeout(900)
def test_resume_skips_incomplete_newer_folder(data_dir, tmp_path):
    _train(_cfg(data_dir, tmp_path / "g", max_steps=2, save_interval=2))
    (tmp_path / "g" / "checkpoint-7" / "transformer").mkdir(parents=True)  # an interrupted save
    tr, rest = _train(_cfg(data_dir, tmp_path / "g", max_steps=3, save_interval=100))
    assert [h["step"] for h in rest] == [2]  # resumed from checkpoint-2, not the incomplete checkpoint-7



def test_conditioning_schema_sets_and_checks_the_channel_widths(data_dir, tmp_path):
    from pan2_b200.training.trainer import architecture_from_config
    tok = architecture_from_config(_cfg(data_dir, tmp_path / "s"))  # the option's default: token_concat
    assert (tok["in_channels"], tok["out_channels"]) == (48, 48)
    ch = architecture_from_config(_cfg(data_dir, tmp_path / "s", conditioning_schema="channel_concat"))
    assert (ch["in_channels"], ch["out_channels"]) == (97, 48)
    bad = _cfg(data_dir, tmp_path / "s", conditioning_schema="channel_concat",
               transformer_config_overrides=json.dumps(dict(TINY_OVERRIDES, in_channels=48)))
    with pytest.raises(ValueError, match="in_channels=48 does not fit"):
        architecture_from_config(bad)
    with pytest.raises(ValueError, match="not divisible by the transformer patch size"):
        _train(_cfg(data_dir, tmp_path / "s", video_width=208, max_steps=1))  # 13 latent columns, patch 2


@pytest.mark.timeout(600)
def test_token_concat_trains_on_the_noised_latent_alone(data_dir, tmp_path):
    from pan2_b200.data.loader import PackedLoader
    from pan2_b200.training.trainer import Trainer
    for schema, width in (("token_concat", 48), ("channel_concat", 97)):
        tr = Trainer(_cfg(data_dir, tmp_path / schema, conditioning_schema=schema, max_steps=1),
                     codec=HashCaptionCodec(embed_dim=64))
        loader = tr.build_loader(None)
        batch, _ = next(iter(loader))
        loader.close()
        assert batch["hidden_states"].shape[0] == width * 4  # channels x (1 x 2 x 2) patch
        assert tr.engine.model.patch_embed.proj.in_channels == width
    with pytest.raises(ValueError, match="conditioning_schema"):
        PackedLoader(None, device="cpu", conditioning_schema="interleave")


def _dead_peer(rank, port, path):
    from pan2_b200.parallel.layout import init_parallel_layout
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    init_parallel_layout(cp=1, backend="gloo", timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks alive
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.time()
    err = None
    try:
        dist.all_reduce(t)  # the peer never joins
    except Exception as e:  # noqa: BLE001 - the collective must fail, whatever the error type
        err = type(e).__name__
    with open(path, "w") as f:
        json.dump(dict(err=err, waited=time.time() - t0), f)
    os._exit(0)


@pytest.mark.timeout(300)
def test_lost_rank_ends_next_collective_with_error(tmp_path):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "dead.json")
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_dead_peer, args=(r, port, path)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    with open(path) as f:
        r = json.load(f)
    assert r["err"] is not None, r
    assert r["waited"] < 60, r


def test_heartbeat_fires_when_stuck():
    fired = []
    hb = Heartbeat(rank=0, threshold_s=0.2, poll_s=0.05, on_stuck=fired.append).start()
    hb.beat("train_step", 7)
    time.sleep(0.6)
    hb.stop()
    assert fired and "stage='train_step'" in fired[0] and "step=7" in fired[0]
    fired.clear()
    hb = Heartbeat(rank=0, threshold_s=0.5, poll_s=0.05, on_stuck=fired.append).start()
    for _ in range(8):
        hb.beat()
        time.sleep(0.1)
    hb.stop()
    assert not fired


def test_anomaly_detector_rules():
    det = AnomalyDetector(warmup_steps=3)
    for s in range(5):
        assert not det(s, 1.0, 0.5)
    assert det(5, 30.0, 0.5)          # loss spike > 20x EMA
    assert det(6, 1.0, 10.0)          # grad spike > 6x EMA
    assert det(7, float("nan"), 0.5)
    assert det(8, 1.0, 2e6)           # hard limit
    early = AnomalyDetector(warmup_steps=100)
    early(0, 1.0, 0.5)
    assert not early(1, 30.0, 0.5)    # spikes are ignored during warmup
    assert early(2, float("inf"), 0.5)


def test_fault_spec_parsing():
    f = FaultInjector("nan_loss@2,stall@3:0.01,inf_grad@4/1", rank=0)
    assert f.poisons_update(2) and not f.poisons_update(4)
    assert FaultInjector("inf_grad@4/1", rank=1).poisons_update(4)
    t = time.time()
    f.before_step(3)
    assert time.time() - t >= 0.01
    m = f.after_step(2, {"loss": 1.0})["loss"]
    assert m != m  # NaN
    assert f.after_step(2, {"loss": 1.0})["loss"] == 1.0  # one-shot
    assert not f.poisons_update(2)
    with pytest.raises(ValueError):
        FaultInjector("melt@1")


# ---------------------------------------------------------------- checkpoint resharding

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _save_ranks(world, rank, port, root):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.checkpoint.io import save_engine, mark_complete
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from tiny import TINY_ARCH, tiny_batch
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    eng = TrainEngine(dict(TINY_ARCH), torch.device("cpu"), group=dist.group.WORLD, seed=4,
                      optim=OptimConfig(lr=1e-2), offload="off")
    with torch.device("meta"):
        m = PanVideoDiffusionTransformer(**TINY_ARCH)
    batch, _ = tiny_batch(m, seed=3)
    eng.forward_backward(batch)
    eng.grad_norm()
    eng.optimizer_step()
    save_engine(eng, root)
    sd = eng.sharded.full_state_dict()
    states = {}
    for u in eng.sharded.units:
        for s in u.slots:
            if not eng._is_muon(s):
                continue
            st = u.state["mom"]
            off = eng._soff[id(s)]
            states[s.name] = st[off:off + s.shard_rows * s.cols].clone()
            break
    dist.barrier()
    if rank == 0:
        mark_complete(root, 1)
        torch.save(sd, os.path.join(root, "expect.pt"))
    dist.destroy_process_group()


@pytest.mark.timeout(900)
def test_checkpoint_reshards_and_consolidates(tmp_path):
    root = str(tmp_path / "checkpoint-1")
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_save_ranks, args=(2, r, port, root)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=600)
        assert p.exitcode == 0
    expect = torch.load(os.path.join(root, "expect.pt"))
    from tiny import TINY_ARCH
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.checkpoint.io import load_engine, consolidate, load_plain_into_engine
    eng = TrainEngine(dict(TINY_ARCH), torch.device("cpu"), seed=99, optim=OptimConfig(lr=1e-2), offload="off")
    load_engine(eng, root)
    got = eng.sharded.full_state_dict()
    for k, v in expect.items():
        assert torch.equal(got[k], v), k
    assert eng.step_count == 1
    assert any(u.state["mom"] is not None and u.state["mom"].abs().sum() > 0 for u in eng.sharded.units)
    out = str(tmp_path / "plain")
    consolidate(root, out, dtype=torch.float32, max_shard_bytes=2 * 1024 ** 2)
    assert len([f for f in os.listdir(out) if f.endswith(".safetensors")]) > 1
    eng2 = TrainEngine(dict(TINY_ARCH), torch.device("cpu"), seed=98, optim=OptimConfig(lr=1e-2), offload="off")
    load_plain_into_engine(eng2, out)
    got2 = eng2.sharded.full_state_dict()
    for k, v in expect.items():
        assert torch.equal(got2[k], v), k
    # the reference's checkpoint converter reads a directory of safetensors shards by merging their
    # key -> tensor maps: the consolidated folder must give every parameter whole, by its name
    import glob
    from safetensors.torch import load_file
    merged = {}
    for shard in sorted(glob.glob(os.path.join(out, "*.safetensors"))):
        merged |= load_file(shard)
    assert set(merged) == set(expect)
    for k, v in expect.items():
        assert torch.equal(merged[k], v.reshape(merged[k].shape)), k


@pytest.mark.timeout(600)
def test_train_cli_runs_and_writes_checkpoint(data_dir, tmp_path):
    """``python train.py`` end to end on CPU (one process, hash captions) for two steps."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = tmp_path / "cli"
    argv = ["--transformer_config_overrides", json.dumps(TINY_OVERRIDES),
            "--packed_dataloader_meta_csv_path", str(data_dir / "videos.csv"),
            "--image_tar_path", str(data_dir / "images.tar"), "--image_sample_prob", "0.3",
            "--packed_joint_token_budget", "300", "--packed_video_token_budget", "260",
            "--packed_caption_token_budget", "200", "--packed_joint_segment_limit", "300",
            "--packed_caption_segment_limit", "100", "--packed_dataloader_max_num_seq", "3",
            "--packed_dataloader_num_buffers", "2", "--packed_dataloader_num_workers", "2",
            "--video_height", "128", "--video_width", "192", "--output_dir", str(out),
            "--learning_rate", "1e-3", "--warmup_steps", "2", "--log_interval", "1",
            "--text_encoder", "hash", "--optimizer_offload", "off", "--profile_step", "-1",
            "--max_steps", "2", "--save_interval", "2"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(root, "train.py")] + argv, cwd=root, env=env,
                       capture_output=True, text=True, timeout=500)
    assert r.returncode == 0, r.stderr[-2000:]
    assert os.path.exists(out / "checkpoint-2" / "COMPLETE")
    assert "Step 2/2" in (r.stdout + r.stderr) or "Step 1/2" in (r.stdout + r.stderr)


def test_launch_scripts_parse():
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for name in ("train.sh", "generate.sh"):
        r = subprocess.run(["bash", "-n", os.path.join(root, "launch", name)], capture_output=True, text=True)
        assert r.returncode == 0, (name, r.stderr)


@pytest.mark.timeout(600)
def test_wandb_reporting_with_a_stand_in_module(data_dir, tmp_path, monkeypatch):
    import sys
    import types
    calls = {"init": [], "log": [], "finish": 0}
    fake = types.ModuleType("wandb")
    fake.init = lambda **kw: calls["init"].append(kw)
    fake.log = lambda d, step=None: calls["log"].append((dict(d), step))

    def finish():
        calls["finish"] += 1
    fake.finish = finish
    monkeypatch.setitem(sys.modules, "wandb", fake)
    _train(_cfg(data_dir, tmp_path / "w", max_steps=2, save_interval=100, report_to="wandb"))
    assert len(calls["init"]) == 1 and "learning_rate" in calls["init"][0]["config"]
    assert len(calls["log"]) == 2
    for d, _ in calls["log"]:
        assert {"train/loss", "train/grad_norm"} <= set(d)
    assert calls["finish"] == 1
