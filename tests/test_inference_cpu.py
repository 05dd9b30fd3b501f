"""Generation on CPU: scheduler, schedules, guidance, prompt inputs, packed-CFG == dense masked
forward, sequence parallel == single rank."""
import json
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pan2_b200.inference.guidance import apply_guidance, resolve_guidance_plan, validate_sampling_extensions
from pan2_b200.inference.inputs import is_complete, load_inference_inputs, render_negative_duration, resolve_frames
from pan2_b200.inference.scheduler import FlowEulerScheduler, apply_timestep_schedule, shifted_sigmas

from tiny import TINY_ARCH

ARCH = dict(TINY_ARCH, text_embed_dim=64)


def test_scheduler_grid_and_step():
    s = FlowEulerScheduler(shift=5.0)
    s.set_timesteps(10)
    g = torch.linspace(1, 0, 11)
    assert torch.allclose(s.sigmas, 5 * g / (1 + 4 * g))
    assert torch.allclose(s.timesteps, s.sigmas[:-1] * 1000)
    x = torch.randn(4, dtype=torch.bfloat16)
    v = torch.randn(4, dtype=torch.bfloat16)
    y = s.step(v, s.timesteps[0], x)
    assert y.dtype == torch.float32
    assert torch.allclose(y, x.float() + v.float() * float(s.sigmas[1] - s.sigmas[0]))
    assert s.step_index == 1
    with pytest.raises(ValueError):
        s.step(v, 3, x)


def test_duplicate_timestep_resolves_to_later():
    s = FlowEulerScheduler()
    s.set_timesteps(4)
    s._set(torch.tensor([1.0, 0.5, 0.5, 0.25, 0.0]), None)
    assert s.index_of(torch.tensor(500.0)) == 2


def test_early_refine_2x():
    s = FlowEulerScheduler(shift=5.0)
    s.set_timesteps(50)
    base = s.sigmas.clone()
    ts = apply_timestep_schedule(s, "early_refine_2x")
    assert ts.numel() == 50 and s.sigmas.numel() == 51
    assert float(s.sigmas[1]) == pytest.approx(float((base[0] + base[1]) / 2))
    assert float(s.sigmas[3]) == pytest.approx(float((base[1] + base[2]) / 2))
    kept = set(round(float(v), 6) for v in s.sigmas)
    assert round(float(base[15]), 6) not in kept and round(float(base[25]), 6) not in kept
    with pytest.raises(ValueError):
        validate_sampling_extensions(30, "early_refine_2x")


def test_guidance_plan():
    p = resolve_guidance_plan(10, start_step=2, end_step=8, skip_interval=(4, 6))
    assert [p.active(i) for i in range(10)] == [False, False, True, True, False, False, True, True, False, False]
    w = resolve_guidance_plan(10, start_step=2, warmup_scale=2.0)
    assert w.active(0) and w.scale_at(0, 5.0) == 2.0 and w.scale_at(3, 5.0) == 5.0
    neg, pos = torch.zeros(3, dtype=torch.bfloat16), torch.ones(3, dtype=torch.bfloat16)
    assert torch.equal(apply_guidance(neg, pos, 4.0, step_index=0, plan=p), pos)
    assert torch.equal(apply_guidance(neg, pos, 4.0, step_index=2, plan=p), neg + 4.0 * (pos - neg))
    stg = resolve_guidance_plan(10, stg_scale=0.5)
    weak = torch.full((3,), 0.5, dtype=torch.bfloat16)
    out = apply_guidance(neg, pos, 4.0, step_index=1, plan=stg, weak_predict_fn=lambda: weak)
    assert torch.allclose(out.float(), torch.full((3,), 4.0 + 0.25))
    for bad in (dict(start_step=5, end_step=5), dict(skip_interval=(3, 2)), dict(warmup_scale=0.5)):
        with pytest.raises(ValueError):
            resolve_guidance_plan(10, **bad)


def test_inputs(tmp_path):
    assert resolve_frames({"duration_sec": 5}, 24) == 121
    assert resolve_frames({"duration_sec": 5.1}, 24) == 125
    assert resolve_frames({"frames": 33}) == 33
    assert resolve_frames({}, fallback=241) == 241
    neg = json.dumps({"a": {"time_range_sec": "0 to 10"}, "b": [{"time_range_sec": "x"}]})
    r = json.loads(render_negative_duration(neg, 121, 24))
    assert r["a"]["time_range_sec"] == "0 to 5" and r["b"][0]["time_range_sec"] == "0 to 5"
    assert render_negative_duration("plain text", 121) == "plain text"
    img = tmp_path / "ref.png"
    img.write_bytes(b"x")
    entries = [{"id": "a b", "prompt": "p1", "duration_sec": 2},
               {"prompt": "p2", "image_path": str(img)},
               {"refined_prompt": "p3r", "prompt": "p3", "relative_path": "sub/x.mp4"}]
    pj = tmp_path / "prompts.json"
    pj.write_text(json.dumps({"entries": entries}))
    recs = load_inference_inputs(pj, tmp_path / "out", task="auto")
    assert [r["task"] for r in recs] == ["t2v", "i2v", "t2v"]
    assert recs[0]["output_path"].endswith("t2v/t2v_a_b.mp4") and recs[0]["video_length"] == 49
    assert recs[2]["prompt"] == "p3r"
    assert len(load_inference_inputs(pj, tmp_path / "out", task="t2v", shard_index=1, shard_count=2)) == 1
    pj.write_text(json.dumps([{"prompt": "p", "relative_path": "../evil.mp4"}]))
    with pytest.raises(ValueError):
        load_inference_inputs(pj, tmp_path / "out")


def test_is_complete(tmp_path):
    import argparse
    a = argparse.Namespace(output_path=str(tmp_path / "v.mp4"), seed=1, prompt="x", output_dir="o")
    assert not is_complete(a)
    (tmp_path / "v.mp4").write_bytes(b"1")
    (tmp_path / "v_config.json").write_text(json.dumps({"arguments": {"seed": 1, "prompt": "x"}}))
    assert is_complete(a)
    a.seed = 2
    with pytest.raises(ValueError):
        is_complete(a)


def _model(seed=0):
    from pan2_b200.pipelines.video import build_inference_model
    return build_inference_model(ARCH, "cpu", dtype=torch.float32, seed=seed)


def test_packed_cfg_prediction_matches_dense_masked_forward():
    from pan2_b200.pipelines.video import PackedDiTRunner
    from pan2_b200.data.patching import patchify, unpatchify
    torch.manual_seed(0)
    m = _model()
    grid = (3, 8, 8)
    N = 3 * 4 * 4
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, N, 48 * 4, generator=g)
    cond = torch.randn(1, N, 49 * 4, generator=g)
    lens = [7, 12]
    text = [torch.randn(n, 64, generator=g) for n in lens]
    t = torch.tensor([700.0, 700.0])
    runner = PackedDiTRunner(m, "cpu")
    p = runner.plan(grid, lens)
    v = runner.predict(p, x.repeat(2, 1, 1), cond.repeat(2, 1, 1), t, torch.cat(text))
    # dense reference: padded text + mask, latents [B, 97, T, H, W]
    L = max(lens)
    tpad = torch.zeros(2, L, 64)
    mask = torch.zeros(2, L, dtype=torch.long)
    for i, tt in enumerate(text):
        tpad[i, :lens[i]] = tt
        mask[i, :lens[i]] = 1
    feat = torch.cat([x, cond], -1)[0]
    lat = unpatchify(feat, (3, 4, 4), (1, 2, 2), 97).unsqueeze(0).repeat(2, 1, 1, 1, 1)
    with torch.no_grad():
        vd, _ = m.forward_dense(lat, t, tpad, mask)
    vd_tok = torch.stack([patchify(vd[i], (1, 2, 2)).t() for i in range(2)])
    err = (v.float() - vd_tok).abs().max().item() / vd_tok.abs().max().item()
    assert err < 1e-4, err


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _sample(world, rank, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from pan2_b200.parallel.layout import init_parallel_layout
    from pan2_b200.pipelines.video import PanVideoPipeline
    L = init_parallel_layout(cp=world, backend="gloo", timeout_s=120)
    m = _model()
    pipe = PanVideoPipeline(m, device="cpu", sp_group=L.cp_group if world > 1 else None, num_inference_steps=3)
    g = torch.Generator().manual_seed(5)
    pos = [torch.randn(9, 64, generator=g)]
    neg = [torch.randn(4, 64, generator=g)]
    ref = torch.randn(48, 1, 8, 8, generator=g)
    out = pipe(prompt_embeds=pos, negative_prompt_embeds=neg, video_length=9, video_height=128, video_width=128,
               seed=3, reference_latents=ref, output_type="latent", guidance_scale=4.0)
    if rank == 0:
        torch.save(out.latents, path)
    dist.barrier()
    dist.destroy_process_group()


def _run(world, tmp):
    ctx = mp.get_context("spawn")
    port = _free_port()
    path = os.path.join(tmp, f"lat{world}.pt")
    ps = [ctx.Process(target=_sample, args=(world, r, port, path)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=600)
        assert p.exitcode == 0
    return torch.load(path)


@pytest.mark.timeout(900)
def test_sequence_parallel_sampling_matches_single_rank(tmp_path):
    a = _run(1, str(tmp_path))
    b = _run(2, str(tmp_path))
    assert a.shape == (1, 48, 3, 8, 8)
    assert torch.isfinite(a).all()
    err = (a - b).abs().max().item() / a.abs().max().item()
    assert err < 1e-4, err


def test_generate_cli_latent_output_and_skip(tmp_path):
    from pan2_b200.generate import main
    prompts = tmp_path / "p.json"
    prompts.write_text(json.dumps([{"id": "one", "prompt": "a red ball", "frames": 5},
                                   {"id": "two", "prompt": "a blue cube", "frames": 5}]))
    over = json.dumps(dict(ARCH, rope_axes_dim=list(ARCH["rope_axes_dim"]), patch_size=list(ARCH["patch_size"])))
    argv = ["--prompt_json", str(prompts), "--output_dir", str(tmp_path / "out"), "--transformer_config_overrides",
            over, "--text_encoder", "hash", "--output_type", "latent", "--video_height", "64", "--video_width", "64",
            "--num_inference_steps", "2", "--flow_shift", "5.0", "--guidance_scale", "4.0", "--dtype", "fp32"]
    written = main(argv)
    assert len(written) == 2 and all(os.path.exists(w) for w in written)
    from safetensors.torch import load_file
    lat = load_file(written[0])["latent"]
    assert lat.shape == (48, 2, 4, 4) and torch.isfinite(lat).all()
    cfg = json.loads((tmp_path / "out" / "t2v_one_config.json").read_text())
    assert cfg["arguments"]["seed"] == 42
    assert not [f for f in os.listdir(tmp_path / "out") if ".partial" in f]  # every file renamed into place
    assert main(argv + ["--skip_existing"]) == []
    # the reference's runtime flags: block streaming (no prefetch) and --compile give the same latents
    argv2 = [a if a != str(tmp_path / "out") else str(tmp_path / "out2") for a in argv]
    again = main(argv2 + ["--offload", "blocks", "--offload_prefetch", "false", "--compile"])
    assert torch.equal(load_file(again[0])["latent"], lat)


def test_write_video_renames_a_finished_file_into_place(tmp_path, monkeypatch):
    import sys
    import types
    from pan2_b200.generate import write_video
    seen = []

    def mimwrite(path, frames, fps, **opts):
        seen.append(path)
        assert not os.path.exists(tmp_path / "v.mp4")  # the final name appears only once the write is done
        with open(path, "wb") as f:
            f.write(b"x" * len(frames))
    fake = types.SimpleNamespace(mimwrite=mimwrite, imwrite=lambda path, frame: open(path, "wb").write(b"y"))
    monkeypatch.setitem(sys.modules, "imageio", types.ModuleType("imageio"))
    sys.modules["imageio"].__dict__.update(vars(fake))
    out = write_video(torch.rand(3, 4, 8, 8), str(tmp_path / "v.mp4"))
    assert out == str(tmp_path / "v.mp4") and seen == [str(tmp_path / "v.partial.mp4")]
    assert os.listdir(tmp_path) == ["v.mp4"] and (tmp_path / "v.mp4").read_bytes() == b"xxxx"


class _CountingTextEncoder:
    """Text encoder stand-in that records where it was when it ran (offloading moves it)."""

    def __init__(self, dim=64):
        from pan2_b200.models.text_encoder import HashTextEncoder
        self.inner = HashTextEncoder(embed_dim=dim)
        self.moves = []

    def to(self, device):
        self.moves.append(str(torch.device(device)))
        return self

    def encode(self, texts, device=None):
        return self.inner.encode(texts, device)


def _pipe_latents(offload, prefetch=True, stg=False):
    from pan2_b200.pipelines.video import PanVideoPipeline
    torch.manual_seed(0)
    m = _model()
    te = _CountingTextEncoder()
    pipe = PanVideoPipeline(m, te, device="cpu", num_inference_steps=3)
    if offload is not None:
        pipe.configure_runtime(offload=offload, prefetch=prefetch)
    extra = dict(stg_scale=0.5, stg_skip_layers=[1]) if stg else {}
    out = pipe(prompt="a red ball", negative_prompt="blurry", video_length=9, video_height=128, video_width=128,
               seed=3, output_type="latent", guidance_scale=4.0, **extra)
    return out.latents, te, m


@pytest.mark.parametrize("stg", [False, True])
def test_offload_modes_give_identical_samples(stg):
    base, _, _ = _pipe_latents(None, stg=stg)
    for mode in ("none", "models", "blocks"):
        lat, te, m = _pipe_latents(mode, stg=stg)
        assert torch.equal(lat, base), mode
        if mode != "none":
            assert te.moves[0] == "cpu" and te.moves[1:] == ["cpu", "cpu"]  # parked, then in and out once
        if mode == "blocks":
            s = m.block_streamer
            # after the run every block points at its host buffer again (nothing holds slot memory)
            for i, blk in enumerate(m.blocks):
                host = s.host[i]
                for prm in blk.parameters():
                    ptr = prm.data_ptr()
                    assert host.data_ptr() <= ptr < host.data_ptr() + host.numel()


def test_block_streamer_follows_the_run_order():
    from pan2_b200.inference.offload import BlockStreamer
    blocks = torch.nn.ModuleList([torch.nn.Linear(4, 4) for _ in range(4)])
    ref = [b.weight.detach().clone() for b in blocks]
    s = BlockStreamer(blocks, "cpu", prefetch=True)  # prefetch needs CUDA; on the CPU it copies in place
    seen = []
    for i, blk in s.run(blocks, [0, 2, 3]):
        slot = s.slots[0]
        assert slot.data_ptr() <= blk.weight.data_ptr() < slot.data_ptr() + slot.numel()
        assert torch.equal(blk.weight, ref[i])
        seen.append(i)
    assert seen == [0, 2, 3]
    with pytest.raises(RuntimeError):
        for i, blk in s.run(blocks, [1, 2]):
            raise RuntimeError("a block failed")
    assert all(torch.equal(b.weight, r) for b, r in zip(blocks, ref))
    assert all(s.host[i].data_ptr() <= b.weight.data_ptr() < s.host[i].data_ptr() + s.host[i].numel()
               for i, b in enumerate(blocks))


def test_choose_offload(monkeypatch):
    from pan2_b200.inference.offload import choose_offload
    assert choose_offload("auto", 10 ** 12, "cpu") == "none"
    assert choose_offload("models", 1, "cpu") == "models"
    with pytest.raises(ValueError):
        choose_offload("disk", 1, "cpu")
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None: (100, 200))
    assert choose_offload("auto", 99, "cuda:0") == "none"
    assert choose_offload("auto", 100, "cuda:0") == "blocks"


def test_sampler_rejects_a_token_concat_transformer():
    from pan2_b200.pipelines.video import PanVideoPipeline, build_inference_model
    m = build_inference_model(dict(ARCH, in_channels=48), "cpu", dtype=torch.float32)
    pipe = PanVideoPipeline(m, device="cpu", num_inference_steps=2)
    with pytest.raises(ValueError, match="channel_concat"):
        pipe(prompt_embeds=[torch.randn(5, 64)], video_length=5, video_height=64, video_width=64,
             output_type="latent", guidance_scale=1.0)
