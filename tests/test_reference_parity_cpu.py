"""Bit-for-bit parity of the rewritten model / sampling / input modules with the reference itself.

Runs only when ``PAN2_REFERENCE_DIR`` points at the reference source tree (skipped otherwise).  Each
reference module is loaded from its file (they need only torch, plus a two-class stand-in for
diffusers' config mixins in the scheduler's case) and compared with this framework's module on
random inputs: equal tensors, equal records, and the same inputs rejected.
"""
import importlib.util
import json
import os
import sys
import types

import pytest
import torch

REF = os.environ.get("PAN2_REFERENCE_DIR")
pytestmark = pytest.mark.skipif(not REF, reason="PAN2_REFERENCE_DIR is not set")


def _load(rel: str, name: str):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _diffusers_stand_in():
    """Just enough of diffusers for the reference scheduler: ``register_to_config`` stores the
    constructor arguments on ``self.config``."""
    import functools
    import inspect
    if "diffusers" in sys.modules:
        return
    cfg_mod = types.ModuleType("diffusers.configuration_utils")

    class ConfigMixin:
        pass

    def register_to_config(init):
        @functools.wraps(init)
        def wrapped(self, *args, **kwargs):
            bound = inspect.signature(init).bind(self, *args, **kwargs)
            bound.apply_defaults()
            self.config = types.SimpleNamespace(**{k: v for k, v in bound.arguments.items() if k != "self"})
            init(self, *args, **kwargs)
        return wrapped

    cfg_mod.ConfigMixin, cfg_mod.register_to_config = ConfigMixin, register_to_config
    sched_mod = types.ModuleType("diffusers.schedulers.scheduling_utils")
    sched_mod.SchedulerMixin = type("SchedulerMixin", (), {})
    root = types.ModuleType("diffusers")
    sys.modules.update({"diffusers": root, "diffusers.configuration_utils": cfg_mod,
                        "diffusers.schedulers": types.ModuleType("diffusers.schedulers"),
                        "diffusers.schedulers.scheduling_utils": sched_mod})


def test_flow_matching_bitwise():
    ref = _load("pan/flow_matching.py", "ref_flow_matching")
    from pan2_b200.diffusion import flow_matching as ours
    torch.manual_seed(0)
    x0, eps = torch.randn(6, 4, 5), torch.randn(6, 4, 5)
    t = torch.rand(6) * 1000
    assert torch.equal(ours.interpolate(x0, eps, t, dim=0, T=1000), ref.interpolate(x0, eps, t, dim=0, T=1000))
    assert torch.equal(ours.interpolate(x0, eps, t[:5], dim=-1, T=1000), ref.interpolate(x0, eps, t[:5], dim=-1, T=1000))
    for dist in ("uniform", "lognorm"):
        g1, g2 = torch.Generator().manual_seed(3), torch.Generator().manual_seed(3)
        a = ours.draw_timesteps(4096, "cpu", g1, distribution=dist, T=1000, loc=0.2, scale=1.1)
        b = ref.draw_timesteps(4096, "cpu", g2, distribution=dist, T=1000, loc=0.2, scale=1.1)
        assert torch.equal(a, b), dist
    assert torch.equal(ours.shift_timesteps(t, 1000, 5.0), ref.shift_timesteps(t, 1000, 5.0))
    shapes = torch.tensor([[21, 22, 40], [1, 44, 80], [31, 30, 52], [5, 8, 8], [121, 44, 80], [2, 2, 2]])
    for kw in (dict(), dict(rescale_factor=1.0, max_shift=3.0), dict(frame_stride=1, pixel_stride_h=8,
                                                                    pixel_stride_w=16)):
        a = ours.shift_timesteps(t, 1000, mode="dynamic", latent_shapes=shapes, **kw)
        b = ref.shift_timesteps(t, 1000, mode="dynamic", latent_shapes=shapes, **kw)
        assert torch.equal(a, b), kw
    with pytest.raises(ValueError):
        ours.shift_timesteps(t, 1000, mode="dynamic")


def test_rope_bitwise():
    ref = _load("pan/models/transformers/modules/rope.py", "ref_rope")
    from pan2_b200.models import rope as ours
    for axes, grid, theta, scale in (((16, 56, 56), (3, 4, 5), 256.0, 16 / 24), ((8, 12, 12), (2, 3, 7), 10000.0,
                                                                              (0.5, 1.0, 2.0))):
        a = ours.rope_tables_for_grid(axes, grid, theta=theta, position_scale=scale)
        b = ref.rope_tables_for_grid(axes, grid, theta=theta, position_scale=scale)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        pos = torch.randint(0, 50, (37, 3)).float()
        a = ours.rope_tables_for_positions(axes, pos, theta=theta, position_scale=scale)
        b = ref.rope_tables_for_positions(axes, pos, theta=theta, position_scale=scale)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    x = torch.randn(3, 7, 16)
    assert torch.equal(ours.rotate_half(x), ref.rotate_half(x))
    cos, sin = ref.rope_tables_for_grid((16, 56, 56), (2, 3, 4), theta=256.0)
    q, k = torch.randn(24, 4, 128).to(torch.bfloat16), torch.randn(24, 4, 128).to(torch.bfloat16)
    for o, r in zip(ours.apply_rope(q, k, (cos, sin)), ref.apply_rope(q, k, (cos, sin))):
        assert torch.equal(o, r)
    with pytest.raises(ValueError):
        ours.rope_tables_for_grid((16, 56, 56), (2, 3))


def test_layers_and_embeddings_bitwise():
    lay = _load("pan/models/transformers/modules/layers.py", "ref_layers")
    emb = _load("pan/models/transformers/modules/embeddings.py", "ref_embeddings")
    from pan2_b200.models import layers, embeddings
    torch.manual_seed(1)
    x = torch.randn(5, 9, 64).to(torch.bfloat16)
    a, b = layers.RMSNorm(64, eps=1e-5), lay.RMSNorm(64, eps=1e-5)
    with torch.no_grad():
        a.weight.copy_(torch.randn(64))
        b.weight.copy_(a.weight)
    assert torch.equal(a(x), b(x))
    a, b = layers.AdaLNProjection(32, 6, "silu", zero_init=False), lay.AdaLNProjection(32, 6, lay.activation_factory("silu"),
                                                                                       zero_init=False)
    b.load_state_dict(a.state_dict())
    e = torch.randn(3, 32)
    assert torch.equal(a(e), b(e))
    te, tr = embeddings.TimestepEncoder(64, "silu"), emb.TimestepEncoder(64, lay.activation_factory("silu"))
    tr.load_state_dict(te.state_dict())
    t = torch.tensor([0.0, 3.5, 999.0, 517.25])
    assert torch.equal(te(t), tr(t))
    te, tr = te.to(torch.bfloat16), tr.to(torch.bfloat16)
    assert torch.equal(te(t), tr(t))
    pe, pr = embeddings.VideoPatchEmbed((1, 2, 2), 4, 32), emb.VideoPatchEmbed((1, 2, 2), 4, 32)
    pr.load_state_dict(pe.state_dict())
    dense = torch.randn(2, 4, 3, 6, 8)
    assert torch.equal(pe(dense), pr(dense))
    packed = torch.randn(16, 20, 1, 1)
    assert torch.equal(pe(packed, packed=True), pr(packed, packed=True))


def test_scheduler_and_timestep_schedule_bitwise():
    _diffusers_stand_in()
    ref = _load("pan/schedulers/scheduling_flow_match_discrete.py", "ref_sched")
    ref_sched = _load("pan/schedulers/timestep_schedule.py", "ref_tsched")
    from pan2_b200.inference.scheduler import FlowEulerScheduler, apply_timestep_schedule
    for shift, name in ((1.0, "standard"), (5.0, "standard"), (5.0, "early_refine_2x"), (12.0, "early_refine_2x")):
        a, b = FlowEulerScheduler(1000, shift), ref.FlowEulerScheduler(num_train_timesteps=1000, shift=shift)
        a.set_timesteps(50)
        b.set_timesteps(50)
        ta, tb = apply_timestep_schedule(a, name), ref_sched.apply_timestep_schedule(b, name)
        assert torch.equal(ta, tb) and torch.equal(a.sigmas, b.sigmas)
        x = torch.randn(3, 8)
        xa, xb = x.clone(), x.clone()
        for t in ta[:5]:
            v = torch.randn(3, 8).to(torch.bfloat16)
            xa, xb = a.step(v, t, xa), b.step(v, t, xb)
        assert torch.equal(xa, xb)


def test_guidance_bitwise_and_same_rejections():
    ref = _load("pan/utils/inference_guidance.py", "ref_guidance")
    from pan2_b200.inference import guidance as ours
    torch.manual_seed(2)
    neg, pos, weak = (torch.randn(4, 16).to(torch.bfloat16) for _ in range(3))
    plans = [dict(), dict(start_step=2, end_step=8, skip_interval=(4, 6)), dict(start_step=3, warmup_scale=2.5),
             dict(stg_scale=0.7, end_step=9), dict(start_step=1, end_step=5, warmup_scale=1.5, stg_scale=0.3)]
    for kw in plans:
        pa, pb = ours.resolve_guidance_plan(10, **kw), ref.resolve_guidance_plan(10, **kw)
        for i in range(10):
            assert pa.active(i) == pb.active(i), (kw, i)
            a = ours.apply_guidance(neg, pos, 4.5, step_index=i, plan=pa, weak_predict_fn=lambda: weak)
            b = ref.apply_guidance(neg, pos, 4.5, step_index=i, plan=pb, weak_predict_fn=lambda: weak)
            assert torch.equal(a, b), (kw, i)
    bad = [dict(start_step=5, end_step=5), dict(skip_interval=(3, 2)), dict(warmup_scale=0.5), dict(stg_scale=-1.0),
           dict(end_step=11), dict(start_step=True), dict(skip_interval=(1.0, 2))]
    for kw in bad:
        for mod in (ours, ref):
            with pytest.raises(ValueError):
                mod.resolve_guidance_plan(10, **kw)
    for mod in (ours, ref):
        with pytest.raises(ValueError):
            mod.validate_sampling_extensions(30, "early_refine_2x")
        with pytest.raises(ValueError):
            mod.apply_guidance(neg, pos, 1.0, step_index=0, plan=mod.resolve_guidance_plan(10))


def test_prompt_inputs_match(tmp_path):
    ref = _load("inference/inputs.py", "ref_inputs")
    from pan2_b200.inference import inputs as ours
    for entry, fps, fb in (({"duration_sec": 5}, 24, 121), ({"duration_sec": 5.1}, 24, 121), ({"duration_sec": "2.5"},
                           30, 121), ({"frames": 33}, 24, 121), ({}, 24, 241), ({"num_target_frames": 17}, 16, 9)):
        assert ours.resolve_frames(entry, fps, fb) == ref.resolve_frames(entry, fps, fb)
    for bad in ({"duration_sec": 0}, {"duration_sec": "nan"}, {"frames": 2.5}, {"duration_sec": True}):
        for mod in (ours, ref):
            with pytest.raises(ValueError):
                mod.resolve_frames(bad)
    neg = json.dumps({"a": {"time_range_sec": "0 to 10"}, "b": [{"time_range_sec": "x"}, 3]})
    assert ours.render_negative_duration(neg, 121, 24) == ref.render_negative_duration(neg, 121, 24)
    assert ours.render_negative_duration("plain words", 121) == ref.render_negative_duration("plain words", 121)
    img = tmp_path / "ref.png"
    img.write_bytes(b"png")
    entries = [{"id": "a 1", "prompt": "p1", "duration_sec": 5}, {"prompt": "p2", "refined_prompt": "p2r"},
               {"type": "i2v", "image": str(img), "caption": "c", "neg_prompt": "n"},
               {"relative_path": "sub/x.mp4", "prompt": "p3", "frames": 9}]
    pf = tmp_path / "prompts.json"
    pf.write_text(json.dumps({"entries": entries}))
    for task in ("t2v", "i2v", "auto"):
        for shard in range(2):
            kw = dict(task=task, shard_index=shard, shard_count=2, default_negative=neg)
            a = ours.load_inference_inputs(pf, tmp_path / "out", **kw)
            b = ref.load_inference_inputs(pf, tmp_path / "out", **kw)
            assert a == b, (task, shard)
    pf.write_text(json.dumps([{"prompt": "p", "relative_path": "../x.mp4"}]))
    for mod in (ours, ref):
        with pytest.raises(ValueError):
            mod.load_inference_inputs(pf, tmp_path / "out")
