"""Checkpoint conversion native <-> diffusers: key layout and an exact round trip."""
import json
import os

import torch

from tiny import TINY_ARCH, tiny_model


def test_round_trip_and_layout(tmp_path):
    from safetensors.torch import save_file
    from pan2_b200.checkpoint.convert import convert_to_diffusers, convert_to_native
    from pan2_b200.checkpoint.io import LazyStateDict
    m = tiny_model(seed=3)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    sd["text_type_embedding.weight"][1:] = 0  # only row 0 is carried by the diffusers layout
    src = tmp_path / "native.safetensors"
    save_file({k: v.contiguous() for k, v in sd.items()}, str(src))
    arch = dict(TINY_ARCH)
    dif = tmp_path / "diffusers"
    convert_to_diffusers(str(src), str(dif), arch)
    cfg = json.loads((dif / "config.json").read_text())
    assert cfg["num_layers"] == 2 and cfg["attention_head_dim"] == 64
    d = LazyStateDict(str(dif / "diffusion_pytorch_model.safetensors.index.json"))
    keys = set(d.keys())
    assert "transformer_blocks.1.attn.add_v_proj.bias" in keys and "context_refiner.3.ff.net.0.proj.weight" in keys
    assert "timestep_encoder.freqs" not in keys and "context_type_embedding" in keys
    h = TINY_ARCH["hidden_size"]
    assert tuple(d.get("transformer_blocks.0.attn.to_q.weight").shape) == (h, h)
    # [w3; w1] packing and [scale; shift] head modulation
    w1 = sd["caption_encoder.blocks.0.ffn.w1.weight"]
    assert torch.equal(d.get("context_refiner.0.ff.net.0.proj.weight")[w1.shape[0]:], w1)
    shift = sd["output_head.modulation.linear.bias"][:h]
    assert torch.equal(d.get("norm_out.linear.bias")[h:], shift)
    back = tmp_path / "back"
    convert_to_native(str(dif), str(back))
    r = LazyStateDict(str(back))
    assert set(r.keys()) == set(sd.keys())
    for k, v in sd.items():
        assert torch.equal(r.get(k).to(v.dtype), v), k
    m2 = tiny_model(seed=9)
    m2.load_state_dict({k: r.get(k) for k in r.keys()})


def test_reference_style_dcp_checkpoint_loads(tmp_path):
    """A torch distributed checkpoint with ``model.``-prefixed keys (the reference trainer's
    ``checkpoint-N/transformer``) loads into the model by name, tensor by tensor."""
    import torch.distributed.checkpoint as dcp
    from pan2_b200.checkpoint.io import LazyStateDict
    from pan2_b200.pipelines.video import load_transformer_weights
    from tiny import tiny_model
    src = tiny_model(seed=3)
    ck = tmp_path / "checkpoint-7" / "transformer"
    sd = {"model." + k: v.clone() for k, v in src.state_dict().items()}
    dcp.save(sd, storage_writer=dcp.FileSystemWriter(str(ck)), no_dist=True)
    lazy = LazyStateDict(str(tmp_path / "checkpoint-7"))
    assert set(lazy.keys()) == set(src.state_dict())
    dst = tiny_model(seed=4)
    load_transformer_weights(dst, str(ck))
    for k, v in src.state_dict().items():
        if k.endswith("freqs"):
            continue
        assert torch.equal(dst.state_dict()[k], v), k
