"""CPU fp32 checks of the model: packed training path == dense (reference) path per sample."""
import torch
import pytest

from tiny import tiny_model, tiny_batch


def test_packed_matches_dense_loss():
    model = tiny_model()
    batch, dense = tiny_batch(model)
    loss = model(**batch)
    # dense path: one sample at a time, velocity vs target, mean over all video elements
    sq, n = 0.0, 0
    for i in range(dense["latents"].shape[0]):
        v, _ = model.forward_dense(dense["latents"][i:i + 1], dense["timestep"][i:i + 1], dense["text"][i:i + 1])
        d = v[0] - dense["target"][i]
        sq += d.pow(2).sum().item()
        n += d.numel()
    assert torch.allclose(loss, torch.tensor(sq / n), rtol=1e-4, atol=1e-5), (loss.item(), sq / n)


def test_packed_grads_match_dense_grads():
    model = tiny_model()
    batch, dense = tiny_batch(model)
    loss = model(**batch)
    loss.backward()
    g_packed = {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}
    model.zero_grad()
    total = 0.0
    n = 0
    outs = []
    for i in range(dense["latents"].shape[0]):
        v, _ = model.forward_dense(dense["latents"][i:i + 1], dense["timestep"][i:i + 1], dense["text"][i:i + 1])
        d = v[0] - dense["target"][i]
        outs.append(d.pow(2).sum())
        n += d.numel()
    (sum(outs) / n).backward()
    g_dense = {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}
    assert set(g_packed) == set(g_dense) - {"timestep_encoder.freqs"}
    for k in g_packed:
        a, b = g_packed[k], g_dense[k]
        err = (a - b).abs().max().item() / (b.abs().max().item() + 1e-12)
        assert err < 2e-3, (k, err)


def test_state_dict_names_match_reference_layout():
    model = tiny_model()
    sd = model.state_dict()
    h = 256
    assert sd["blocks.0.qkv_proj.weight"].shape == (6 * h, h)
    assert sd["blocks.0.qkv_proj.q_weight"].shape == (2 * 64,)
    assert sd["blocks.0.out_proj.weight"].shape == (2 * h, h)
    assert sd["blocks.0.modulation.linear.weight"].shape == (6 * h, h)
    assert sd["blocks.0.text_modulation"].shape == (6 * h,)
    assert sd["blocks.0.ffn.w_up_video"].shape == (8 * h, h)
    assert sd["blocks.0.ffn.w_down_text"].shape == (h, 4 * h)
    assert sd["patch_embed.proj.weight"].shape == (h, 97, 1, 2, 2)
    assert sd["output_head.proj.weight"].shape == (192, h)
    assert sd["output_head.modulation.linear.weight"].shape == (2 * h, h)
    assert sd["text_type_embedding.weight"].shape == (3, h)
    assert sd["caption_encoder.blocks.3.ffn.w2.weight"].shape == (h, 4 * h)
    assert sd["timestep_encoder.freqs"].shape == (128,)
    assert sd["cap_embedder.0.weight"].shape == (4096,)


def test_legacy_block_keys_load():
    model = tiny_model(num_layers=1)
    sd = model.state_dict()
    legacy = {}
    h3 = 3 * 256
    for k, v in sd.items():
        if k == "blocks.0.qkv_proj.weight":
            legacy["blocks.0.linear1_qkv.weight"], legacy["blocks.0.text_linear1_qkv.weight"] = v[:h3], v[h3:]
        elif k == "blocks.0.qkv_proj.bias":
            legacy["blocks.0.linear1_qkv.bias"], legacy["blocks.0.text_linear1_qkv.bias"] = v[:h3], v[h3:]
        else:
            legacy[k] = v
    m2 = tiny_model(num_layers=1, seed=5)
    m2.load_state_dict(legacy)
    assert torch.equal(m2.state_dict()["blocks.0.qkv_proj.weight"], sd["blocks.0.qkv_proj.weight"])


def test_timestep_freqs_stay_exact_fp32():
    from pan2_b200.models.embeddings import sinusoid_frequencies, timestep_embedding
    exact = sinusoid_frequencies(256, 10000.0)
    model = tiny_model(num_layers=1).to(torch.bfloat16)
    sd = model.state_dict()
    assert sd["timestep_encoder.freqs"].dtype == torch.float32 and torch.equal(sd["timestep_encoder.freqs"], exact)
    enc = model.timestep_encoder
    t = torch.tensor([0.0, 17.0, 999.0])
    want = enc.out_proj(enc.act(enc.in_proj(timestep_embedding(t, exact).to(torch.bfloat16))))
    assert torch.equal(enc(t), want)
    sd["timestep_encoder.freqs"] = sd["timestep_encoder.freqs"].to(torch.bfloat16).float()  # a lossy copy
    model.load_state_dict(sd)
    assert torch.equal(model.state_dict()["timestep_encoder.freqs"], exact)
