"""Generation on the B200: the packed CFG runner (sm_100a kernels) against the dense masked forward,
and a short image-to-video sampling run through the public pipeline."""
import pytest
import torch

from tiny import TINY_ARCH

pytestmark = pytest.mark.gpu

ARCH = dict(TINY_ARCH, hidden_size=512, num_attention_heads=4, rope_axes_dim=(32, 48, 48), text_embed_dim=128)


def test_packed_cfg_gpu_matches_dense():
    from pan2_b200.pipelines.video import PackedDiTRunner, build_inference_model
    from pan2_b200.data.patching import patchify, unpatchify
    from pan2_b200.ops._ext import ext
    m = build_inference_model(ARCH, "cuda", dtype=torch.bfloat16, seed=1)
    grid = (5, 16, 16)
    N = 5 * 8 * 8
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, N, 192, generator=g).cuda()
    cond = torch.randn(1, N, 196, generator=g).cuda()
    lens = [40, 77]
    text = [torch.randn(n, 128, generator=g).cuda().bfloat16() for n in lens]
    t = torch.tensor([600.0, 600.0], device="cuda")
    runner = PackedDiTRunner(m, "cuda")
    v = runner.predict(runner.plan(grid, lens), x.repeat(2, 1, 1), cond.repeat(2, 1, 1), t, torch.cat(text))
    L = max(lens)
    tpad = torch.zeros(2, L, 128, device="cuda", dtype=torch.bfloat16)
    mask = torch.zeros(2, L, dtype=torch.long, device="cuda")
    for i, tt in enumerate(text):
        tpad[i, :lens[i]] = tt
        mask[i, :lens[i]] = 1
    lat = unpatchify(torch.cat([x, cond], -1)[0], (5, 8, 8), (1, 2, 2), 97).unsqueeze(0).repeat(2, 1, 1, 1, 1)
    with torch.no_grad():
        vd, _ = m.forward_dense(lat.bfloat16(), t, tpad, mask)
    vd_tok = torch.stack([patchify(vd[i], (1, 2, 2)).t() for i in range(2)]).float()
    torch.cuda.synchronize()
    assert ext().error_flag(True) == 0
    cos = torch.nn.functional.cosine_similarity(v.float().flatten(), vd_tok.flatten(), dim=0).item()
    assert cos > 0.995, cos


def test_pipeline_i2v_cfg_runs():
    from pan2_b200.pipelines.video import PanVideoPipeline, build_inference_model
    from pan2_b200.ops._ext import ext
    m = build_inference_model(ARCH, "cuda", dtype=torch.bfloat16, seed=1)
    pipe = PanVideoPipeline(m, device="cuda")
    g = torch.Generator().manual_seed(3)
    out = pipe(prompt_embeds=[torch.randn(33, 128, generator=g)], negative_prompt_embeds=[torch.randn(9, 128, generator=g)],
               reference_latents=torch.randn(48, 1, 16, 16, generator=g), video_length=17, video_height=256,
               video_width=256, num_inference_steps=4, seed=7, output_type="latent", time_steps=True,
               timestep_schedule="standard", cfg_skip_interval=(1, 2))
    torch.cuda.synchronize()
    assert ext().error_flag(True) == 0
    assert out.latents.shape == (1, 48, 5, 16, 16)
    assert torch.isfinite(out.latents).all()
    assert len(out.step_ms) == 4


@pytest.mark.parametrize("prefetch", [True, False], ids=["prefetch", "no_prefetch"])
def test_block_streaming_offload_matches_resident_weights(prefetch):
    """Generation with the DiT's blocks streamed from host memory through two device slots (the next
    block copied on a side stream while the current one runs) gives the same latents as the model
    kept on the GPU."""
    from pan2_b200.pipelines.video import PanVideoPipeline, build_inference_model
    from pan2_b200.ops._ext import ext
    g = torch.Generator().manual_seed(5)
    kw = dict(prompt_embeds=[torch.randn(33, 128, generator=g)], negative_prompt_embeds=[torch.randn(9, 128, generator=g)],
              video_length=17, video_height=256, video_width=256, num_inference_steps=3, seed=7,
              output_type="latent")
    outs = []
    for mode in (None, "blocks"):
        m = build_inference_model(ARCH, "cuda", dtype=torch.bfloat16, seed=1)
        pipe = PanVideoPipeline(m, device="cuda")
        if mode is not None:
            pipe.configure_runtime(offload=mode, prefetch=prefetch)
        outs.append(pipe(**kw).latents.float().cpu())
        torch.cuda.synchronize()
        del pipe, m
        torch.cuda.empty_cache()
    assert ext().error_flag(True) == 0
    assert torch.equal(outs[0], outs[1])
