"""Tiny MMDiT on the B200 (sm_100a kernels, bf16) against the same model on CPU in fp32."""
import pytest
import torch

from tiny import tiny_model, tiny_batch

pytestmark = pytest.mark.gpu

GPU_ARCH = dict(hidden_size=512, num_attention_heads=4, rope_axes_dim=(32, 48, 48))


def _to(batch, device, dtype):
    out = {}
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            out[k] = v.to(device, dtype) if v.is_floating_point() and k != "timestep" else v.to(device)
        elif k == "packed_seq_params":
            out[k] = v.to(device)
        else:
            out[k] = v
    return out


def test_tiny_model_packed_gpu_matches_cpu():
    from pan2_b200.ops._ext import ext
    model = tiny_model(**GPU_ARCH)
    batch, _ = tiny_batch(model)
    loss_cpu = model(**batch)
    loss_cpu.backward()
    g_cpu = {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}
    model.zero_grad()
    model = model.cuda()
    loss_gpu = model(**_to(batch, "cuda", torch.bfloat16))
    loss_gpu.backward()
    torch.cuda.synchronize()
    assert ext().error_flag(True) == 0
    rel = abs(loss_gpu.item() - loss_cpu.item()) / abs(loss_cpu.item())
    assert rel < 2e-2, (loss_gpu.item(), loss_cpu.item())
    worst = []
    no_grad = [k for k, p in model.named_parameters() if k in g_cpu and p.grad is None]
    assert not no_grad, no_grad
    for k, p in model.named_parameters():
        if k not in g_cpu:
            continue
        a, b = p.grad.float().cpu(), g_cpu[k]
        if b.abs().max() == 0:  # e.g. the last block's text FFN: no path to the video loss
            assert a.abs().max() == 0, k
            continue
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
        worst.append((cos, k))
    worst.sort()
    assert worst[0][0] > 0.98, worst[:5]


def test_tiny_model_dense_gpu_matches_cpu():
    model = tiny_model(**GPU_ARCH).eval()
    _, dense = tiny_batch(model)
    with torch.no_grad():
        v_cpu, _ = model.forward_dense(dense["latents"][:1], dense["timestep"][:1], dense["text"][:1])
        m = model.cuda()
        v_gpu, _ = m.forward_dense(dense["latents"][:1].cuda().bfloat16(), dense["timestep"][:1].cuda(),
                                   dense["text"][:1].cuda().bfloat16())
    cos = torch.nn.functional.cosine_similarity(v_gpu.float().cpu().flatten(), v_cpu.flatten(), dim=0).item()
    assert cos > 0.99, cos
