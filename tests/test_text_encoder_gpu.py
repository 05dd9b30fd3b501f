"""Packed Qwen3.5 caption encoding on a B200 (tiny random model, tame weights).

fp32 on CUDA: the packed encode equals each caption encoded alone by the Hugging Face model on the
CPU.  bf16 on CUDA: the packed encode is held to the Hugging Face bf16 forward's own distance from
that fp32 reference."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu
pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")


@pytest.fixture
def exact_fp32():
    """fp32 on CUDA without TF32 (cuDNN convolutions default to it)."""
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def test_packed_forward_matches_each_caption_alone_on_cuda(exact_fp32):
    from test_text_encoder_cpu import LENGTHS, tiny_qwen
    from pan2_b200.models.qwen_packed import PackedQwenForward
    m_cpu = tiny_qwen(3, noise=0.02)
    m32 = copy.deepcopy(m_cpu).cuda()
    m16 = copy.deepcopy(m_cpu).cuda().to(torch.bfloat16)
    torch.manual_seed(0)
    ids = [torch.randint(0, 512, (n,)) for n in LENGTHS]
    flat = torch.cat(ids).cuda()
    p32 = PackedQwenForward(m32)(flat, LENGTHS).float().cpu()
    p16 = PackedQwenForward(m16)(flat, LENGTHS).float().cpu()
    a = 0
    for n, i in zip(LENGTHS, ids):
        with torch.no_grad():
            ref = m_cpu(input_ids=i[None], use_cache=False).last_hidden_state[0]
            r16 = m16(input_ids=i[None].cuda(), use_cache=False).last_hidden_state[0].float().cpu()
            r32 = m32(input_ids=i[None].cuda(), use_cache=False).last_hidden_state[0].cpu()
        scale = ref.abs().max().item()
        err32 = (p32[a:a + n] - ref).abs().max().item()
        assert err32 < 2e-3 * scale, (n, err32, "Hugging Face fp32 on CUDA vs CPU:", (r32 - ref).abs().max().item())
        err_packed = (p16[a:a + n] - ref).abs().max().item()
        err_hf = (r16 - ref).abs().max().item()
        assert err_packed <= 1.5 * err_hf + 1e-2 * scale, (n, err_packed, err_hf)
        a += n
