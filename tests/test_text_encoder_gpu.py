"""Packed Qwen3.5 caption encoding on a B200 (tiny random model).

fp32: the packed encode equals each caption encoded alone by the Hugging Face model.  bf16: the
random toy model amplifies rounding (the Hugging Face bf16 forward itself moves far from fp32), so
the packed bf16 encode is held to the Hugging Face bf16 forward's own distance from fp32."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu
pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")


@pytest.fixture
def exact_fp32():
    """fp32 references without TF32 (cuDNN convolutions default to it)."""
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def test_packed_forward_matches_each_caption_alone_on_cuda(exact_fp32):
    from test_text_encoder_cpu import LENGTHS, tiny_qwen
    from pan2_b200.models.qwen_packed import PackedQwenForward
    m32 = tiny_qwen(3).cuda()
    m16 = copy.deepcopy(m32).to(torch.bfloat16)
    torch.manual_seed(0)
    ids = [torch.randint(0, 512, (n,)) for n in LENGTHS]
    flat = torch.cat(ids).cuda()
    p32 = PackedQwenForward(m32)(flat, LENGTHS).float()
    p16 = PackedQwenForward(m16)(flat, LENGTHS).float()
    a = 0
    for n, i in zip(LENGTHS, ids):
        with torch.no_grad():
            r32 = m32(input_ids=i[None].cuda(), use_cache=False).last_hidden_state[0].float()
            r16 = m16(input_ids=i[None].cuda(), use_cache=False).last_hidden_state[0].float()
        scale = r32.abs().max().item()
        assert (p32[a:a + n] - r32).abs().max().item() < 1e-3 * scale, n
        err_packed = (p16[a:a + n] - r32).abs().max().item()
        err_hf = (r16 - r32).abs().max().item()
        assert err_packed <= 1.5 * err_hf + 1e-2 * scale, (n, err_packed, err_hf)
        a += n
