"""Packed Qwen3.5 caption encoding on a B200 (bf16, tiny random model): equal to each caption
encoded alone by the Hugging Face model, within bf16 rounding."""
import pytest
import torch

pytestmark = pytest.mark.gpu
pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")


def test_packed_bf16_forward_matches_each_caption_alone():
    from test_text_encoder_cpu import LENGTHS, tiny_qwen
    from pan2_b200.models.qwen_packed import PackedQwenForward
    m = tiny_qwen(3).to("cuda", torch.bfloat16)
    ids = [torch.randint(0, 512, (n,)) for n in LENGTHS]
    packed = PackedQwenForward(m)(torch.cat(ids).cuda(), LENGTHS).float()
    a = 0
    for n, i in zip(LENGTHS, ids):
        with torch.no_grad():
            ref = m(input_ids=i[None].cuda(), use_cache=False).last_hidden_state[0].float()
        err = (packed[a:a + n] - ref).abs().max().item()
        assert err < 5e-2 * ref.abs().max().item(), (n, err)
        a += n
