"""Caption codec logic and the packed Qwen3.5 encode.

* chat template, prefix crop, truncation and padding, with an injected character-level tokenizer and
  a toy language model (the Qwen weights are not needed to check which token rows reach the DiT);
* with a tiny random Qwen3.5 from transformers: the gated delta rule over a packed,
  caption-restarted chunk grid equals the token-by-token recurrence of its definition; the packed
  forward of several captions equals the Hugging Face model run on each caption alone (captions
  shorter than, equal to and longer than one 64-token chunk); ``embed`` / ``encode`` agree on the
  packed and the right-padded paths.
"""
import pytest
import torch
import torch.nn as nn

from pan2_b200.models.text_encoder import SYSTEM_PROMPT, USER_HEADER, QwenCaptionCodec, chat_for


class CharTokenizer:
    pad_token_id = 0
    eos_token_id = 1

    @staticmethod
    def _enc(text):
        return [2 + (ord(c) % 500) for c in text]

    def __call__(self, text, add_special_tokens=False):
        return {"input_ids": self._enc(text)}

    def apply_chat_template(self, chat, add_generation_prompt=True, tokenize=True, return_dict=True,
                            truncation=False, max_length=None, return_tensors="pt"):
        text = "".join(f"<|im_start|>{m['role']}\n{m['content']}<|im_end|>\n" for m in chat)
        if add_generation_prompt:
            text += "<|im_start|>assistant\n"
        ids = self._enc(text)
        if truncation and max_length is not None:
            ids = ids[:max_length]
        return {"input_ids": torch.tensor([ids])}


class Out:
    def __init__(self, h):
        self.last_hidden_state = h


class ToyLM(nn.Module):
    """Hidden state of a token = its id in every channel (so rows identify their tokens)."""

    def __init__(self, dim=8):
        super().__init__()
        self.w = nn.Parameter(torch.ones(dim))
        self.config = type("C", (), {"hidden_size": dim})()

    def forward(self, input_ids, attention_mask=None, use_cache=False):
        return Out(input_ids[..., None].float() * self.w)


def test_prefix_crop_truncation_and_padding():
    tok = CharTokenizer()
    codec = QwenCaptionCodec(tokenizer=tok, model=ToyLM(), max_caption_tokens=40)
    templ = f"<|im_start|>system\n{SYSTEM_PROMPT}<|im_end|>\n{USER_HEADER}"
    assert codec.prefix_len == len(templ)
    assert chat_for("")[1]["content"] == " "  # an empty caption becomes one space
    short = codec.tokenize("a red fox", 100)
    assert short.prefix_len == codec.prefix_len
    assert short.cropped_length == short.full_length - short.prefix_len
    long = codec.tokenize("x" * 200, 100)
    assert long.cropped_length == 40  # capped by max_caption_tokens
    emb = codec.embed([short, long], "cpu")
    assert emb.shape == (short.cropped_length + long.cropped_length, 8)
    # the first kept row is the first caption character, not a template token
    assert emb[0, 0].item() == 2 + ord("a")
    assert emb[short.cropped_length, 0].item() == 2 + ord("x")
    e, m = codec.encode(["a red fox", "x" * 200])
    assert e.shape[0] == 2 and m[0].sum().item() == short.cropped_length and m[1].sum().item() == 40


def _qwen_modules():
    transformers = pytest.importorskip("transformers")
    mq = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
    return transformers, mq


LENGTHS = [5, 70, 130, 1, 64, 3]


def tiny_qwen(seed=0, noise=0.2):
    """A 4-layer Qwen3.5 (3:1 linear / full attention like the 9B) with random weights; ``noise``
    scales the perturbation (0.2 makes rounding grow fast through the layers, 0.02 keeps it tame)."""
    transformers, mq = _qwen_modules()
    torch.manual_seed(seed)
    cfg = transformers.Qwen3_5TextConfig(
        vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=4, num_attention_heads=4,
        num_key_value_heads=2, head_dim=16, linear_num_value_heads=4, linear_num_key_heads=2,
        linear_key_head_dim=16, linear_value_head_dim=8, linear_conv_kernel_dim=4,
        layer_types=["linear_attention", "full_attention", "linear_attention", "full_attention"])
    cfg._attn_implementation = "sdpa"
    m = mq.Qwen3_5TextModel(cfg).eval()
    # the reference runs Hugging Face's own PyTorch implementations: where flash-linear-attention
    # is importable (a GPU machine), its Triton gated norm and delta-rule kernels would replace them
    for layer in m.layers:
        la = getattr(layer, "linear_attn", None)
        if la is None:
            continue
        norm = mq.Qwen3_5RMSNormGated(la.head_v_dim, eps=la.layer_norm_epsilon)
        with torch.no_grad():
            norm.weight.copy_(la.norm.weight.detach().cpu())
        la.norm = norm
        la.chunk_gated_delta_rule = mq.torch_chunk_gated_delta_rule
        la.causal_conv1d_fn = None
    with torch.no_grad():
        for p in m.parameters():
            p.add_(torch.randn_like(p) * noise)
    return m


def _recurrence(q, k, v, beta, g):
    """Token-by-token gated delta rule of one caption: q, k [T, H, dk], v [T, H, dv], beta, g [T, H]."""
    T, H, dk = q.shape
    q = torch.nn.functional.normalize(q, dim=-1, eps=1e-3) * dk ** -0.5
    k = torch.nn.functional.normalize(k, dim=-1, eps=1e-3)
    S = torch.zeros(H, dk, v.shape[-1], dtype=torch.float64)
    out = []
    for t in range(T):
        S = S * torch.exp(g[t]).view(H, 1, 1)
        pred = torch.einsum("hk,hkv->hv", k[t], S)
        S = S + torch.einsum("hk,hv->hkv", k[t], beta[t].view(H, 1) * (v[t] - pred))
        out.append(torch.einsum("hk,hkv->hv", q[t], S))
    return torch.stack(out)


def test_chunked_delta_rule_equals_the_recurrence():
    from pan2_b200.models.qwen_packed import _layout, gated_delta_rule_packed
    torch.manual_seed(1)
    lens = [3, 64, 65, 150]
    T, H, dk, dv = sum(lens), 3, 8, 5
    q, k = torch.randn(T, H, dk, dtype=torch.float64), torch.randn(T, H, dk, dtype=torch.float64)
    v = torch.randn(T, H, dv, dtype=torch.float64)
    beta = torch.rand(T, H, dtype=torch.float64)
    g = -torch.rand(T, H, dtype=torch.float64) * 0.3
    got = gated_delta_rule_packed(q, k, v, beta, g, _layout(lens, 64, "cpu"))
    a = 0
    for n in lens:
        ref = _recurrence(q[a:a + n], k[a:a + n], v[a:a + n], beta[a:a + n], g[a:a + n])
        assert (got[a:a + n].double() - ref).abs().max() < 1e-4 * ref.abs().max(), n
        a += n


def test_packed_forward_equals_each_caption_alone():
    from pan2_b200.models.qwen_packed import PackedQwenForward
    m = tiny_qwen()
    ids = [torch.randint(0, 512, (n,)) for n in LENGTHS]
    packed = PackedQwenForward(m)(torch.cat(ids), LENGTHS)
    a = 0
    for n, i in zip(LENGTHS, ids):
        with torch.no_grad():
            ref = m(input_ids=i[None], use_cache=False).last_hidden_state[0]
        assert (packed[a:a + n] - ref).abs().max() < 1e-4 * ref.abs().max(), n
        a += n


def test_codec_packed_and_padded_paths_agree():
    m = tiny_qwen(2)
    codec = QwenCaptionCodec(model=m, tokenizer=CharTokenizer(), max_caption_tokens=90, embed_dim=64)
    assert codec._packed is not None
    texts = ["a red fox", "", "the camera pans slowly over a wide river valley at dawn, mist rising " * 2, "x"]
    caps = [codec.tokenize(t, 90) for t in texts]
    rows = codec.embed(caps, "cpu")
    assert rows.shape == (sum(c.cropped_length for c in caps), 64)
    a = 0
    for c in caps:
        with torch.no_grad():
            ref = m(input_ids=c.token_ids[None], use_cache=False).last_hidden_state[0, c.prefix_len:]
        assert (rows[a:a + c.cropped_length] - ref).abs().max() < 1e-4 * ref.abs().max()
        a += c.cropped_length
    emb, mask = codec.encode(texts, device="cpu")
    codec._packed = None
    emb_pad, mask_pad = codec.encode(texts, device="cpu")
    assert torch.equal(mask, mask_pad)
    assert (emb - emb_pad).abs().max() < 1e-4 * emb_pad.abs().max()
