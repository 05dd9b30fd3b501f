"""Caption codec logic (chat template, prefix crop, truncation, padding) with an injected
character-level tokenizer and a toy language model: the Qwen weights are not needed to check which
token rows reach the DiT."""
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
