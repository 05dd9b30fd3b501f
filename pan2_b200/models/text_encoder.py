"""Qwen3.5 caption encoder shared by training and generation.

Same recipe as the reference (pan/models/text_encoders/__init__.py:33-276): the frozen Qwen3.5-9B
language model with its last ``hidden_state_skip_layer`` decoder layers dropped and the final norm
replaced by identity (so the features are the raw output of layer ``L - skip``); the vision tower and
LM head are discarded.  Every caption is wrapped in the video chat template (a fixed system turn, the
caption as the user turn, the assistant turn opened); Qwen encodes the whole templated prompt and
only the rows after the user-turn header (``prefix_len`` tokens, measured once from the tokenizer)
reach the DiT.  An empty caption becomes one space, so the user turn is never empty.

A batch of captions is encoded as ONE packed sequence (:class:`~pan2_b200.models.qwen_packed.
PackedQwenForward`: per-caption positions, causal attention within each caption, the GatedDeltaNet
convolution and recurrence restarted at every caption start), so no GEMM of the 9B encoder spends
work on padding rows -- the reference's packed encode (``dataset/packed_dataloader.py:225-244``).
A model without Qwen3.5's layer structure falls back to a right-padded batch with an attention mask.

The model and tokenizer come from a Hugging Face id or a local folder (``transformers``); they can
also be injected (tests, other checkpoints).  :class:`QwenCaptionCodec` is the training loader's
interface (:class:`~pan2_b200.data.items.CaptionCodec`) and also serves generation through
:meth:`QwenCaptionCodec.encode`.
"""
from __future__ import annotations

import os
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn

from ..data.items import Caption, CaptionCodec
from .qwen_packed import PackedQwenForward

DEFAULT_TEXT_ENCODER = "Qwen/Qwen3.5-9B"
SYSTEM_PROMPT = "You are a helpful assistant. Generate the video with the following instructions."
USER_HEADER = "<|im_start|>user\n"

os.environ.setdefault("TOKENIZERS_PARALLELISM", "false")


def chat_for(caption: str):
    return [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": caption or " "}]


def load_qwen_language_model(path: str = DEFAULT_TEXT_ENCODER, hidden_state_skip_layer: int = 2, device="cuda",
                             dtype=torch.bfloat16, attn_implementation: str = "sdpa") -> nn.Module:
    from transformers import AutoConfig, AutoModelForImageTextToText
    skip = int(hidden_state_skip_layer)
    if skip < 0:
        raise ValueError(f"cannot drop a negative number of decoder layers ({skip})")
    cfg = AutoConfig.from_pretrained(path)
    tcfg = getattr(cfg, "text_config", cfg)
    if skip >= tcfg.num_hidden_layers:
        raise ValueError(f"hidden_state_skip_layer={skip} must be below num_hidden_layers={tcfg.num_hidden_layers}")
    tcfg.num_hidden_layers -= skip
    if getattr(tcfg, "layer_types", None):
        tcfg.layer_types = list(tcfg.layer_types)[:tcfg.num_hidden_layers]
    full = AutoModelForImageTextToText.from_pretrained(path, config=cfg, dtype=dtype, device_map=str(device),
                                                       attn_implementation=attn_implementation)
    lm = full.model.language_model
    for attr in ("visual",):
        if hasattr(full.model, attr):
            delattr(full.model, attr)
    if hasattr(full, "lm_head"):
        del full.lm_head
    lm.norm = nn.Identity()
    lm.requires_grad_(False)
    return lm.eval()


class QwenCaptionCodec(CaptionCodec):
    def __init__(self, path: str = DEFAULT_TEXT_ENCODER, *, device="cuda", hidden_state_skip_layer: int = 2,
                 max_caption_tokens: int = 1000, model: Optional[nn.Module] = None, tokenizer=None,
                 embed_dim: Optional[int] = None):
        if tokenizer is None:
            from transformers import AutoTokenizer
            tokenizer = AutoTokenizer.from_pretrained(path, padding_side="right")
        self.tokenizer = tokenizer
        self.model = model if model is not None else load_qwen_language_model(path, hidden_state_skip_layer, device)
        self.max_caption_tokens = int(max_caption_tokens)
        self._prefix: Optional[int] = None
        self.embed_dim = embed_dim or int(getattr(getattr(self.model, "config", None), "hidden_size", 4096))
        self._packed = PackedQwenForward(self.model) if PackedQwenForward.supports(self.model) else None

    def to(self, device) -> "QwenCaptionCodec":
        """Move the language model (generation offloading parks it on the CPU between prompts)."""
        self.model.to(device)
        return self

    # ---- tokens
    def _ids(self, caption: str, max_length: Optional[int]) -> torch.Tensor:
        out = self.tokenizer.apply_chat_template(chat_for(caption), add_generation_prompt=True, tokenize=True,
                                                 return_dict=True, truncation=max_length is not None,
                                                 max_length=max_length, return_tensors="pt")
        return out["input_ids"][0]

    @property
    def prefix_len(self) -> int:
        if self._prefix is None:
            ids = self._ids("probe", None).tolist()
            head = self.tokenizer(USER_HEADER, add_special_tokens=False)["input_ids"]
            for pos in range(len(ids) - len(head) + 1):
                if ids[pos:pos + len(head)] == head:
                    self._prefix = pos + len(head)
                    break
            else:
                raise ValueError(f"user-turn header {USER_HEADER!r} not found in the templated prompt")
        return self._prefix

    def tokenize(self, text: str, limit: int) -> Caption:
        limit = min(int(limit), self.max_caption_tokens)
        ids = self._ids(text, self.prefix_len + limit)
        return Caption(text=text, full_length=int(ids.numel()), prefix_len=self.prefix_len,
                       cropped_length=int(ids.numel()) - self.prefix_len, token_ids=ids)

    # ---- features
    def _model_device(self):
        return next(self.model.parameters()).device

    @torch.no_grad()
    def _caption_rows(self, captions: Sequence[Caption]) -> Tuple[torch.Tensor, list]:
        """Hidden states of every caption's cropped span, packed in order (on the model's device),
        and the span lengths."""
        if self._packed is None:
            hidden, _ = self._padded(captions, self._model_device())
            rows = [hidden[i, :c.cropped_length] for i, c in enumerate(captions)]
            return torch.cat(rows, 0), [c.cropped_length for c in captions]
        lengths = [int(c.full_length) for c in captions]
        hidden = self._packed(torch.cat([c.token_ids.view(-1)[:n] for c, n in zip(captions, lengths)]), lengths)
        rows, a = [], 0
        for c, n in zip(captions, lengths):
            rows.append(hidden[a + c.prefix_len:a + n])
            a += n
        return torch.cat(rows, 0), [c.cropped_length for c in captions]

    @torch.no_grad()
    def _padded(self, captions: Sequence[Caption], device) -> Tuple[torch.Tensor, torch.Tensor]:
        pad = self.tokenizer.pad_token_id if self.tokenizer.pad_token_id is not None else self.tokenizer.eos_token_id
        L = max(c.full_length for c in captions)
        ids = torch.full((len(captions), L), pad, dtype=torch.long)
        mask = torch.zeros((len(captions), L), dtype=torch.long)
        for i, c in enumerate(captions):
            ids[i, :c.full_length] = c.token_ids
            mask[i, :c.full_length] = 1
        dev = self._model_device()
        hidden = self.model(input_ids=ids.to(dev), attention_mask=mask.to(dev), use_cache=False).last_hidden_state
        p = self.prefix_len
        return hidden[:, p:].to(device), mask[:, p:].to(device)

    def embed(self, captions: Sequence[Caption], device) -> torch.Tensor:
        if not captions:
            return torch.zeros(0, self.embed_dim, device=device)
        rows, _ = self._caption_rows(captions)
        return rows.to(device)

    def encode(self, texts, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Generation: ``(embeds [B, L, D], mask [B, L])`` of the caption spans, right-padded."""
        texts = [texts] if isinstance(texts, str) else list(texts)
        caps = [self.tokenize(t, self.max_caption_tokens) for t in texts]
        device = device if device is not None else self._model_device()
        rows, lengths = self._caption_rows(caps)
        L = max(lengths)
        out = rows.new_zeros(len(caps), L, rows.shape[-1])
        mask = torch.zeros(len(caps), L, dtype=torch.long)
        a = 0
        for i, n in enumerate(lengths):
            out[i, :n] = rows[a:a + n]
            mask[i, :n] = 1
            a += n
        return out.to(device), mask.to(device)


class HashTextEncoder:
    """Generation-side twin of :class:`~pan2_b200.data.items.HashCaptionCodec` (offline runs)."""

    def __init__(self, embed_dim: int = 4096, max_caption_tokens: int = 1000):
        from ..data.items import HashCaptionCodec
        self.codec = HashCaptionCodec(embed_dim=embed_dim)
        self.max_caption_tokens = max_caption_tokens

    def encode(self, texts, device=None):
        texts = [texts] if isinstance(texts, str) else list(texts)
        caps = [self.codec.tokenize(t, self.max_caption_tokens) for t in texts]
        L = max(c.cropped_length for c in caps)
        out = torch.zeros(len(caps), L, self.codec.embed_dim)
        mask = torch.zeros(len(caps), L, dtype=torch.long)
        for i, c in enumerate(caps):
            out[i, :c.cropped_length] = self.codec.embed([c], "cpu")
            mask[i, :c.cropped_length] = 1
        return out.to(device), mask.to(device)
