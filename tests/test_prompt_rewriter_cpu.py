"""Structured-caption tools: schema validation, negative rendering, assembly, token counting."""
import json

import pytest
import torch

from pan2_b200.inference.prompt_rewriter import (CaptionError, EncoderTokenCounter, assemble, render_negative,
                                                  validate_positive, validate_records)
from decimal import Decimal


def _positive(duration=4):
    half = duration / 2
    cap = {"video_style": "cinematic", "lighting": "soft daylight", "perspective_view": "eye level",
           "subjects_lifecycle": [{"subject_id": "<|Subject1|>", "display_name": "a dog",
                                   "subject_attribute": "brown fur"}],
           "init_frame_visual_description": "A dog sits on grass.",
           "events": [{"event_index": 0, "time_range_sec": f"0 to {half:g}", "event_description": "The dog stands.",
                       "camera_motion": [{"time_range_sec": f"0 to {half:g}", "camera_motion": ["static"]}],
                       "contained_actions": [{"time_range_sec": f"0 to {half:g}", "action": "<|Subject1|> stands up"}]},
                      {"event_index": 1, "time_range_sec": f"{half:g} to {duration:g}", "event_description": "It runs.",
                       "camera_motion": [{"time_range_sec": f"{half:g} to {duration:g}", "camera_motion": ["pan_left", "zoom_in"]}],
                       "contained_actions": []}],
           "quality": {"video_quality": "sharp", "text_logos_overlays": None, "artifacts": None}}
    return cap


NEG = json.dumps({"video_style": "x", "lighting": "x", "perspective_view": "x", "subjects_lifecycle": [],
                  "init_frame_visual_description": "x",
                  "events": [{"time_range_sec": "0 to {duration_sec}", "camera_motion": [{"time_range_sec": "0 to {duration_sec}"}],
                              "contained_actions": [{"time_range_sec": "0 to {duration_sec}"}]}],
                  "quality": {}})


def test_validate_positive_accepts_and_rejects():
    good = json.dumps(_positive())
    validate_positive(good, Decimal(4))
    bad_cases = []
    c = _positive(); c["events"][1]["time_range_sec"] = "2 to 3"; bad_cases.append(c)        # gap at the end
    c = _positive(); c["events"][0]["camera_motion"][0]["camera_motion"] = ["fly"]; bad_cases.append(c)
    c = _positive(); c["events"][0]["contained_actions"][0]["action"] = "stands <|Subject1|>"; bad_cases.append(c)
    c = _positive(); c["subjects_lifecycle"][0]["subject_id"] = "<|Subject2|>"; bad_cases.append(c)
    c = _positive(); c["quality"]["artifacts"] = "blur"; bad_cases.append(c)
    c = _positive(); c["lighting"] = "lit on <|Subject1|>"; bad_cases.append(c)
    for c in bad_cases:
        with pytest.raises(CaptionError):
            validate_positive(json.dumps(c), Decimal(4))
    with pytest.raises(CaptionError):
        validate_positive('{"video_style": 1, "video_style": 2}', Decimal(4))


def test_negative_and_assembly():
    neg = render_negative(NEG, 7.5)
    assert neg.count('"0 to 7.5"') == 3 and "{duration_sec}" not in neg
    assert neg.replace('"0 to 7.5"', '"0 to {duration_sec}"') == NEG
    req = [{"original_prompt": "a dog runs", "duration_sec": 4, "id": "x"}]
    pos = [{"refined_prompt": json.dumps(_positive(), separators=(",", ":"))}]
    out = assemble(req, pos, NEG)
    assert out[0]["id"] == "x" and out[0]["negative_prompt"].count('"0 to 4"') == 3
    rep = validate_records(out)
    assert rep["ok"] and not rep["token_verified"]
    default = assemble({"original_prompt": "p"}, {"refined_prompt": json.dumps(_positive(13))}, NEG)
    assert default["duration_sec"] == 13
    with pytest.raises(CaptionError):
        assemble({"original_prompt": "p", "duration_sec": 5}, {"refined_prompt": json.dumps(_positive(4))}, NEG)


class _FakeTok:
    def apply_chat_template(self, chat, add_generation_prompt, tokenize, return_dict, truncation, max_length,
                            return_tensors):
        text = "".join(f"<|im_start|>{m['role']}\n{m['content']}" for m in chat) + "<|im_start|>assistant\n"
        return {"input_ids": torch.tensor([[ord(c) for c in text]])}

    def __call__(self, text, add_special_tokens=False):
        return {"input_ids": [ord(c) for c in text]}


def test_token_counter_crops_the_template():
    c = EncoderTokenCounter(tokenizer=_FakeTok())
    tail = len("<|im_start|>assistant\n")
    assert c("abcd") == 4 + tail
    assert c("abcdefgh") - c("abcd") == 4
