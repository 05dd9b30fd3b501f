"""Training options: one table that is at once the CLI, the YAML schema and the defaults.

The option names, flags, defaults and validation rules are the reference trainer's
(train.py:107-412) so existing YAML files and launch lines keep working: YAML keys are option names
grouped under any sections; unknown keys, duplicate keys and removed keys are errors; ``sp_size``,
``i2v_prob`` and ``v2v_prob`` are accepted as legacy spellings; the command line overrides the
YAML file, which overrides the defaults.  Options specific to this framework live under the
``kernels`` / ``comm`` names and are registered here as well, so strictness is kept.
"""
from __future__ import annotations

import argparse
import json
import math
import os
from dataclasses import MISSING, dataclass, field, fields
from enum import Enum
from typing import Any, Dict, List, Mapping, Optional

from ..diffusion.flow_matching import NoiseDraw, ShiftRule


class ConditioningSchema(str, Enum):
    TOKEN_CONCAT = "token_concat"
    CHANNEL_CONCAT = "channel_concat"


LR_SCHEDULER_TYPES = ("constant_with_warmup", "linear_decay", "cosine_decay")
LEGACY_KEYS = {"sp_size": "cp_size", "i2v_prob": "image_cond_prob", "v2v_prob": "video_cond_prob"}
# removed keys still accepted when they carry their only meaningful value
IGNORED_KEYS = {"single_stream_only": (True, False), "single_stream_block_type": ("mm_joint_attn",),
                "single_stream_depth": (None,)}


def str_to_bool(v) -> bool:
    if isinstance(v, bool):
        return v
    s = str(v).strip().lower()
    if s in ("1", "true", "t", "yes", "y", "on"):
        return True
    if s in ("0", "false", "f", "no", "n", "off"):
        return False
    raise argparse.ArgumentTypeError(f"{v!r} is not a boolean (true/false, yes/no, 1/0)")


def parse_json_object(raw, name: str) -> Optional[Dict[str, Any]]:
    """A JSON object given inline, as a path to a JSON file, or already as a mapping."""
    if raw is None or isinstance(raw, Mapping):
        return None if raw is None else dict(raw)
    text = str(raw)
    if os.path.isfile(text):
        with open(text) as f:
            text = f.read()
    try:
        obj = json.loads(text)
    except json.JSONDecodeError as exc:
        raise ValueError(f"--{name}: neither a JSON object nor a readable JSON file ({exc})") from exc
    if not isinstance(obj, dict):
        raise ValueError(f"--{name} holds JSON that is not an object")
    return obj


def opt(default, kind, help, factory=None, **cli):
    """One option: ``kind`` is a type or 'switch' / 'set' / 'unset' / 'list'; ``cli`` may hold flags,
    dest, choices, convert or cli=False."""
    meta = {"kind": kind, "help": help, **cli}
    return field(default_factory=factory, metadata=meta) if factory is not None else field(default=default, metadata=meta)


@dataclass
class TrainingConfig:
    # -- model
    transformer_config_overrides: Optional[Dict[str, Any]] = opt(
        None, str, "Architecture overrides (JSON object, JSON file, or YAML mapping).",
        convert=lambda raw: parse_json_object(raw, "transformer_config_overrides"))
    zero_init_modulation: bool = opt(False, "switch", "Start every adaLN modulation projection at zero.")
    text_encoder_hidden_state_skip_layer: int = opt(2, int, "Drop this many final text-encoder layers.")
    load_transformer_weights: bool = opt(False, "switch", "Warm start from pretrained_transformer_path.")
    pretrained_transformer_path: Optional[str] = opt(None, str, "State dict file/folder or checkpoint-N directory.")
    # -- optimization
    use_muon: bool = opt(True, "switch", "Muon for 2-D weight matrices, AdamW for the rest.")
    learning_rate: float = opt(1e-5, float, "Peak learning rate.")
    weight_decay: float = opt(0.05, float, "Decoupled weight decay.")
    max_steps: int = opt(10000, int, "Optimizer steps.")
    warmup_steps: int = opt(500, int, "Linear warmup steps.")
    lr_warmup_start_ratio: float = opt(0.0, float, "Warmup starts at this fraction of the peak LR.")
    lr_scheduler_type: str = opt("constant_with_warmup", str, "LR shape after warmup.", choices=LR_SCHEDULER_TYPES)
    lr_decay_steps: Optional[int] = opt(None, int, "Decay length; max_steps - warmup_steps when unset.")
    lr_decay_floor_ratio: float = opt(0.30, float, "Decay ends at this fraction of the peak LR.")
    gradient_accumulation_steps: int = opt(1, int, "Micro-batches per optimizer step.")
    max_grad_norm: float = opt(1.0, float, "Global gradient-norm clip; 0 disables.")
    # -- flow matching
    num_train_timesteps: int = opt(1000, int, "Length T of the training time axis.", cli=False)
    snr_type: NoiseDraw = opt(NoiseDraw.LOGNORM, str, "Noise-level distribution.",
                              flags=["--flow_snr_type"], dest="flow_snr_type",
                              choices=[d.value for d in NoiseDraw], convert=NoiseDraw)
    flow_lognorm_loc: float = opt(0.0, float, "Logit-normal mean.")
    flow_lognorm_scale: float = opt(1.0, float, "Logit-normal std.")
    train_timestep_shift_mode: ShiftRule = opt(ShiftRule.FIXED, str, "fixed or dynamic shift.",
                                               choices=[m.value for m in ShiftRule], convert=ShiftRule)
    train_timestep_shift: float = opt(5.0, float, "Fixed-mode time shift s.")
    train_timestep_rescale_factor: float = opt(0.5, float, "Dynamic mode: exponent scale.")
    train_timestep_max_shift: float = opt(1000.0, float, "Dynamic mode: upper bound of the shift.")
    # -- conditioning
    image_cond_prob: float = opt(0.3, float, "Fraction trained as image-to-video.",
                                 flags=["--image_cond_prob", "--i2v_prob"])
    video_cond_prob: float = opt(0.0, float, "Fraction trained as video continuation.",
                                 flags=["--video_cond_prob", "--v2v_prob"])
    cfg_drop_prob: float = opt(0.1, float, "Fraction with every condition dropped (CFG).")
    conditioning_schema: ConditioningSchema = opt(ConditioningSchema.TOKEN_CONCAT, str, "How context frames enter.",
                                                  choices=[c.value for c in ConditioningSchema],
                                                  convert=ConditioningSchema)
    # -- data
    packed_dataloader_meta_csv_path: list = opt(None, "list", "Video metadata CSV files or folders.",
                                                factory=lambda: ["dummy_meta.csv"])
    image_tar_path: list = opt(None, "list", "Image-latent tar shards (folders, tars or list files).", factory=list)
    image_sample_prob: float = opt(0.0, float, "Chance an item comes from image_tar_path.")
    video_height: int = opt(480, int, "Frame height.")
    video_width: int = opt(832, int, "Frame width.")
    batch_size: int = opt(1, int, "Per-rank batch size (packed batches are budget-sized).")
    packed_joint_token_budget: int = opt(7312, int, "Video + caption tokens per packed batch.")
    packed_video_token_budget: int = opt(7056, int, "Video tokens per packed batch.")
    packed_caption_token_budget: int = opt(1024, int, "Caption tokens per packed batch.")
    packed_joint_segment_limit: int = opt(7312, int, "Video + caption tokens of one sequence.")
    packed_caption_segment_limit: int = opt(256, int, "Caption tokens of one sequence.")
    packed_dataloader_max_num_seq: int = opt(8, int, "Sequences per packed batch at most.")
    packed_dataloader_num_buffers: int = opt(4, int, "Packing buffers.")
    packed_dataloader_prefetch_factor: int = opt(2, int, "Batches prepared ahead.")
    packed_dataloader_num_workers: int = opt(32, int, "Loader threads.")
    resume_video_csv: bool = opt(True, "switch", "On resume, continue the video CSV stream.")
    # -- parallelism and memory
    cp_size: int = opt(1, int, "Ulysses context-parallel degree.", flags=["--cp_size", "--sp_size"])
    hybrid_shard: bool = opt(False, "set", "Shard within a node, replicate across nodes.")
    enable_gradient_checkpointing: bool = opt(True, "switch", "Recompute block activations in backward.")
    use_dedicated_gradient_checkpointing: bool = opt(False, "set", "Selective checkpointing: keep each block's attention "
                                                     "output from the forward instead of recomputing it.")
    compile_text_encoder: bool = opt(False, "set", "Compile the text encoder (not used: eager CUDA kernels).")
    compile_transformer: bool = opt(False, "set", "Compile the transformer (not used: eager CUDA kernels).")
    compile_optimizer: bool = opt(False, "set", "Compile the optimizer (not used: fused CUDA kernels).")
    dtype: str = opt("bf16", str, "Compute precision.", choices=("bf16", "fp32"))
    legacy_eager_mode: bool = opt(True, "switch", "Validated execution mode; must stay true.")
    # -- checkpoints, logging, safety
    output_dir: str = opt("./outputs", str, "checkpoint-N/ directories and logs.")
    save_interval: int = opt(1000, int, "Checkpoint every this many steps.")
    save_total_limit: int = opt(0, int, "Keep this many recent checkpoints; 0 keeps all.")
    log_interval: int = opt(10, int, "Log every this many steps.")
    report_to: str = opt("none", str, "Metrics sink.", choices=("none", "wandb"))
    seed: int = opt(42, int, "Seed (model init identical on all ranks; data adds the data rank).")
    anomaly_detection: bool = opt(True, "unset", "Disable loss/grad anomaly checks.", flags=["--no_anomaly"],
                                  dest="anomaly_detection")
    anomaly_detection_warmup_steps: int = opt(100, int, "No spike-based stop during these steps.")
    max_consecutive_skipped_steps: int = opt(5, int, "Skipped non-finite steps before recovery.")
    # -- this framework
    optimizer_offload: str = opt("auto", str, "Optimizer state placement: auto, on or off.", choices=("auto", "on", "off"))
    activation_reserve_gb: float = opt(0.0, float, "GPU memory kept free for activations when planning offload "
                                                   "(0: automatic).")
    fault_injection: Optional[str] = opt(None, str, "Host-side fault injection spec, e.g. 'nan_loss@5,stall@7:2'.")
    text_encoder: str = opt("qwen", str, "Caption embeddings: the Qwen3.5 encoder, or a deterministic hash "
                                         "stand-in for offline smoke runs.", choices=("qwen", "hash"))
    text_encoder_path: str = opt("Qwen/Qwen3.5-9B", str, "Hugging Face id or local folder of the text encoder.")
    heartbeat_timeout_s: float = opt(50000.0, float, "Exit a rank whose loop made no progress for this long.")
    process_group_timeout_s: float = opt(1800.0, float, "Collective timeout of the process groups.")
    profile_step: int = opt(10, int, "cudaProfilerStart after this step (-1: never).")

    def check(self) -> None:
        """Reject inconsistent settings with an error naming the option."""
        if not self.legacy_eager_mode:
            raise ValueError("legacy_eager_mode=false is not supported: this trainer always runs eagerly")
        if self.warmup_steps < 0:
            raise ValueError(f"warmup_steps={self.warmup_steps} is negative")
        if self.lr_decay_steps is not None and self.lr_decay_steps < 0:
            raise ValueError(f"lr_decay_steps={self.lr_decay_steps} is negative")
        for name in ("lr_warmup_start_ratio", "lr_decay_floor_ratio"):
            v = getattr(self, name)
            if not math.isfinite(v) or not 0.0 <= v <= 1.0:
                raise ValueError(f"{name}={v!r} is not a finite value between 0 and 1")
        if self.anomaly_detection_warmup_steps < 0:
            raise ValueError("anomaly_detection_warmup_steps cannot be negative")
        if not (math.isfinite(self.image_cond_prob) and math.isfinite(self.video_cond_prob)):
            raise ValueError("image_cond_prob and video_cond_prob must be finite numbers")
        if self.image_cond_prob < 0 or self.video_cond_prob < 0 or self.image_cond_prob + self.video_cond_prob > 1:
            raise ValueError("image_cond_prob and video_cond_prob are probabilities of exclusive tasks: each >= 0, together <= 1")
        if not (math.isfinite(self.flow_lognorm_loc) and math.isfinite(self.flow_lognorm_scale)):
            raise ValueError("flow_lognorm_loc and flow_lognorm_scale must be finite numbers")
        if self.flow_lognorm_scale <= 0:
            raise ValueError("flow_lognorm_scale (the logit-normal std) must be positive")
        if self.train_timestep_shift <= 0:
            raise ValueError("train_timestep_shift must be positive")
        if self.train_timestep_rescale_factor < 0:
            raise ValueError("train_timestep_rescale_factor cannot be negative")
        if self.train_timestep_max_shift <= 0:
            raise ValueError("train_timestep_max_shift must be positive")
        if self.pretrained_transformer_path and not self.load_transformer_weights:
            raise ValueError("a pretrained_transformer_path is given while load_transformer_weights is off; set one consistently with the other")
        if self.load_transformer_weights and not self.pretrained_transformer_path:
            raise ValueError("load_transformer_weights is on but no pretrained_transformer_path is given")
        if self.load_transformer_weights and not os.path.exists(self.pretrained_transformer_path):
            raise FileNotFoundError(f"pretrained_transformer_path {self.pretrained_transformer_path} does not exist")
        if self.gradient_accumulation_steps < 1:
            raise ValueError("gradient_accumulation_steps must be at least 1")


def _cli_fields():
    return [(f, f.metadata) for f in fields(TrainingConfig) if f.metadata.get("cli", True)]


def build_arg_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="Train PAN 2 on video data (B200)")
    ap.add_argument("--config", type=str, default=None, help="YAML file; command-line flags take precedence.")
    for f, meta in _cli_fields():
        default = f.default_factory() if f.default is MISSING else f.default
        if isinstance(default, Enum):
            default = default.value
        spec = {"dest": meta.get("dest", f.name), "help": meta["help"]}
        kind = meta["kind"]
        if kind == "switch":
            spec.update(type=str_to_bool, nargs="?", const=True, default=default)
        elif kind == "set":
            spec.update(action="store_true")
        elif kind == "unset":
            spec.update(action="store_false")
        elif kind == "list":
            spec.update(type=str, nargs="+", default=default)
        else:
            spec.update(type=kind, default=default)
        if "choices" in meta:
            spec["choices"] = list(meta["choices"])
        ap.add_argument(*meta.get("flags", [f"--{f.name}"]), **spec)
    return ap


def load_yaml_defaults(path: str, parser: argparse.ArgumentParser) -> Dict[str, Any]:
    """Flatten a sectioned YAML file into option defaults (strict about unknown / duplicate keys)."""
    import yaml
    with open(path, "r", encoding="utf-8") as f:
        obj = yaml.safe_load(f)
    if obj is None:
        return {}
    if not isinstance(obj, Mapping):
        raise ValueError(f"{path}: the training config must be a YAML mapping of sections")
    actions = {a.dest: a for a in parser._actions if a.dest not in ("help", argparse.SUPPRESS)}
    out: Dict[str, Any] = {}

    def visit(node: Mapping, trail=()):
        for raw_key, value in node.items():
            key = LEGACY_KEYS.get(str(raw_key), str(raw_key))
            here = (*trail, str(raw_key))
            if key in IGNORED_KEYS:
                if value not in IGNORED_KEYS[key]:
                    raise ValueError(f"Training config key {'.'.join(here)!r} is no longer supported")
                continue
            if key in actions:
                if key in out:
                    raise ValueError(f"training config sets {key!r} twice (again at {'.'.join(here)})")
                out[key] = value
            elif isinstance(value, Mapping):
                visit(value, here)
            else:
                raise ValueError(f"training config key {'.'.join(here)!r} is not an option")

    visit(obj)
    for key, value in list(out.items()):
        a = actions[key]
        if a.type is str_to_bool and isinstance(value, str):
            value = str_to_bool(value)
        if a.nargs in ("+", "*") and value is not None and not isinstance(value, list):
            value = [value]
        out[key] = value
    return out


def parse_training_config(argv: Optional[List[str]] = None) -> TrainingConfig:
    """Defaults <- YAML (--config) <- command line, converted and checked."""
    parser = build_arg_parser()
    probe, _ = parser.parse_known_args(argv)
    if probe.config:
        parser.set_defaults(**load_yaml_defaults(probe.config, parser))
    args = parser.parse_args(argv)
    values = {}
    for f, meta in _cli_fields():
        raw = getattr(args, meta.get("dest", f.name))
        values[f.name] = meta["convert"](raw) if "convert" in meta else raw
    cfg = TrainingConfig(**values)
    cfg.check()
    return cfg
