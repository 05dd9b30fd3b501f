"""Convert transformer weights between this framework's layout and the diffusers layout
(``PAN2Transformer3DModel``), in both directions, one block at a time.

    python -m pan2_b200.checkpoint.convert to-native --input PAN2/transformer --output pan2-native
    python -m pan2_b200.checkpoint.convert to-diffusers --input outputs/checkpoint-500 \\
        --output PAN2/transformer --training_config config/sft_29B_720p.yaml --dtype bf16

The diffusers tensor names and packing are fixed by the released checkpoints (the reference's
scripts/convert_checkpoint.py:1-304 documents them): fused projections are split there (QKV into
``to_q/k/v`` + ``add_q/k/v_proj``, ``out_proj`` into ``to_out.0`` + ``to_add_out``, the caption
encoder ``qkv`` into ``to_q/k/v``, per-modality q/k norm weights into ``norm_q/k`` +
``norm_added_q/k``); SwiGLU stores ``[w3; w1]``; the output-head modulation stores ``[scale; shift]``
(native: ``[shift; scale]``); only row 0 of the text-type table is kept; the timestep frequency table
is a constant rebuilt on load.

Inputs of ``to-diffusers`` are anything :class:`~pan2_b200.checkpoint.io.LazyStateDict` reads (this
framework's sharded ``checkpoint-N``, consolidated or single safetensors, ``.pt``, torch distributed
checkpoints); tensors are read
per block, so host memory holds one block at a time.  Outputs are 5 GB safetensors shards with an
index (and ``config.json`` for diffusers).
"""
from __future__ import annotations

import argparse
import glob
import json
import math
import os
from dataclasses import dataclass
from typing import Callable, Dict, List, Sequence, Tuple

import torch

SHARD_BYTES = 5 * 1024 ** 3
QKV6 = ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj")


@dataclass(frozen=True)
class Rule:
    """One native tensor <-> its diffusers parts.

    kind ``same``: one diffusers tensor; ``cat``: native = cat(parts, 0); ``swap``: native =
    cat(reversed(parts)) (the SwiGLU / head-modulation order flips); ``row0``: native is a table
    whose row 0 is the diffusers tensor (other rows zero)."""
    native: str
    diffusers: Tuple[str, ...]
    kind: str = "same"
    rows: int = 0  # row0: table height


def _rules(num_layers: int, num_refiner: int) -> List[List[Rule]]:
    """Rules grouped per conversion unit (globals, each refiner block, each joint block)."""
    g = [Rule("patch_embed.proj.weight", ("x_embedder.weight",)),
         Rule("patch_embed.proj.bias", ("x_embedder.bias",)),
         Rule("timestep_encoder.in_proj.weight", ("time_embedder.linear_1.weight",)),
         Rule("timestep_encoder.in_proj.bias", ("time_embedder.linear_1.bias",)),
         Rule("timestep_encoder.out_proj.weight", ("time_embedder.linear_2.weight",)),
         Rule("timestep_encoder.out_proj.bias", ("time_embedder.linear_2.bias",)),
         Rule("cap_embedder.0.weight", ("context_embedder.0.weight",)),
         Rule("cap_embedder.1.weight", ("context_embedder.1.weight",)),
         Rule("cap_embedder.1.bias", ("context_embedder.1.bias",)),
         Rule("text_type_embedding.weight", ("context_type_embedding",), "row0", rows=3),
         Rule("output_head.modulation.linear.weight", ("norm_out.linear.weight",), "swap"),
         Rule("output_head.modulation.linear.bias", ("norm_out.linear.bias",), "swap"),
         Rule("output_head.proj.weight", ("proj_out.weight",)),
         Rule("output_head.proj.bias", ("proj_out.bias",))]
    units = [g]
    for i in range(num_refiner):
        n, d = f"caption_encoder.blocks.{i}.", f"context_refiner.{i}."
        units.append([Rule(n + "attn_norm.weight", (d + "norm1.weight",)),
                      Rule(n + "ffn_norm.weight", (d + "norm2.weight",)),
                      Rule(n + "qkv.weight", tuple(d + f"attn.to_{x}.weight" for x in "qkv"), "cat"),
                      Rule(n + "q_norm.weight", (d + "attn.norm_q.weight",)),
                      Rule(n + "k_norm.weight", (d + "attn.norm_k.weight",)),
                      Rule(n + "attn_out.weight", (d + "attn.to_out.0.weight",)),
                      Rule(n + "ffn.w2.weight", (d + "ff.net.2.weight",)),
                      # diffusers packs [w3; w1] into one projection
                      Rule(n + "ffn.w1.weight", (d + "ff.net.0.proj.weight",), "half1"),
                      Rule(n + "ffn.w3.weight", (d + "ff.net.0.proj.weight",), "half0")])
    for i in range(num_layers):
        n, d = f"blocks.{i}.", f"transformer_blocks.{i}."
        u = [Rule(n + "modulation.linear.weight", (d + "norm1.linear.weight",)),
             Rule(n + "modulation.linear.bias", (d + "norm1.linear.bias",)),
             Rule(n + "text_modulation", (d + "scale_shift_table_context",)),
             Rule(n + "qkv_proj.weight", tuple(d + f"attn.{x}.weight" for x in QKV6), "cat"),
             Rule(n + "qkv_proj.bias", tuple(d + f"attn.{x}.bias" for x in QKV6), "cat"),
             Rule(n + "qkv_proj.q_weight", (d + "attn.norm_q.weight", d + "attn.norm_added_q.weight"), "cat"),
             Rule(n + "qkv_proj.k_weight", (d + "attn.norm_k.weight", d + "attn.norm_added_k.weight"), "cat"),
             Rule(n + "out_proj.weight", (d + "attn.to_out.0.weight", d + "attn.to_add_out.weight"), "cat"),
             Rule(n + "out_proj.bias", (d + "attn.to_out.0.bias", d + "attn.to_add_out.bias"), "cat")]
        for mod, ff in (("video", "ff"), ("text", "ff_context")):
            u += [Rule(n + f"ffn.w_up_{mod}", (d + f"{ff}.net.0.proj.weight",)),
                  Rule(n + f"ffn.b_up_{mod}", (d + f"{ff}.net.0.proj.bias",)),
                  Rule(n + f"ffn.w_down_{mod}", (d + f"{ff}.net.2.weight",)),
                  Rule(n + f"ffn.b_down_{mod}", (d + f"{ff}.net.2.bias",))]
        units.append(u)
    return units


def timestep_freqs(num_features: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    half = num_features // 2
    return torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32) / half)


def _to_native(rule: Rule, get: Callable[[str], torch.Tensor]) -> torch.Tensor:
    parts = [get(k) for k in rule.diffusers]
    if rule.kind == "same":
        return parts[0]
    if rule.kind == "cat":
        return torch.cat(parts, 0)
    if rule.kind == "swap":
        a, b = parts[0].chunk(2)
        return torch.cat([b, a], 0)
    if rule.kind == "half0":
        return parts[0].chunk(2)[0]
    if rule.kind == "half1":
        return parts[0].chunk(2)[1]
    if rule.kind == "row0":
        t = parts[0]
        return torch.cat([t[None], t.new_zeros(rule.rows - 1, *t.shape)], 0)
    raise ValueError(rule.kind)


def _to_diffusers(unit: Sequence[Rule], get: Callable[[str], torch.Tensor]) -> Dict[str, torch.Tensor]:
    out: Dict[str, torch.Tensor] = {}
    for r in unit:
        t = get(r.native)
        if r.kind == "same":
            out[r.diffusers[0]] = t
        elif r.kind == "cat":
            for k, p in zip(r.diffusers, t.chunk(len(r.diffusers), 0)):
                out[k] = p
        elif r.kind == "swap":
            a, b = t.chunk(2)
            out[r.diffusers[0]] = torch.cat([b, a], 0)
        elif r.kind in ("half0", "half1"):
            key = r.diffusers[0]
            halves = out.setdefault(key, [None, None])
            halves[0 if r.kind == "half0" else 1] = t
        elif r.kind == "row0":
            out[r.diffusers[0]] = t[0]
    for k, v in list(out.items()):
        if isinstance(v, list):
            if v[0] is None or v[1] is None:
                raise ValueError(f"incomplete SwiGLU pair for {k}")
            out[k] = torch.cat(v, 0)
    return out


class _ShardWriter:
    def __init__(self, out_dir: str, prefix: str, dtype=None):
        self.out_dir, self.prefix, self.dtype = out_dir, prefix, dtype
        os.makedirs(out_dir, exist_ok=True)
        self.cur: Dict[str, torch.Tensor] = {}
        self.size = 0
        self.files: List[Tuple[str, List[str]]] = []
        self.total = 0

    def add(self, tensors: Dict[str, torch.Tensor]) -> None:
        for k, v in tensors.items():
            v = v.to(self.dtype) if self.dtype is not None and v.is_floating_point() else v
            nb = v.numel() * v.element_size()
            if self.cur and self.size + nb > SHARD_BYTES:
                self._flush()
            self.cur[k] = v.contiguous()
            self.size += nb
            self.total += nb

    def _flush(self) -> None:
        from safetensors.torch import save_file
        name = f"{self.prefix}-{len(self.files) + 1:05d}.tmp.safetensors"
        save_file(self.cur, os.path.join(self.out_dir, name), metadata={"format": "pt"})
        self.files.append((name, list(self.cur)))
        self.cur, self.size = {}, 0

    def close(self) -> List[str]:
        if self.cur or not self.files:
            self._flush()
        n = len(self.files)
        weight_map, paths = {}, []
        for i, (tmp, keys) in enumerate(self.files, 1):
            final = f"{self.prefix}-{i:05d}-of-{n:05d}.safetensors"
            os.replace(os.path.join(self.out_dir, tmp), os.path.join(self.out_dir, final))
            paths.append(os.path.join(self.out_dir, final))
            for k in keys:
                weight_map[k] = final
        with open(os.path.join(self.out_dir, f"{self.prefix}.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": self.total}, "weight_map": weight_map}, f, indent=1)
        return paths


def _diffusers_reader(folder: str):
    from safetensors import safe_open
    idx = os.path.join(folder, "diffusion_pytorch_model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            wm = json.load(f)["weight_map"]
    else:
        wm = {}
        for shard in glob.glob(os.path.join(folder, "*.safetensors")):
            with safe_open(shard, "pt") as h:
                wm.update({k: os.path.basename(shard) for k in h.keys()})
    handles, used = {}, set()

    def get(k):
        fn = wm[k]
        if fn not in handles:
            handles[fn] = safe_open(os.path.join(folder, fn), "pt")
        used.add(k)
        return handles[fn].get_tensor(k)
    return wm, get, used


def convert_to_native(src: str, out_dir: str, dtype=None, prefix: str = "model") -> List[str]:
    with open(os.path.join(src, "config.json")) as f:
        cfg = json.load(f)
    wm, get, used = _diffusers_reader(src)
    w = _ShardWriter(out_dir, prefix, dtype)
    for unit in _rules(int(cfg["num_layers"]), int(cfg["num_refiner_layers"])):
        w.add({r.native: _to_native(r, get) for r in unit})
    w.add({"timestep_encoder.freqs": timestep_freqs()})
    left = sorted(set(wm) - used)
    if left:
        raise ValueError(f"unconverted diffusers tensors: {left[:10]}")
    return w.close()


def diffusers_config(arch: dict, num_refiner: int = 4) -> dict:
    return {"_class_name": "PAN2Transformer3DModel",
            "attention_head_dim": arch["hidden_size"] // arch["num_attention_heads"],
            "context_mlp_ratio": float(arch["context_mlp_ratio"]), "in_channels": arch["in_channels"],
            "mlp_ratio": float(arch["mlp_ratio"]), "num_attention_heads": arch["num_attention_heads"],
            "num_layers": arch["num_layers"], "num_refiner_layers": num_refiner, "out_channels": arch["out_channels"],
            "patch_size": list(arch["patch_size"]), "refiner_mlp_ratio": 4.0,
            "rope_axes_dim": list(arch["rope_axes_dim"]), "rope_temporal_scale": float(arch["rope_temporal_scale"]),
            "rope_theta": float(arch["rope_theta"]), "text_embed_dim": arch["text_embed_dim"]}


def convert_to_diffusers(src: str, out_dir: str, arch: dict, dtype=None, num_refiner: int = 4) -> List[str]:
    from .io import LazyStateDict
    sd = LazyStateDict(src)
    strip = {}
    for k in sd.keys():
        strip[k.removeprefix("module.").removeprefix("model.")] = k
    used = set()

    def get(k):
        if k not in strip:
            raise KeyError(f"{src} has no tensor {k}")
        used.add(k)
        return sd.get(strip[k])
    w = _ShardWriter(out_dir, "diffusion_pytorch_model", dtype)
    for unit in _rules(int(arch["num_layers"]), num_refiner):
        w.add(_to_diffusers(unit, get))
    left = sorted(set(strip) - used - {"timestep_encoder.freqs"})
    if left:
        raise ValueError(f"unconverted native tensors: {left[:10]}")
    paths = w.close()
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(diffusers_config(arch, num_refiner), f, indent=2)
    return paths


def _arch_from_yaml(path: str) -> dict:
    import yaml
    from ..models.transformer import ARCH_DEFAULTS, translate_architecture_config
    with open(path) as f:
        doc = yaml.safe_load(f) or {}
    arch = dict(ARCH_DEFAULTS)
    arch.update(translate_architecture_config((doc.get("model") or {}).get("transformer_config_overrides") or {}))
    return arch


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="direction", required=True)
    p = sub.add_parser("to-native", help="diffusers transformer folder -> this framework's layout")
    p.add_argument("--input", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--dtype", choices=["bf16", "fp32"], default=None)
    p = sub.add_parser("to-diffusers", help="this framework's checkpoint -> diffusers transformer folder")
    p.add_argument("--input", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--training_config", default="config/sft_29B_720p.yaml")
    p.add_argument("--dtype", choices=["bf16", "fp32"], default=None)
    a = ap.parse_args(argv)
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32, None: None}[a.dtype]
    if a.direction == "to-native":
        paths = convert_to_native(a.input, a.output, dt)
    else:
        paths = convert_to_diffusers(a.input, a.output, _arch_from_yaml(a.training_config), dt)
    print(f"wrote {len(paths)} shard(s) to {a.output}")


if __name__ == "__main__":
    main()
