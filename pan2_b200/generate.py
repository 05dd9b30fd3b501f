"""Video generation entry point (``python generate.py ...`` / ``torchrun ... generate.py ...``).

Same command-line surface as the reference's generate.py:1-595 -- prompt or prompt JSON input, task
filter, prompt sharding, skip-existing, all sampler and guidance controls, training-YAML architecture
import, checkpoint loading, video writing and the ``<video>_config.json`` settings record -- plus:

* ``--sp_size N``: Ulysses sequence parallel over N ranks per prompt (the other ranks of the job shard
  the prompts); one process per GPU;
* ``--text_encoder {qwen,hash}``: the Qwen3.5 caption encoder, or a deterministic stand-in for runs
  without its weights;
* ``--output_type {video,latent}``: latents are written as ``<stem>.latent.safetensors`` when no VAE
  (diffusers + Wan 2.2 weights) is available.

Checkpoints: a training ``checkpoint-N`` folder (or its ``transformer/``) in this framework's sharded
format, consolidated safetensors shards, a single safetensors file or a plain ``.pt`` state dict.
"""
from __future__ import annotations

import os

os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import argparse
import copy
import datetime
import json
import sys
from typing import List

import torch
import torch.distributed as dist

from .config.training import parse_json_object, str_to_bool
from .inference.guidance import validate_sampling_extensions
from .inference.inputs import GUIDANCE_KEYS, is_complete, load_inference_inputs

MODEL_LABEL = "pan2"


def _main_rank() -> bool:
    return not dist.is_initialized() or dist.get_rank() == 0


def _log(msg: str) -> None:
    if _main_rank():
        print(msg, flush=True)


def write_video(video: torch.Tensor, path: str, fps: float = 24, crf=None, preset=None, pix_fmt=None) -> str:
    """Float video in [0, 1] (``[C, F, H, W]`` or ``[1, C, F, H, W]``) -> file.  Uses imageio/ffmpeg when
    installed; otherwise writes the frames as PNGs into ``<stem>_frames/`` and returns that folder."""
    if video.ndim == 5:
        if video.shape[0] != 1:
            raise ValueError(f"write_video takes one video, got a batch of {video.shape[0]}")
        video = video[0]
    frames = (video * 255).clamp(0, 255).to(torch.uint8).permute(1, 2, 3, 0).cpu().numpy()
    try:
        import imageio
    except ImportError:
        from PIL import Image
        folder = os.path.splitext(path)[0] + "_frames"
        os.makedirs(folder, exist_ok=True)
        for i, f in enumerate(frames):
            Image.fromarray(f).save(os.path.join(folder, f"{i:05d}.png"))
        return folder
    # written under a temporary name and renamed, so an interrupted write never leaves a truncated
    # file under the final name (the resume check treats a present, non-empty file as finished)
    stem, ext = os.path.splitext(path)
    tmp = f"{stem}.partial{ext}"
    if frames.shape[0] == 1:
        imageio.imwrite(tmp, frames[0])
        os.replace(tmp, path)
        return path
    opts, params = {}, []
    if crf is not None:
        opts.update(codec="libx264", quality=None)
        params += ["-crf", str(crf)]
    if preset is not None:
        params += ["-preset", preset]
    if params:
        opts["ffmpeg_params"] = params
    if pix_fmt is not None:
        opts["pixelformat"] = pix_fmt
    imageio.mimwrite(tmp, frames, fps=fps, **opts)
    os.replace(tmp, path)
    return path


def save_settings(args, video_path: str, task: str) -> str:
    def plain(v):
        try:
            json.dumps(v)
            return v
        except (TypeError, ValueError):
            return str(v)
    doc = {"model": MODEL_LABEL, "task": task, "video": video_path, "written_at": datetime.datetime.now().isoformat(),
           "arguments": {k: plain(v) for k, v in vars(args).items() if not k.startswith("_") and not callable(v)}}
    out = os.path.splitext(video_path)[0] + "_config.json"
    with open(out + ".partial", "w", encoding="utf-8") as f:
        json.dump(doc, f, indent=2, ensure_ascii=False)
    os.replace(out + ".partial", out)
    return out


def read_training_config(args) -> None:
    """Architecture and text-encoder settings from the training YAML's ``model`` / ``data`` sections."""
    if not args.training_config:
        return
    import yaml
    if not os.path.isfile(args.training_config):
        raise ValueError(f"training config {args.training_config} does not exist")
    with open(args.training_config, encoding="utf-8") as f:
        doc = yaml.safe_load(f) or {}
    model, data = doc.get("model") or {}, doc.get("data") or {}
    if not isinstance(model, dict) or not isinstance(data, dict):
        raise ValueError(f"{args.training_config}: the model and data sections must be YAML mappings")
    if model.get("single_stream_block_type", "mm_joint_attn") != "mm_joint_attn":
        raise ValueError("only joint-attention blocks exist here: model.single_stream_block_type must be mm_joint_attn")
    arch = dict(model.get("transformer_config_overrides") or {})
    if model.get("zero_init_modulation") is not None:
        arch["zero_init_modulation"] = model["zero_init_modulation"]
    if arch:
        args.transformer_config_overrides = json.dumps(arch)
    if model.get("text_encoder_hidden_state_skip_layer") is not None:
        args.text_encoder_hidden_state_skip_layer = model["text_encoder_hidden_state_skip_layer"]
    if data.get("packed_caption_segment_limit") is not None:
        args.text_encoder_max_length = int(data["packed_caption_segment_limit"])


def architecture(overrides) -> dict:
    from .models.transformer import ARCH_DEFAULTS, translate_architecture_config
    arch = dict(ARCH_DEFAULTS)
    arch.update(translate_architecture_config(parse_json_object(overrides, "transformer_config_overrides") or {}))
    return arch


def prepare_jobs(args, task: str) -> List[argparse.Namespace]:
    if args.image_root is not None and not args.prompt_json:
        raise ValueError("--image_root remaps the images of a prompt file: give --prompt_json too")
    if task == "auto" and not args.prompt_json:
        raise ValueError("--task auto reads each entry's task from a prompt file: give --prompt_json")
    if args.prompt_json:
        if args.output_path or not args.output_dir or args.image_path:
            raise ValueError("a prompt file writes one video per entry under --output_dir; reference images belong in its entries, not in --image_path")
        recs = load_inference_inputs(args.prompt_json, args.output_dir, task=task, fps=args.fps, fallback=args.video_length,
                                     shard_index=0 if task == "auto" else args.prompt_shard_index,
                                     shard_count=1 if task == "auto" else args.prompt_shard_count,
                                     default_negative=args.negative_prompt, image_root=args.image_root)
        if task == "auto":
            if args.stg_scale != 0 and any(r["task"] == "i2v" for r in recs):
                raise ValueError("skip-layer guidance is text-to-video only, and this prompt file has image-to-video entries")
            recs = recs[args.prompt_shard_index::args.prompt_shard_count]
    else:
        if args.output_dir or (args.prompt_shard_index, args.prompt_shard_count) != (0, 1):
            raise ValueError("--output_dir and --prompt_shard_* apply to prompt files: give --prompt_json")
        prompts = args.prompt if isinstance(args.prompt, list) else [args.prompt]
        refs = args.image_path if task == "i2v" else None
        if task == "i2v" and not refs:
            raise ValueError("image-to-video needs a reference image: --image_path, or per-entry images in --prompt_json")
        if refs is not None and len(refs) != len(prompts):
            raise ValueError("give one reference image per --prompt")
        recs = []
        for i, pr in enumerate(prompts):
            out = args.output_path
            if out and len(prompts) > 1:
                b, e = os.path.splitext(out)
                out = f"{b}_{i}{e}"
            r = dict(prompt=pr, negative_prompt=args.negative_prompt, video_length=args.video_length, output_path=out)
            if refs is not None:
                r["image_path"] = refs[i]
            recs.append(r)
    jobs = []
    for r in recs:
        j = copy.copy(args)
        vars(j).update(r)
        j.task = r.get("task", task)
        j.i2v_skip_first_latent_cfg = j.task == "i2v" and args.i2v_skip_first_latent_cfg
        if args.skip_existing and j.output_path and is_complete(j):
            _log(f"skipping complete output: {j.output_path}")
        else:
            jobs.append(j)
    return jobs


def build_pipeline(args, sp_group=None):
    from .models.text_encoder import HashTextEncoder, QwenCaptionCodec
    from .pipelines.video import PanVideoPipeline, build_inference_model, load_transformer_weights
    from .inference.offload import choose_offload
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    arch = architecture(args.transformer_config_overrides)
    dtype = {"bf16": torch.bfloat16, "fp32": torch.float32}[args.dtype]
    offload = choose_offload(args.offload, dit_bytes(arch, dtype), dev)
    if args.compile:
        _log("--compile has no effect: the transformer blocks run hand-written kernels")
    # with offloading the models are built on the CPU and moved to the GPU while they run
    home = dev if offload == "none" else torch.device("cpu")
    model = build_inference_model(arch, home, dtype=dtype, seed=0)
    if args.checkpoint_path:
        load_transformer_weights(model, args.checkpoint_path)
        _log(f"transformer weights loaded from {args.checkpoint_path}")
    max_len = args.text_encoder_max_length or 1000
    if args.text_encoder == "hash":
        te = HashTextEncoder(embed_dim=int(arch.get("text_embed_dim", 4096)), max_caption_tokens=max_len)
    else:
        te = QwenCaptionCodec(args.text_encoder_path, device=home, hidden_state_skip_layer=args.text_encoder_hidden_state_skip_layer,
                              max_caption_tokens=max_len)
    vae = None
    if args.output_type == "video":
        from .models.vae import WanVAE
        vae = WanVAE(args.wan_vae_checkpoint, device=home)
    pipe = PanVideoPipeline(model, te, vae, device=dev, sp_group=sp_group)
    pipe.configure_runtime(offload=offload, prefetch=args.offload_prefetch)
    _log(f"offload={offload} prefetch={args.offload_prefetch}")
    return pipe


def dit_bytes(arch: dict, dtype) -> int:
    """Bytes of the DiT's weights in ``dtype`` (counted on the meta device, nothing allocated)."""
    from .models.transformer import PanVideoDiffusionTransformer
    with torch.device("meta"):
        m = PanVideoDiffusionTransformer(**arch)
    return sum(p.numel() for p in m.parameters()) * torch.empty(0, dtype=dtype).element_size()


def generate(args, sp_group=None, sp_rank: int = 0) -> List[str]:
    task = "i2v" if args.image_path else (args.task or "t2v")
    if args.task is not None and task != args.task:
        raise ValueError("--task t2v was given together with a reference image")
    jobs = prepare_jobs(args, task)
    if not jobs:
        _log("no pending prompts in this shard")
        return []
    pipe = build_pipeline(args, sp_group)
    written = []
    for k, job in enumerate(jobs, 1):
        ref_lat = None
        if job.task == "i2v" and str(job.image_path).endswith(".safetensors"):
            from .data.items import load_latent
            ref_lat = load_latent(job.image_path)[:, :1]
        out = pipe(prompt=job.prompt, negative_prompt=job.negative_prompt, video_length=job.video_length,
                   video_height=args.video_height, video_width=args.video_width,
                   num_inference_steps=job.num_inference_steps, guidance_scale=job.guidance_scale,
                   flow_shift=job.flow_shift, seed=args.seed,
                   reference_image=job.image_path if job.task == "i2v" and ref_lat is None else None,
                   reference_latents=ref_lat, i2v_skip_first_latent_cfg=job.i2v_skip_first_latent_cfg,
                   cfg_skip_interval=job.cfg_skip_interval, cfg_warmup_scale=job.cfg_warmup_scale,
                   timestep_schedule=job.timestep_schedule, first_step_velocity_scale=job.first_step_velocity_scale,
                   output_type=args.output_type, **{key: getattr(job, key) for key in GUIDANCE_KEYS})
        if sp_rank != 0:
            continue
        path = job.output_path or os.path.join("outputs", f"output_{MODEL_LABEL}_{datetime.datetime.now():%Y-%m-%d_%H-%M-%S}.mp4")
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        if out.videos is not None:
            target = write_video(out.videos, path, fps=args.fps, crf=args.video_crf, preset=args.video_preset,
                                 pix_fmt=args.video_pixel_format)
        else:
            from safetensors.torch import save_file
            target = os.path.splitext(path)[0] + ".latent.safetensors"
            save_file({"latent": out.latents[0].contiguous()}, target + ".partial")
            os.replace(target + ".partial", target)
            with open(path + ".partial", "wb") as f:  # placeholder so resume checks see a finished output
                f.write(b"latent-only output; see " + os.path.basename(target).encode())
            os.replace(path + ".partial", path)
        if args.save_settings:
            job.output_path = path
            save_settings(job, path, job.task)
        written.append(target)
        _log(f"completed {k}/{len(jobs)}: {target} (seed {out.seed})")
    return written


def build_arg_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Generate videos with a PAN 2 checkpoint")
    src = p.add_mutually_exclusive_group(required=True)
    src.add_argument("--prompt", type=str, nargs="+", help="text prompt(s)")
    src.add_argument("--prompt_json", help="T2V/I2V prompt-entry JSON")
    p.add_argument("--task", choices=["t2v", "i2v", "auto"], default=None)
    p.add_argument("--output_dir")
    p.add_argument("--image_root")
    p.add_argument("--prompt_shard_index", type=int, default=0)
    p.add_argument("--prompt_shard_count", type=int, default=1)
    p.add_argument("--skip_existing", type=str_to_bool, nargs="?", const=True, default=False)
    p.add_argument("--timestep_schedule", choices=["standard", "early_refine_2x"], default="standard")
    p.add_argument("--first_step_velocity_scale", type=float, default=1.0)
    p.add_argument("--cfg_start_step", type=int, default=0)
    p.add_argument("--cfg_end_step", type=int, default=None)
    p.add_argument("--cfg_warmup_scale", type=float, default=1.0)
    p.add_argument("--cfg_skip_interval", type=int, nargs=2, metavar=("START", "END"), default=None)
    p.add_argument("--i2v_skip_first_latent_cfg", type=str_to_bool, nargs="?", const=True, default=True)
    p.add_argument("--stg_scale", type=float, default=0.0)
    p.add_argument("--stg_skip_layers", type=int, nargs="+", default=None)
    p.add_argument("--video_crf", type=int, default=None)
    p.add_argument("--video_preset", default=None, choices=["ultrafast", "superfast", "veryfast", "faster", "fast",
                                                            "medium", "slow", "slower", "veryslow", "placebo"])
    p.add_argument("--video_pixel_format", choices=["yuv420p", "yuv444p"], default=None)
    p.add_argument("--negative_prompt", default="", type=str)
    p.add_argument("--negative_prompt_file", default=None, type=str)
    p.add_argument("--guidance_scale", default=None, type=float)
    p.add_argument("--flow_shift", default=None, type=float)
    p.add_argument("--video_height", default=704, type=int)
    p.add_argument("--video_width", default=1248, type=int)
    p.add_argument("--num_inference_steps", default=None, type=int)
    p.add_argument("--video_length", default=241, type=int)
    p.add_argument("--fps", default=24.0, type=float)
    p.add_argument("--offload", default="auto", choices=("auto", "none", "models", "blocks"),
                   help="none: every model on the GPU; models: text encoder, DiT and VAE wait on the CPU between "
                        "uses; blocks: also stream the DiT's blocks to the GPU while it runs; auto (default): blocks "
                        "only when the DiT's weights do not fit in free GPU memory, else none")
    p.add_argument("--offload_prefetch", default=True, type=str_to_bool, nargs="?", const=True,
                   help="with --offload blocks: copy the next block on a side stream while the current one runs")
    p.add_argument("--compile", default=False, type=str_to_bool, nargs="?", const=True,
                   help="accepted for command-line compatibility; the blocks already run hand-written kernels, "
                        "so there is nothing to compile")
    p.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    p.add_argument("--seed", default=42, type=int)
    p.add_argument("--image_path", default=None, type=str, nargs="+")
    p.add_argument("--output_path", default=None, type=str)
    p.add_argument("--save_settings", default=True, type=str_to_bool, nargs="?", const=True)
    p.add_argument("--checkpoint_path", default=None, type=str)
    p.add_argument("--training_config", default=None, type=str)
    p.add_argument("--transformer_config_overrides", default=None, type=str)
    p.add_argument("--text_encoder_hidden_state_skip_layer", default=2, type=int)
    p.add_argument("--text_encoder_max_length", default=None, type=int)
    p.add_argument("--wan_vae_checkpoint", default=None, type=str)
    p.add_argument("--sp_size", default=1, type=int, help="Ulysses sequence-parallel ranks per prompt")
    p.add_argument("--text_encoder", default="qwen", choices=["qwen", "hash"])
    p.add_argument("--text_encoder_path", default="Qwen/Qwen3.5-9B")
    p.add_argument("--output_type", default="video", choices=["video", "latent"])
    return p


def check_args(args, argv) -> None:
    validate_sampling_extensions(args.num_inference_steps or 50, args.timestep_schedule)
    if not 0 <= args.first_step_velocity_scale <= 1:
        raise ValueError("--first_step_velocity_scale is a factor between 0 and 1")
    if not 1.0 <= args.cfg_warmup_scale < float("inf"):
        raise ValueError("--cfg_warmup_scale must be a finite number no smaller than 1")
    if args.stg_scale == 0 and not any(a == "--stg_skip_layers" or a.startswith("--stg_skip_layers=") for a in argv):
        args.stg_skip_layers = None
    if args.skip_existing and (not args.save_settings or any(getattr(args, k) is None for k in
                                                            ("num_inference_steps", "flow_shift", "guidance_scale"))):
        raise ValueError("--skip_existing compares saved settings, so --num_inference_steps, --flow_shift and --guidance_scale must be given explicitly")
    if args.skip_existing and not (args.output_path or args.output_dir):
        raise ValueError("--skip_existing needs a fixed --output_path or --output_dir to look for finished videos")
    if args.video_crf is not None and not 0 <= args.video_crf <= 51:
        raise ValueError(f"--video_crf {args.video_crf} is outside the encoder's 0..51 range")
    if args.negative_prompt_file:
        if args.negative_prompt:
            raise ValueError("give the negative prompt once: --negative_prompt or --negative_prompt_file")
        with open(args.negative_prompt_file, encoding="utf-8") as f:
            args.negative_prompt = f.read().strip()
    read_training_config(args)
    if isinstance(args.image_path, list) and len(args.image_path) == 1 and args.image_path[0].strip().lower() == "none":
        args.image_path = None
    if args.video_height <= 0 or args.video_width <= 0 or args.fps <= 0:
        raise ValueError("--video_height, --video_width and --fps take positive values")
    for k, v in (("num_inference_steps", 50), ("flow_shift", 5.0), ("guidance_scale", 4.0)):
        if getattr(args, k) is None and not args.skip_existing:
            setattr(args, k, v)


def main(argv=None) -> List[str]:
    argv = sys.argv[1:] if argv is None else list(argv)
    args = build_arg_parser().parse_args(argv)
    check_args(args, argv)
    from .parallel.layout import init_parallel_layout
    L = init_parallel_layout(cp=args.sp_size)
    if torch.cuda.is_available():
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    # ranks of one sequence-parallel group share a prompt; groups shard the prompt list
    if L.dp_size > 1:
        if not args.prompt_json:
            raise ValueError(f"{L.world_size} ranks with --sp_size {args.sp_size}: direct --prompt inputs need "
                             "--sp_size equal to the number of ranks (or use --prompt_json)")
        if args.prompt_shard_count != 1:
            raise ValueError("with several ranks the prompts are sharded automatically; drop --prompt_shard_*")
        args.prompt_shard_index, args.prompt_shard_count = L.dp_rank, L.dp_size
    try:
        return generate(args, L.cp_group if args.sp_size > 1 else None, L.cp_rank)
    finally:
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
