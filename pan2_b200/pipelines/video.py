"""Text/image-to-video sampling with the MMDiT: packed CFG batches, Ulysses sequence parallel, Euler.

Behaviour of the reference pipeline (pan/pipelines/pan_video_pipeline.py:52-575), on this framework's
packed kernels:

* the negative and positive prompts of every video form ONE packed batch (``[neg_1..neg_B,
  pos_1..pos_B]``), each sample being the video tokens plus only its own valid caption tokens.  That is
  exactly the reference's padded ``[2B, ...]`` batch with a text mask (masked keys excluded, masked rows
  discarded) without computing the padding;
* the sampler state lives in token space (``[B, N, C*pt*ph*pw]``, the patchified latent): CFG, the
  i2v positive-only first latent frame, the first-step velocity scale and the fp32 Euler update are
  elementwise, so they give the same numbers as on ``[B, C, T, H, W]``, and no patchify runs per step;
* noise is drawn on the CPU from the seed (same video on any GPU count), in bf16 as the reference;
* with ``sp_size > 1`` each rank of the sequence-parallel group holds the full weights and its strided
  share of every sample's tokens; attention trades tokens for heads with the Ulysses all-to-all, and
  one all-gather of the velocity rows per step gives every rank the full prediction for the update;
* decoding (and image conditioning) go through a VAE object with ``encode_image`` / ``decode``
  (:mod:`pan2_b200.models.vae`); without one the pipeline returns latents.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..data.patching import packed_rope_tables, patchify, unpatchify
from ..inference.guidance import apply_guidance, resolve_guidance_plan, validate_sampling_extensions
from ..inference.scheduler import FlowEulerScheduler, apply_timestep_schedule
from ..models.packed import PackedSequenceParams, build_packed_params

WAN22_LATENT_CHANNELS = 48
WAN22_SPATIAL_STRIDE = 16
WAN22_TEMPORAL_STRIDE = 4


def latent_grid(num_frames: int, height: int, width: int, patch_size) -> Tuple[int, int, int]:
    """``(T, H, W)`` of the Wan latent of a ``num_frames x height x width`` video."""
    if height <= 0 or width <= 0:
        raise ValueError(f"height and width must be positive, got {height}x{width}")
    if height % WAN22_SPATIAL_STRIDE or width % WAN22_SPATIAL_STRIDE:
        raise ValueError(f"height and width ({height}x{width}) must both divide by {WAN22_SPATIAL_STRIDE}, the VAE's spatial stride")
    rows, cols = height // WAN22_SPATIAL_STRIDE, width // WAN22_SPATIAL_STRIDE
    ph, pw = tuple(patch_size)[-2:]
    if rows % ph or cols % pw:
        raise ValueError(f"the {rows}x{cols} latent of a {height}x{width} video does not tile into {(ph, pw)} patches")
    grid = ((num_frames - 1) // WAN22_TEMPORAL_STRIDE + 1, rows, cols)
    if min(grid) <= 0:
        raise ValueError(f"empty latent grid {grid} for {num_frames} frames at {height}x{width}")
    return grid


@dataclass
class _Plan:
    meta: PackedSequenceParams
    n_samples: int
    n_tokens: int
    idx_v: Optional[torch.Tensor] = None        # local video rows (sequence parallel)
    gather_src: Optional[torch.Tensor] = None   # rows of the all-gathered buffer that are real
    gather_dst: Optional[torch.Tensor] = None   # their positions in the full video block
    max_local: int = 0


class PackedDiTRunner:
    """Velocity predictions of the MMDiT for packed multi-sample batches (optionally sequence parallel)."""

    def __init__(self, model, device, sp_group=None):
        self.model = model
        self.device = torch.device(device)
        self.sp_group = sp_group
        self.sp = dist.get_world_size(sp_group) if sp_group is not None else 1
        self.sp_rank = dist.get_rank(sp_group) if sp_group is not None else 0
        self._plans: Dict[tuple, _Plan] = {}
        self.dtype = next(model.parameters()).dtype   # compute dtype of the model inputs

    def plan(self, grid: Tuple[int, int, int], caption_lens: Sequence[int]) -> _Plan:
        key = (tuple(grid), tuple(int(c) for c in caption_lens))
        p = self._plans.get(key)
        if p is not None:
            return p
        m = self.model
        pt, ph, pw = m.patch_size
        tok_grid = (grid[0] // pt, grid[1] // ph, grid[2] // pw)
        N = tok_grid[0] * tok_grid[1] * tok_grid[2]
        n = len(caption_lens)
        vlen, clen = [N] * n, [int(c) for c in caption_lens]
        total = sum(vlen) + sum(clen)
        if self.sp == 1:
            total = (total + 127) // 128 * 128
        axes, theta, scale = m.rope_settings()
        cos, sin = packed_rope_tables(axes, theta, scale, [tok_grid] * n, clen, total)
        meta = build_packed_params(vlen, clen, total, cos, sin).to(self.device)
        p = _Plan(meta=meta, n_samples=n, n_tokens=N)
        if self.sp > 1:
            from ..data.cp_batch import local_params, shard_rows
            p.meta, p.idx_v = local_params(meta, self.sp, self.sp_rank, self.sp_group, self.device)
            rows = [shard_rows(vlen, clen, self.sp, r)[0] for r in range(self.sp)]
            p.max_local = max(len(r) for r in rows)
            src, dst = [], []
            for r, rr in enumerate(rows):
                src += range(r * p.max_local, r * p.max_local + len(rr))
                dst += rr
            p.gather_src = torch.tensor(src, dtype=torch.long, device=self.device)
            p.gather_dst = torch.tensor(dst, dtype=torch.long, device=self.device)
        self._plans[key] = p
        return p

    @torch.no_grad()
    def predict(self, p: _Plan, x_tok: torch.Tensor, cond_tok: torch.Tensor, timesteps: torch.Tensor,
                text_rows: torch.Tensor, skip_layers: Sequence[int] = ()) -> torch.Tensor:
        """``x_tok`` ``[n_samples, N, Cp]`` and ``cond_tok`` ``[n_samples, N, Cp']`` -> velocity
        ``[n_samples, N, C_out*p]`` (bf16).  ``text_rows``: all samples' caption rows, packed."""
        n, N = p.n_samples, p.n_tokens
        dt = self.dtype
        rows = torch.cat([x_tok.to(dt), cond_tok.to(dt)], dim=-1).reshape(n * N, -1)
        if p.idx_v is not None:
            rows = rows.index_select(0, p.idx_v)
        hidden = rows.t()[:, :, None, None]
        pred = self.model.predict_packed(hidden, timesteps, text_rows, p.meta, skip_layers=tuple(skip_layers))
        if p.idx_v is not None:
            pred = self._gather(p, pred)
        return pred.reshape(n, N, -1)

    def _gather(self, p: _Plan, local: torch.Tensor) -> torch.Tensor:
        F = local.shape[1]
        buf = local.new_zeros(p.max_local, F)
        buf[:local.shape[0]] = local
        out = local.new_empty(self.sp * p.max_local, F)
        if local.is_cuda:
            dist.all_gather_into_tensor(out, buf, group=self.sp_group)
        else:
            dist.all_gather(list(out.chunk(self.sp)), buf, group=self.sp_group)
        full = local.new_empty(p.n_samples * p.n_tokens, F)
        full.index_copy_(0, p.gather_dst, out.index_select(0, p.gather_src))
        return full


@dataclass
class PipelineOutput:
    videos: Optional[torch.Tensor]              # [B, 3, F, H, W] in [0, 1] (CPU) when a VAE is present
    latents: torch.Tensor                       # [B, 48, T, H, W] fp32
    step_ms: List[float] = field(default_factory=list)
    seed: int = 0


class PanVideoPipeline:
    def __init__(self, transformer, text_encoder=None, vae=None, *, device="cuda", sp_group=None,
                 flow_shift: float = 5.0, guidance_scale: float = 4.0, num_inference_steps: int = 50):
        self.transformer = transformer.eval()
        self.text_encoder = text_encoder
        self.vae = vae
        self.device = torch.device(device)
        self.runner = PackedDiTRunner(transformer, self.device, sp_group)
        self.defaults = dict(flow_shift=flow_shift, guidance_scale=guidance_scale,
                             num_inference_steps=num_inference_steps)
        self.offload = "none"
        self._dit = transformer   # what moves between host and device in the models / blocks modes

    def configure_runtime(self, offload: str = "none", prefetch: bool = True) -> None:
        """Offloading, set once after construction (reference: pan_video_pipeline.py:111-158).

        ``none``: every model stays on the device.  ``models``: the text encoder, the DiT and the VAE
        wait on the CPU and each moves to the device only while it runs.  ``blocks``: as ``models``,
        and the DiT's blocks stay in host memory and are streamed to the device block by block
        while it runs (:class:`~pan2_b200.inference.offload.BlockStreamer`; ``prefetch`` overlaps
        the copy of the next block with the current one on a side stream)."""
        from ..inference.offload import OFFLOAD_MODES, NonBlockParts, enable_block_streaming
        if offload not in OFFLOAD_MODES:
            raise ValueError(f"offload must be one of {OFFLOAD_MODES}, got {offload!r}")
        if self.offload != "none":
            raise ValueError("configure_runtime runs once per pipeline")
        self.offload = offload
        if offload == "blocks":
            enable_block_streaming(self.transformer, self.device, prefetch=prefetch)
            self._dit = NonBlockParts(self.transformer)
        if offload != "none":  # every model waits on the CPU until it runs
            for m in (self.text_encoder, self._dit, self.vae):
                if m is not None and hasattr(m, "to"):
                    m.to(torch.device("cpu"))

    def _resident(self, *models):
        from ..inference.offload import resident
        return resident(self.offload != "none", self.device, *models)

    # ------------------------------------------------------------------ inputs
    def _caption_rows(self, texts: List[str]) -> List[torch.Tensor]:
        if self.text_encoder is None:
            raise ValueError("no text encoder: pass prompt_embeds / negative_prompt_embeds")
        emb, mask = self.text_encoder.encode(texts, device=self.device)
        lens = mask.sum(1).tolist()
        return [emb[i, :int(lens[i])] for i in range(len(texts))]

    def _condition(self, B: int, grid, image_latents: Optional[torch.Tensor]) -> torch.Tensor:
        """Patchified ``[cond (48) | mask (1)]`` tokens ``[B, N, 49*p]``."""
        T, H, W = grid
        cond = torch.zeros(B, WAN22_LATENT_CHANNELS + 1, T, H, W)
        if image_latents is not None:
            src = image_latents.float().cpu()
            if src.dim() == 4:
                src = src.unsqueeze(0)
            if src.shape[0] not in (1, B):
                raise ValueError(f"{src.shape[0]} reference latents for {B} prompts (give one, or one per prompt)")
            k = min(int(src.shape[2]), T)
            cond[:, :WAN22_LATENT_CHANNELS, :k] = src[:, :, :k].expand(B, -1, -1, -1, -1)
            cond[:, WAN22_LATENT_CHANNELS, :k] = 1.0
        ps = self.transformer.patch_size
        return torch.stack([patchify(cond[b], ps).t() for b in range(B)]).to(self.device, self.runner.dtype)

    # ------------------------------------------------------------------ sampling
    @torch.no_grad()
    def __call__(self, prompt=None, video_length: int = 121, num_inference_steps: Optional[int] = None,
                 guidance_scale: Optional[float] = None, negative_prompt=None, seed: Optional[int] = None,
                 flow_shift: Optional[float] = None, reference_image=None, reference_latents=None,
                 video_height: int = 704, video_width: int = 1248, cfg_start_step: int = 0,
                 cfg_end_step: Optional[int] = None, stg_scale: float = 0.0, stg_skip_layers=None,
                 i2v_skip_first_latent_cfg: bool = True, cfg_skip_interval=None, cfg_warmup_scale: float = 1.0,
                 timestep_schedule: str = "standard", first_step_velocity_scale: float = 1.0,
                 prompt_embeds: Optional[Sequence[torch.Tensor]] = None,
                 negative_prompt_embeds: Optional[Sequence[torch.Tensor]] = None, output_type: str = "video",
                 time_steps: bool = False) -> PipelineOutput:
        d = self.defaults
        guidance_scale = d["guidance_scale"] if guidance_scale is None else guidance_scale
        flow_shift = d["flow_shift"] if flow_shift is None else flow_shift
        steps = d["num_inference_steps"] if num_inference_steps is None else num_inference_steps
        i2v = reference_image is not None or reference_latents is not None
        if not isinstance(i2v_skip_first_latent_cfg, bool):
            raise ValueError("i2v_skip_first_latent_cfg takes True or False")
        if type(first_step_velocity_scale) not in (int, float) or not 0 <= first_step_velocity_scale <= 1:
            raise ValueError("first_step_velocity_scale must be finite and in [0, 1]")
        validate_sampling_extensions(steps, timestep_schedule)
        guided = (timestep_schedule != "standard" or cfg_start_step != 0 or cfg_end_step is not None
                  or stg_scale != 0 or stg_skip_layers is not None or cfg_skip_interval is not None
                  or cfg_warmup_scale != 1.0 or first_step_velocity_scale != 1.0)
        if guided:
            if not guidance_scale > 1:
                raise ValueError("guidance controls require guidance_scale > 1")
            if stg_scale != 0 and i2v:
                raise ValueError("STG supports T2V only")
        if stg_scale == 0 and stg_skip_layers is not None:
            raise ValueError("stg_skip_layers has no effect unless stg_scale is positive")
        use_cfg = guidance_scale > 1

        # ---- text
        encode = prompt_embeds is None or (use_cfg and negative_prompt_embeds is None)
        with self._resident(self.text_encoder if encode else None):
            if prompt_embeds is not None:
                pos = [t.to(self.device) for t in prompt_embeds]
            else:
                prompts = [prompt] if isinstance(prompt, str) else list(prompt)
                pos = self._caption_rows(prompts)
            B = len(pos)
            neg = []
            if use_cfg:
                if negative_prompt_embeds is not None:
                    neg = [t.to(self.device) for t in negative_prompt_embeds]
                else:
                    negs = (list(negative_prompt) if isinstance(negative_prompt, (list, tuple))
                            else [negative_prompt or ""] * B)
                    if len(negs) != B:
                        raise ValueError(f"got {len(negs)} negative prompts for {B} prompts")
                    neg = self._caption_rows(negs)
                if len(neg) != B:
                    raise ValueError("one negative embedding per prompt is required")
        samples = neg + pos
        dt = self.runner.dtype
        text_rows = torch.cat([t.to(dt) for t in samples], 0)

        # ---- schedule and guidance
        sched = FlowEulerScheduler(shift=flow_shift)
        sched.set_timesteps(steps, device=self.device)
        timesteps = apply_timestep_schedule(sched, timestep_schedule)
        plan = resolve_guidance_plan(len(timesteps), start_step=cfg_start_step, end_step=cfg_end_step,
                                     stg_scale=stg_scale, skip_interval=cfg_skip_interval,
                                     warmup_scale=cfg_warmup_scale)
        skip = ()
        if plan.stg_scale:
            self.transformer.eval()
            skip = self.transformer.validate_stg_layers(stg_skip_layers)

        # ---- latents, condition
        if int(self.transformer.in_channels) != 2 * WAN22_LATENT_CHANNELS + 1:
            # the sampler feeds [noisy latent | condition | condition mask] (reference:
            # pan_video_pipeline.py:356-359): a token_concat-trained transformer does not fit it
            raise ValueError(f"sampling needs a {2 * WAN22_LATENT_CHANNELS + 1}-channel (channel_concat) "
                             f"transformer, got in_channels={self.transformer.in_channels}")
        grid = latent_grid(video_length, video_height, video_width, self.transformer.patch_size)
        if seed in (None, -1):
            seed = random.randint(100000, 999999)
        gen = torch.Generator().manual_seed(int(seed))
        noise = torch.randn((B, WAN22_LATENT_CHANNELS, *grid), generator=gen, dtype=torch.bfloat16)
        ps = self.transformer.patch_size
        x = torch.stack([patchify(noise[b], ps).t() for b in range(B)]).to(self.device)   # [B, N, 48p] bf16
        if reference_image is not None and reference_latents is None:
            if self.vae is None:
                raise ValueError("image conditioning needs a VAE (or pass reference_latents)")
            with self._resident(self.vae):
                reference_latents = self.vae.encode_image(reference_image, video_height, video_width)
        cond = self._condition(B, grid, reference_latents if i2v else None)
        runner = self.runner
        n_samp = len(samples)
        p = runner.plan(grid, [int(t.shape[0]) for t in samples])
        p_pos = runner.plan(grid, [int(t.shape[0]) for t in pos]) if plan.stg_scale else None
        cond_all = cond.repeat(2, 1, 1) if use_cfg else cond
        frame0 = (grid[1] // ps[1]) * (grid[2] // ps[2])  # tokens of latent frame 0 (temporal patch 1)
        step_ms = []
        with self._resident(self._dit):
            for i, t in enumerate(timesteps):
                if time_steps and self.device.type == "cuda":
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                x_in = x.repeat(2, 1, 1) if use_cfg else x
                tb = t.reshape(1).expand(n_samp).float()
                v = runner.predict(p, x_in, cond_all, tb, text_rows)
                if use_cfg:
                    v_neg, v_pos = v[:B], v[B:]
                    if guided:
                        def weak():
                            return runner.predict(p_pos, x, cond, tb[:B], torch.cat([r.to(dt) for r in pos]),
                                                  skip_layers=skip)
                        v = apply_guidance(v_neg, v_pos, guidance_scale, step_index=i, plan=plan, weak_predict_fn=weak)
                    else:
                        v = v_neg + guidance_scale * (v_pos - v_neg)
                    if i2v and i2v_skip_first_latent_cfg and plan.active(i):
                        v = v.clone()
                        v[:, :frame0] = v_pos[:, :frame0]
                if i == 0 and first_step_velocity_scale != 1.0:
                    v = v * first_step_velocity_scale
                x = sched.step(v, t, x)
                if time_steps and self.device.type == "cuda":
                    e1.record()
                    e1.synchronize()
                    step_ms.append(e0.elapsed_time(e1))
        lat = torch.stack([unpatchify(x[b].float(), tuple(s // q for s, q in zip(grid, ps)), ps, WAN22_LATENT_CHANNELS)
                           for b in range(B)])
        videos = None
        if output_type == "video":
            if self.vae is None:
                raise ValueError("no VAE: use output_type='latent'")
            with self._resident(self.vae):
                videos = self.vae.decode(lat)
        return PipelineOutput(videos=videos, latents=lat, step_ms=step_ms, seed=int(seed))


def build_inference_model(arch: dict, device, dtype=torch.bfloat16, seed: int = 0):
    """The MMDiT in ``dtype`` on ``device``, materialised block by block (random init, seeded)."""
    from ..models.transformer import JointAttentionBlock, PanVideoDiffusionTransformer
    device = torch.device(device)
    with torch.device("meta"):
        model = PanVideoDiffusionTransformer(**arch)
    blk_opts = dict(attention_backend=model.attention_backend, mlp_ratio=arch.get("mlp_ratio", 8.0),
                    context_mlp_ratio=arch.get("context_mlp_ratio", 4.0),
                    zero_init_modulation=arch.get("zero_init_modulation", True),
                    text_modulation_timestep_dependent=arch.get("text_modulation_timestep_dependent", False))
    for i in range(len(model.blocks)):
        torch.manual_seed(seed * 1000003 + i)
        with torch.device(device):
            blk = JointAttentionBlock(model.hidden_size, model.num_attention_heads, **blk_opts)
        model.blocks[i] = blk.to(dtype)
    torch.manual_seed(seed * 1000003 + len(model.blocks))
    with torch.device(device):
        small = PanVideoDiffusionTransformer(**{**arch, "num_layers": 0})
    for name, child in small.named_children():
        if name != "blocks":
            setattr(model, name, child.to(dtype))
    return model.eval()


def load_transformer_weights(model, path: str, strict: bool = True) -> List[str]:
    """Load weights from a sharded training checkpoint, consolidated safetensors shards, a single
    safetensors file or a plain ``.pt`` state dict; block by block, so host memory stays bounded.
    Legacy per-modality block keys are converted by the block's own state-dict hook."""
    from ..checkpoint.io import LazyStateDict
    sd = LazyStateDict(path)
    keys = list(sd.keys())
    missing = []
    for i, blk in enumerate(model.blocks):
        pre = f"blocks.{i}."
        sub = {k[len(pre):]: sd.get(k) for k in keys if k.startswith(pre)}
        res = blk.load_state_dict(sub, strict=False)
        missing += [pre + k for k in res.missing_keys]
    root = {k: sd.get(k) for k in keys if not k.startswith("blocks.")}
    own = {k: v for k, v in model.state_dict().items() if not k.startswith("blocks.")}
    for k, v in own.items():
        if k in root:
            v.copy_(root[k].to(v.dtype))
        else:
            missing.append(k)
    missing = [m for m in missing if not m.endswith("freqs")]
    if strict and missing:
        raise ValueError(f"{len(missing)} transformer tensors absent from {path} (first: {missing[:5]})")
    return missing
