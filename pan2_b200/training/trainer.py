"""The training loop: data, steps, logging, checkpoints, resume, anomaly recovery, heartbeat.

Behaviour of the reference's PanVideoTrainer (train.py:461-1729) on this framework's engine:

* one process per GPU; the process groups come from :func:`init_parallel_layout` (dp x cp, with the
  shard group within a node under ``hybrid_shard``);
* every data-parallel rank streams its own slice of the video CSVs (``csv[dp_rank::dp_size]``; fewer
  CSVs than ranks is an error) and of the image tar shards, packs them under the token budgets and
  assembles batches on its GPU; with context parallelism only cp-rank 0 loads and the batch is
  broadcast and split across the cp group (:mod:`pan2_b200.data.cp_batch`);
* a step is forward + backward over ``gradient_accumulation_steps`` micro-batches, the global norm and
  clip coefficient, a cross-rank vote that the update is finite, the optimizer (skipped when not),
  and the LR schedule (:class:`~pan2_b200.training.step.StepRunner`);
* log line ``Step N/M | Loss: ... | Grad Norm: ... | LR: ... | CPU Wall: ... | (Prev Step CUDA) Data:
  ... | Train: ... | Elapsed: ...`` on rank 0 every ``log_interval`` steps;
* skipped non-finite steps are counted; anomalies (see :class:`AnomalyDetector`) roll back to the latest
  checkpoint unless the update was skipped and fewer than ``max_consecutive_skipped_steps`` skips ran;
* ``checkpoint-<step>/`` every ``save_interval`` steps and at the end, with retention
  (``save_total_limit``) and a ``save_logging/checkpoint_<step>.txt`` record; resume from the latest
  complete checkpoint, falling back to the one before it; warm start (weights only) from
  ``pretrained_transformer_path`` while ``output_dir`` has no checkpoint of its own;
* the heartbeat watchdog, NVTX ranges, and ``cudaProfilerStart`` after ``profile_step``.
"""
from __future__ import annotations

import glob
import json
import logging
import os
import random
import sys
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Dict, Iterator, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..checkpoint import io as ckpt
from ..config.training import TrainingConfig
from ..data.items import Budgets, CaptionCodec, HashCaptionCodec
from ..data.loader import LoaderMeta, PackedLoader
from ..data.packing import DataloaderState, PackingDataset, expand_csv_paths, expand_tar_paths
from ..models.transformer import ARCH_DEFAULTS, translate_architecture_config
from ..optim.lr import make_lr_lambda
from ..parallel.layout import ParallelLayout, init_parallel_layout
from .engine import OptimConfig, TrainEngine
from .fault import AnomalyDetector, FaultInjector, Heartbeat
from .step import StepRunner

IMAGE_TAR_SHUFFLE_SEED = 1234
WAN22_SPATIAL_RATIO = 16
WAN22_LATENT_CHANNELS = 48

log = logging.getLogger("pan2_b200.train")


def configure_logging(rank: int) -> None:
    fmt = logging.Formatter(f"%(asctime)s | %(levelname)-7s | rank{rank} | %(message)s", "%Y-%m-%d %H:%M:%S")
    h = logging.StreamHandler(sys.stdout)
    h.setFormatter(fmt)
    log.handlers[:] = [h]
    log.setLevel(logging.INFO if rank == 0 else logging.WARNING)
    log.propagate = False


def format_duration(seconds: float) -> str:
    s = int(seconds)
    d, s = divmod(s, 86400)
    h, s = divmod(s, 3600)
    m, s = divmod(s, 60)
    return (f"{d}d " if d else "") + f"{h:02d}:{m:02d}:{s:02d}"


@contextmanager
def nvtx(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def build_caption_codec(cfg: TrainingConfig, device, embed_dim: int = 4096) -> CaptionCodec:
    """``hash``: the offline stand-in, with the model's caption embedding width; otherwise the Qwen
    caption encoder at ``text_encoder_path``."""
    if cfg.text_encoder == "hash":
        return HashCaptionCodec(embed_dim=int(embed_dim))
    from ..models.text_encoder import QwenCaptionCodec
    return QwenCaptionCodec(cfg.text_encoder_path, device=device,
                            hidden_state_skip_layer=cfg.text_encoder_hidden_state_skip_layer)


def architecture_from_config(cfg: TrainingConfig) -> dict:
    """The transformer architecture of a run: the defaults, the YAML overrides, and the input /
    output widths the conditioning schema implies (reference: train.py:572-601)."""
    over = translate_architecture_config(cfg.transformer_config_overrides or {})
    if "zero_init_modulation" in over and bool(over["zero_init_modulation"]) != bool(cfg.zero_init_modulation):
        log.warning(f"transformer_config_overrides['zero_init_modulation'] ({over['zero_init_modulation']}) is "
                    f"overridden by the config's zero_init_modulation ({cfg.zero_init_modulation})")
    schema = getattr(cfg.conditioning_schema, "value", cfg.conditioning_schema)
    # channel_concat: [noised (48) | clean condition (48) | mask (1)]; token_concat: the noised latent
    expected = {"in_channels": 2 * WAN22_LATENT_CHANNELS + 1 if schema == "channel_concat" else WAN22_LATENT_CHANNELS,
                "out_channels": WAN22_LATENT_CHANNELS}
    for key, want in expected.items():
        if key in over and int(over[key]) != want:
            raise ValueError(f"transformer_config_overrides.{key}={over[key]} does not fit {schema} "
                             f"conditioning of Wan 2.2 latents, which needs {want}")
    arch = dict(ARCH_DEFAULTS)
    arch.update(over)
    arch.update(expected)
    arch["zero_init_modulation"] = bool(cfg.zero_init_modulation)
    return arch


class Trainer:
    def __init__(self, cfg: TrainingConfig, *, codec: Optional[CaptionCodec] = None,
                 layout: Optional[ParallelLayout] = None):
        self.cfg = cfg
        self.layout = layout or init_parallel_layout(cfg.cp_size, cfg.hybrid_shard, cfg.process_group_timeout_s)
        L = self.layout
        self.rank, self.world = L.rank, L.world_size
        self.is_main = self.rank == 0
        configure_logging(self.rank)
        if torch.cuda.is_available():
            self.device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")
        self.arch = architecture_from_config(cfg)
        self.codec = codec
        optim = OptimConfig(lr=cfg.learning_rate, weight_decay=cfg.weight_decay, use_muon=cfg.use_muon,
                            max_grad_norm=cfg.max_grad_norm)
        act = int(cfg.activation_reserve_gb * 1e9)
        self.engine = TrainEngine(self.arch, self.device, group=L.shard_group if self.world > 1 else None,
                                  seed=cfg.seed, optim=optim, offload=cfg.optimizer_offload,
                                  activation_bytes_estimate=act, replicate_group=L.replicate_group)
        self.engine.set_activation_checkpointing(cfg.enable_gradient_checkpointing,
                                                 cfg.use_dedicated_gradient_checkpointing)
        if cfg.cp_size > 1:
            self.engine.set_context_parallel(L.cp_group, L.cp_size, L.cp_rank)
        self.engine.set_accumulation(cfg.gradient_accumulation_steps)
        self.lr_lambda = make_lr_lambda(cfg.lr_scheduler_type, cfg.warmup_steps, cfg.lr_decay_steps, cfg.max_steps,
                                        cfg.lr_warmup_start_ratio, cfg.lr_decay_floor_ratio)
        self.runner = StepRunner(self.engine, self.lr_lambda, base_lr=cfg.learning_rate, cpu_group=L.cpu_group)
        self.global_step = 0
        self.resume_dataloader_state: Optional[DataloaderState] = None
        self.last_dataloader_state: Optional[DataloaderState] = None
        self.detector = AnomalyDetector(warmup_steps=cfg.anomaly_detection_warmup_steps, group=L.cpu_group)
        self.injector = FaultInjector(cfg.fault_injection, rank=self.rank)
        self.consecutive_skipped = 0
        self.total_skipped = 0
        self.recoveries = 0
        self.util: Dict[str, Optional[float]] = dict(seq=None, image=None, joint=None, video=None, caption=None)
        self.history: List[Dict] = []
        self.heartbeat: Optional[Heartbeat] = None
        self.wandb = None
        if cfg.report_to == "wandb" and self.is_main:
            try:
                import wandb
                wandb.init(project=os.environ.get("WANDB_PROJECT", "pan2_b200"), config=vars(cfg))
                self.wandb = wandb
            except Exception as e:  # not installed / no credentials: keep training, say so once
                log.warning(f"report_to=wandb but wandb is unavailable ({e}); metrics go to the log only")
        if self.is_main:
            log.info(f"model: {self.engine.total_params / 1e9:.2f}B parameters, world {self.world} "
                     f"(dp {L.dp_size} x cp {L.cp_size}, shard {L.shard_size}), device {self.device}, "
                     f"optimizer state offload: {self.engine.offload}")

    # ------------------------------------------------------------------ data
    def build_dataset(self, resume: Optional[DataloaderState]) -> PackingDataset:
        cfg, L = self.cfg, self.layout
        csvs = sorted(expand_csv_paths(cfg.packed_dataloader_meta_csv_path or []))
        if len(csvs) < L.dp_size:
            msg = (f"{L.dp_size} data-parallel ranks read whole CSV files, but packed_dataloader_meta_csv_path "
                   f"lists only {len(csvs)}: {L.dp_size - len(csvs)} rank(s) would have no data.  Provide at least "
                   f"{L.dp_size} CSV files, or run fewer data-parallel ranks (fewer GPUs or a larger cp_size).")
            raise ValueError(msg)
        csvs = csvs[L.dp_rank::L.dp_size]
        tars: List[str] = []
        if cfg.image_tar_path and cfg.image_sample_prob > 0:
            tars = expand_tar_paths(cfg.image_tar_path)
            random.Random(IMAGE_TAR_SHUFFLE_SEED).shuffle(tars)
            tars = tars[L.dp_rank::L.dp_size]
        pt, ph, pw = self.arch["patch_size"]
        if cfg.video_height % WAN22_SPATIAL_RATIO or cfg.video_width % WAN22_SPATIAL_RATIO:
            raise ValueError(f"video size {cfg.video_height}x{cfg.video_width} is not a multiple of the VAE's "
                             f"spatial ratio {WAN22_SPATIAL_RATIO}")
        if pt != 1:
            raise ValueError("packed training needs a temporal patch size of 1")
        lat_h, lat_w = cfg.video_height // WAN22_SPATIAL_RATIO, cfg.video_width // WAN22_SPATIAL_RATIO
        if lat_h % ph or lat_w % pw:
            raise ValueError(f"latent grid {(lat_h, lat_w)} of {cfg.video_height}x{cfg.video_width} video is not "
                             f"divisible by the transformer patch size {tuple(self.arch['patch_size'])}")
        budgets = Budgets(joint=cfg.packed_joint_token_budget, video=cfg.packed_video_token_budget,
                          caption=cfg.packed_caption_token_budget,
                          text_encoder=cfg.packed_caption_token_budget + 64 * cfg.packed_dataloader_max_num_seq,
                          joint_segment=cfg.packed_joint_segment_limit,
                          caption_segment=cfg.packed_caption_segment_limit,
                          max_num_seq=cfg.packed_dataloader_max_num_seq)
        if self.codec is None:
            self.codec = build_caption_codec(cfg, self.device, embed_dim=self.arch["text_embed_dim"])
        return PackingDataset(csvs, self.codec, budgets, patch_size=self.arch["patch_size"],
                              rope_axes=tuple(self.arch["rope_axes_dim"]), rope_theta=float(self.arch["rope_theta"]),
                              rope_scale=(float(self.arch["rope_temporal_scale"]), 1.0, 1.0),
                              num_buffers=cfg.packed_dataloader_num_buffers, seed=cfg.seed + L.dp_rank,
                              image_tars=tars, image_sample_prob=cfg.image_sample_prob,
                              video_cond_prob=cfg.video_cond_prob, image_cond_prob=cfg.image_cond_prob,
                              cfg_drop_prob=cfg.cfg_drop_prob, num_workers=min(cfg.packed_dataloader_num_workers, 64),
                              resume=resume)

    def build_loader(self, resume: Optional[DataloaderState]) -> PackedLoader:
        cfg = self.cfg
        ds = self.build_dataset(resume)
        return PackedLoader(ds, device=self.device, dtype=torch.bfloat16 if cfg.dtype == "bf16" else torch.float32,
                            prefetch=cfg.packed_dataloader_prefetch_factor,
                            seed=cfg.seed + 7919 * self.layout.dp_rank,
                            start_index=self.global_step * cfg.gradient_accumulation_steps,
                            T=cfg.num_train_timesteps, timestep_distribution=str(cfg.snr_type.value),
                            timestep_loc=cfg.flow_lognorm_loc, timestep_scale=cfg.flow_lognorm_scale,
                            shift=cfg.train_timestep_shift, shift_mode=str(cfg.train_timestep_shift_mode.value),
                            shift_kwargs=dict(rescale_factor=cfg.train_timestep_rescale_factor,
                                              max_shift=cfg.train_timestep_max_shift),
                            conditioning_schema=str(getattr(cfg.conditioning_schema, "value", cfg.conditioning_schema)))

    # ------------------------------------------------------------------ checkpoints
    def checkpoint_dir(self, step: int) -> str:
        return os.path.join(self.cfg.output_dir, f"checkpoint-{step}")

    def _barrier(self):
        if self.world > 1:
            dist.barrier(group=self.layout.cpu_group)

    def save_checkpoint(self) -> str:
        if self.device.type == "cuda":
            self._check_device_errors()  # never mark a checkpoint complete over incomplete kernel output
        step = self.global_step
        root = self.checkpoint_dir(step)
        if self.is_main:
            os.makedirs(root, exist_ok=True)
            ckpt.clear_complete(root)  # a folder being rewritten (after a rollback) is incomplete until done
        self._barrier()
        ckpt.save_engine(self.engine, root, group=self.layout.cpu_group if self.world > 1 else None)
        _, _, state_file = ckpt.checkpoint_layout(root)
        if self.is_main:
            torch.save({"lr_schedulers": {"transformer": self.runner.state_dict()}, "global_step": step,
                        "skipped_steps": self.total_skipped}, state_file)
        if self.last_dataloader_state is not None and self.layout.cp_rank == 0:
            d = os.path.join(root, "dataloader")
            os.makedirs(d, exist_ok=True)
            Path(d, f"{self.layout.dp_rank}.json").write_text(self.last_dataloader_state.to_json())
        self._barrier()
        if self.is_main:
            ckpt.mark_complete(root, step)
            rec = os.path.join(self.cfg.output_dir, "save_logging")
            os.makedirs(rec, exist_ok=True)
            with open(os.path.join(rec, f"checkpoint_{step}.txt"), "a") as f:
                f.write(f"{step}: {root}\n")
            removed = ckpt.cleanup_old(self.cfg.output_dir, self.cfg.save_total_limit)
            for r in removed:
                log.info(f"removed old checkpoint {r}")
            log.info(f"Step {step}: checkpoint written to {root}")
        self._barrier()
        return root

    def _load_checkpoint(self, root: str, load_dataloader_state: bool) -> None:
        if not ckpt.is_complete(root):
            raise ValueError(f"{root} is incomplete (no {ckpt.COMPLETE} marker)")
        ckpt.load_engine(self.engine, root, load_optimizer=True, strict=True)
        _, _, state_file = ckpt.checkpoint_layout(root)
        st = torch.load(state_file, map_location="cpu", weights_only=False)
        self.runner.load_state_dict(st["lr_schedulers"]["transformer"])
        self.global_step = int(st["global_step"])
        self.runner.global_step = self.global_step
        if load_dataloader_state:
            p = os.path.join(root, "dataloader", f"{self.layout.dp_rank}.json")
            if not os.path.exists(p):
                raise ValueError(f"{p} does not exist: {root} was saved by a run with a different number of "
                                 f"data-parallel ranks than this one (rank {self.layout.dp_rank})")
            self.resume_dataloader_state = DataloaderState.from_json(Path(p).read_text())
            if not self.cfg.resume_video_csv:
                self.resume_dataloader_state = self.resume_dataloader_state.reset_video_stream()
                log.info("resume_video_csv=false: video CSV stream reset; image-tar cursor kept")

    def load_checkpoint(self, load_dataloader_state: bool = True) -> Optional[str]:
        """Resume from the latest complete checkpoint, falling back to the one before it."""
        every = ckpt.list_checkpoints(self.cfg.output_dir)
        cks = [(s, d) for s, d in every if ckpt.is_complete(d)]
        skipped = [d for s, d in every if not ckpt.is_complete(d) and (not cks or s > cks[-1][0])]
        if skipped:
            log.warning(f"skipping incomplete checkpoint folder(s) {skipped} (interrupted saves)")
        if not cks:
            if every:
                raise ValueError(f"no complete checkpoint in {self.cfg.output_dir}: {[d for _, d in every]} "
                                 f"all lack the {ckpt.COMPLETE} marker")
            return None
        last = cks[-1][1]
        prev = cks[-2][1] if len(cks) > 1 else None
        try:
            self._load_checkpoint(last, load_dataloader_state)
            used = last
        except Exception as e1:
            if prev is None:
                raise ValueError(f"failed to load checkpoint {last}: {e1}; no earlier checkpoint") from e1
            log.warning(f"latest checkpoint {last} unreadable ({e1}); trying {prev}")
            try:
                self._load_checkpoint(prev, load_dataloader_state)
                used = prev
            except Exception as e2:
                raise ValueError(f"failed to load checkpoint: {e1} for {last}, {e2} for {prev}") from e2
        log.info(f"resumed from {used} at step {self.global_step}")
        return used

    def warm_start(self, path: str) -> None:
        if os.path.isdir(path) and (os.path.exists(os.path.join(path, "transformer", "meta.json"))
                                    or os.path.exists(os.path.join(path, "meta.json"))):
            root = path if os.path.exists(os.path.join(path, "transformer")) else os.path.dirname(path.rstrip("/"))
            ckpt.load_engine(self.engine, root, load_optimizer=False, strict=True)
        else:
            ckpt.load_plain_into_engine(self.engine, path, strict=True)
        log.info(f"warm start from {path}: transformer weights only")

    def _check_device_errors(self) -> None:
        """Stop the run when a kernel gave up a bounded wait (a peer that never arrived, a copy
        that never landed): its outputs are incomplete, so continuing would train on them, and a
        checkpoint written afterwards would be marked complete over bad state.  Every rank reads its
        flag and the ranks agree on the largest code (one small all-reduce over the host group), so
        all of them stop together instead of the others waiting in their next collective."""
        from ..ops._ext import ext
        flag = int(ext().error_flag(True))
        if self.world > 1:
            t = torch.tensor([flag], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.layout.cpu_group)
            flag = int(t.item())
        if flag:
            raise RuntimeError(f"device error code {flag} after step {self.global_step - 1}: a kernel stopped "
                               "waiting (peer rank gone or stalled, or a transfer that never completed)")

    def recover(self) -> None:
        log.warning("recovering from the latest checkpoint")
        used = self.load_checkpoint(load_dataloader_state=False)
        if used is None:
            raise ValueError("no checkpoint found for recovery")
        self.detector.reset()
        self.consecutive_skipped = 0
        self.recoveries += 1
        log.warning(f"recovery complete from {used}")

    # ------------------------------------------------------------------ metrics
    def _update_util(self, meta: LoaderMeta) -> None:
        vals = dict(seq=meta.active_sequence_count, image=meta.active_image_count, joint=meta.active_joint_length,
                    video=meta.active_video_length, caption=meta.active_caption_length)
        for k, v in vals.items():
            cur = self.util[k]
            self.util[k] = float(v) if cur is None else 0.99 * cur + 0.01 * float(v)

    def log_packing_utilization(self) -> None:
        if self.util["seq"] is None:
            return
        buf = torch.tensor([self.util[k] for k in ("seq", "image", "joint", "video", "caption")], dtype=torch.float64)
        if self.world > 1:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.layout.cpu_group)
            buf /= self.world
        seq, image, joint, video, caption = buf.tolist()
        c = self.cfg
        log.info(f"(avg) sequence count: {seq:5.2f} (image: {image:5.2f}, video: {seq - image:5.2f}); "
                 f"joint: {joint:5.0f}/{c.packed_joint_token_budget:5} = {joint / c.packed_joint_token_budget * 100:2.0f}%; "
                 f"video/image: {video:5.0f}/{c.packed_video_token_budget:5} = "
                 f"{video / c.packed_video_token_budget * 100:2.0f}%; "
                 f"caption: {caption:4.0f}/{c.packed_caption_token_budget:4} = "
                 f"{caption / c.packed_caption_token_budget * 100:2.0f}%")

    # ------------------------------------------------------------------ loop
    def _next_batches(self, it: Iterator) -> Tuple[list, Optional[LoaderMeta]]:
        out, meta = [], None
        for _ in range(self.cfg.gradient_accumulation_steps):
            if self.layout.cp_enabled:
                from ..data.cp_batch import broadcast_and_split
                b, m = next(it) if it is not None else (None, None)
                b, m = broadcast_and_split(b, m, self.layout, self.device)
            else:
                b, m = next(it)
            out.append(b)
            if m is not None:
                meta = m
        return out, meta

    def train(self) -> List[Dict]:
        cfg = self.cfg
        resumed = self.load_checkpoint()
        if cfg.load_transformer_weights and cfg.pretrained_transformer_path:
            if resumed is None:
                self.warm_start(cfg.pretrained_transformer_path)
            else:
                log.info(f"resumed from {resumed}: {cfg.output_dir} holds checkpoints, so the warm start is skipped")
        self._barrier()
        if self.is_main:
            log.info(f"Training for {cfg.max_steps} steps: batch_size={cfg.batch_size} (packed batches are sized "
                     f"by the token budgets) lr={cfg.learning_rate} weight_decay={cfg.weight_decay} "
                     f"zero_init_modulation={cfg.zero_init_modulation} activation_checkpointing="
                     f"{'kept-attention' if self.engine.keep_attention else cfg.enable_gradient_checkpointing}")
        loader = None
        it = None
        if not self.layout.cp_enabled or self.layout.cp_rank == 0:
            loader = self.build_loader(self.resume_dataloader_state)
            it = iter(loader)
        self.heartbeat = Heartbeat(self.rank, cfg.heartbeat_timeout_s).start()
        t0 = prev = time.perf_counter()
        cuda = self.device.type == "cuda"
        mk = (lambda: torch.cuda.Event(enable_timing=True)) if cuda else (lambda: None)
        ev = {k: mk() for k in ("pre", "post", "step", "pre2", "post2", "step2")}
        if cuda:
            for k in ("pre2", "post2", "step2"):
                ev[k].record()
        try:
            while self.global_step < cfg.max_steps:
                self.heartbeat.beat("dataloader_next", self.global_step)
                with nvtx("dataloader_next"):
                    if cuda:
                        ev["pre"].record()
                    batches, meta = self._next_batches(it)
                    if meta is not None and meta.dataloader_state is not None:
                        self.last_dataloader_state = meta.dataloader_state
                    if cuda:
                        ev["post"].record()
                self.heartbeat.beat("train_step")
                self.injector.before_step(self.global_step)
                with nvtx("train_step"):
                    stats = self.runner.device_step(batches, poison=self.injector.poisons_update(self.global_step))
                stats = self.injector.after_step(self.global_step, stats)
                if cuda:  # every step: the flag read is one small device-to-host copy
                    self._check_device_errors()
                if meta is not None:
                    self._update_util(meta)
                if cuda:
                    ev["step"].record()
                now = time.perf_counter()
                wall, prev = now - prev, now
                data_t = train_t = 0.0
                if cuda and ev["post2"].query() and ev["step2"].query():
                    data_t = ev["pre2"].elapsed_time(ev["post2"]) / 1000
                    train_t = ev["post2"].elapsed_time(ev["step2"]) / 1000
                if self.global_step % cfg.log_interval == 0:
                    log.info(" | ".join([f"Step {self.global_step}/{cfg.max_steps}", f"Loss: {stats['loss']:.6f}",
                                         f"Grad Norm: {stats['grad_norm']:.4f}", f"LR: {stats['lr']:.2e}",
                                         f"CPU Wall: {wall:.3f}s", f"(Prev Step CUDA) Data: {data_t:.3f}s",
                                         f"Train: {train_t:.3f}s", f"Elapsed: {format_duration(now - t0)}"]))
                self.history.append(dict(step=self.global_step, **stats))
                if self.wandb is not None and self.global_step % cfg.log_interval == 0:
                    self.wandb.log({"train/loss": stats["loss"], "train/grad_norm": stats["grad_norm"],
                                    "train/lr": stats["lr"]}, step=self.global_step)
                if stats["step_skipped"]:
                    self.consecutive_skipped += 1
                    self.total_skipped += 1
                    log.warning(f"step {self.global_step}: update not applied, loss {stats['loss']} / grad norm "
                                f"{stats['grad_norm']} not finite ({self.consecutive_skipped} in a row, "
                                f"{self.total_skipped} so far)")
                else:
                    self.consecutive_skipped = 0
                self.global_step += 1
                self.heartbeat.beat("post_step", self.global_step)
                recover = cfg.anomaly_detection and self.detector(self.global_step, stats["loss"], stats["grad_norm"])
                if recover and self.detector.last_reasons:
                    log.error(f"anomaly at step {self.global_step} on rank {self.rank}: "
                              + "; ".join(self.detector.last_reasons))
                if (recover and stats["step_skipped"]
                        and self.consecutive_skipped <= cfg.max_consecutive_skipped_steps):
                    recover = False
                    log.warning("not recovering: the anomalous update was skipped, so the training state is clean "
                                f"({self.consecutive_skipped}/{cfg.max_consecutive_skipped_steps} consecutive skips)")
                if recover:
                    self.heartbeat.beat("recover_from_checkpoint")
                    if cuda:
                        self._check_device_errors()
                    self.recover()
                elif self.global_step % cfg.save_interval == 0:
                    self.heartbeat.beat("save_checkpoint")
                    self.log_packing_utilization()
                    self.save_checkpoint()
                if cuda:
                    ev["pre"], ev["pre2"] = ev["pre2"], ev["pre"]
                    ev["post"], ev["post2"] = ev["post2"], ev["post"]
                    ev["step"], ev["step2"] = ev["step2"], ev["step"]
                if cuda and cfg.profile_step >= 0 and self.global_step == cfg.profile_step:
                    self.log_packing_utilization()
                    self._barrier()
                    torch.cuda.synchronize()
                    torch.cuda.cudart().cudaProfilerStart()
            if cuda:
                torch.cuda.cudart().cudaProfilerStop()
            self.log_packing_utilization()
            if not ckpt.is_complete(self.checkpoint_dir(self.global_step)):
                self.save_checkpoint()
            elif cuda:
                self._check_device_errors()
            log.info(f"Training finished at step {self.global_step}")
            if self.wandb is not None:
                self.wandb.finish()
        finally:
            self.heartbeat.stop()
            if loader is not None:
                loader.close()
        return self.history


def main(argv=None) -> None:
    from ..config.training import parse_training_config
    cfg = parse_training_config(argv)
    trainer = Trainer(cfg)
    trainer.train()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
