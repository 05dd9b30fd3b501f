"""One tiny training step of the flagship MMDiT on ``cuda:0`` through the package's own kernels.

A 2-layer, 512-wide model of the 29B architecture (same blocks, packed layout, Muon + AdamW) takes one
synthetic packed batch through :class:`~pan2_b200.training.engine.TrainEngine`: forward (tcgen05 GEMMs,
packed elementwise kernels, varlen attention), backward, gradient norm and one optimizer step.  The
kernels' device error flags must stay clear and the loss finite.
"""
from __future__ import annotations

import torch

SMOKE_ARCH = dict(patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=512, num_attention_heads=4,
                  num_layers=2, mlp_ratio=8.0, context_mlp_ratio=4.0, rope_axes_dim=(32, 48, 48), rope_theta=256,
                  rope_temporal_scale=16 / 24, text_embed_dim=4096, zero_init_modulation=False)


def run_smoke(device: str = "cuda:0") -> float:
    from .data.synthetic import batch_to_device, synthetic_packed_batch
    from .ops._ext import ext
    from .training.engine import OptimConfig, TrainEngine

    if not torch.cuda.is_available():
        raise RuntimeError("smoke() needs a CUDA device")
    dev = torch.device(device)
    torch.cuda.set_device(dev)
    lib = ext()  # raises if the sm_100a extension is missing
    lib.error_flag(True)
    eng = TrainEngine(SMOKE_ARCH, dev, seed=0, optim=OptimConfig(lr=1e-4), offload="off")
    batch = synthetic_packed_batch(2, (3, 16, 16), 40, rope_axes=(32, 48, 48), seed=0, pin=True)
    batch = batch_to_device(batch, dev)
    loss = eng.forward_backward(batch)
    norm = eng.grad_norm()
    eng.optimizer_step()
    torch.cuda.synchronize(dev)
    flag = lib.error_flag(True)
    if flag != 0:
        raise RuntimeError(f"device error flag {flag:#x} after the smoke step")
    value = float(loss.item())
    if not torch.isfinite(torch.tensor(value)) or not bool(torch.isfinite(norm).all()):
        raise RuntimeError(f"non-finite smoke step: loss {value}, grad norm {norm}")
    print(f"smoke: loss {value:.5f} grad-norm {float(norm.reshape(-1)[0]):.4f}")
    return value


if __name__ == "__main__":
    run_smoke()
