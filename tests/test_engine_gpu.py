"""The sharded engine on the B200 (world 1): forward/backward through BlockCheckpoint + flat
gradients must equal plain autograd on the same bf16 weights; one optimizer step runs clean."""
import pytest
import torch

from tiny import TINY_ARCH, tiny_batch

pytestmark = pytest.mark.gpu

ARCH = dict(TINY_ARCH, hidden_size=512, num_attention_heads=4, rope_axes_dim=(32, 48, 48))


def _dev(batch):
    from pan2_b200.data.synthetic import batch_to_device
    b = batch_to_device(batch, "cuda")
    for k in ("hidden_states", "text_states", "target"):
        b[k] = b[k].to(torch.bfloat16)
    return b


def test_engine_matches_autograd_and_steps():
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    from pan2_b200.ops._ext import ext
    eng = TrainEngine(ARCH, torch.device("cuda"), seed=5, optim=OptimConfig(lr=1e-3), offload="off")
    ref = PanVideoDiffusionTransformer(**ARCH).cuda()
    sd = {k: v.to(torch.bfloat16).float() for k, v in eng.sharded.full_state_dict().items()}
    # engine computes with the bf16 truncation of the masters: give the reference the same weights
    hi_sd = {}
    for u in eng.sharded.units:
        for s in u.slots:
            hi_sd[s.name] = u.slot_full(u.hi, s).float().clone()
    ref.load_state_dict(hi_sd, strict=False)
    ref = ref.to(torch.bfloat16)
    batch, _ = tiny_batch(ref)
    b = _dev(batch)
    loss_e = eng.forward_backward(b)
    loss_r = ref(**b)
    loss_r.backward()
    assert abs(loss_e.item() - loss_r.item()) < 1e-3 * abs(loss_r.item()) + 1e-5
    grads_e = {}
    for u in eng.sharded.units:
        for s in u.slots:
            grads_e[s.name] = u.slot_full(u.full_grad, s).float()
    worst = 1.0
    for n, p in ref.named_parameters():
        if p.grad is None or n not in grads_e:
            continue
        c = torch.nn.functional.cosine_similarity(grads_e[n].flatten(), p.grad.float().flatten(), dim=0).item()
        if p.grad.abs().max() > 0:
            worst = min(worst, c)
    assert worst > 0.999, worst
    norm = eng.grad_norm()
    eng.optimizer_step()
    torch.cuda.synchronize()
    assert torch.isfinite(norm).all()
    assert ext().error_flag(True) == 0
    loss2 = eng.forward_backward(b)
    assert torch.isfinite(loss2)


@pytest.mark.parametrize("shape", [(6, 128, 512), (1, 384, 256), (2, 256, 640)])
def test_gram_newton_schulz_matches_cpu(shape):
    """tcgen05 batched Gram Newton-Schulz == the CPU recurrence with the same bf16 rounding points,
    for every step count (the reset at step 2 included); 5 steps orthogonalise."""
    from pan2_b200.optim.muon import gram_newton_schulz, _ns_cpu, NS_COEFFS, NS_EPS
    torch.manual_seed(0)
    G = torch.randn(*shape)
    transpose = shape[1] > shape[2]
    for steps in range(1, 6):
        out_gpu = gram_newton_schulz(G.cuda().to(torch.bfloat16), steps=steps).float().cpu()
        X = G.transpose(-1, -2) if transpose else G
        ref = _ns_cpu(X, NS_COEFFS, steps, NS_EPS, 2, round_bf16=True)
        ref = ref.transpose(-1, -2) if transpose else ref
        c = torch.nn.functional.cosine_similarity(out_gpu.flatten(), ref.flatten(), dim=0).item()
        assert c > 0.99, (shape, steps, c)
    s = torch.linalg.svdvals(out_gpu[0])
    assert s.max() < 1.3 and s.min() > 0.5, (shape, s.min(), s.max())


def test_deferred_offloaded_optimizer_matches_synchronous():
    """Host-offloaded optimizer state: updates overlapped with the next forward give the same
    weights as the synchronous streamed optimizer."""
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    from pan2_b200.ops._ext import ext
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**ARCH)
    batch, _ = tiny_batch(shape_model)
    b = _dev(batch)
    res = {}
    for defer in (False, True):
        # an activation reserve larger than the GPU puts every lo half and optimizer state on the host
        eng = TrainEngine(ARCH, torch.device("cuda"), seed=5, optim=OptimConfig(lr=1e-3), offload="on",
                          activation_bytes_estimate=int(1e15))
        assert all(u.lo.device.type == "cpu" for u in eng.sharded.units)
        eng.defer_optimizer = defer
        losses = []
        for step in range(3):
            loss = eng.forward_backward(b)
            eng.grad_norm()
            eng.optimizer_step()
            eng.set_lr(1e-3 * (0.5 ** (step + 1)))  # changed right after the step, as the step runner does
            losses.append(loss.item())
        eng.flush_updates()
        torch.cuda.synchronize()
        res[defer] = (losses, [u.hi.float().cpu().clone() for u in eng.sharded.units])
        assert ext().error_flag(True) == 0
        del eng
    assert res[False][0] == res[True][0]
    for a, c in zip(res[False][1], res[True][1]):
        assert torch.equal(a, c)


def _unit_state_bytes(u):
    ts = [u.lo] + [t for t in u.state.values() if t is not None]
    return sum(t.numel() * t.element_size() for t in ts)


def test_offloaded_state_placed_in_forward_order():
    """A GPU budget for part of the offloadable state gives the root unit and then the first blocks
    their lo halves and optimizer state on the GPU, whole; the last block streams from the host; the
    overlapped updates over that mixed placement equal the synchronous ones."""
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**ARCH)
    batch, _ = tiny_batch(shape_model)
    b = _dev(batch)
    probe = TrainEngine(ARCH, torch.device("cuda"), seed=5, optim=OptimConfig(lr=1e-3), offload="on",
                        offload_gpu_bytes=0)
    units = probe.sharded.units
    budget = _unit_state_bytes(units[-1]) + _unit_state_bytes(units[0]) + (4 << 20)  # slack of the root estimate
    del probe
    res = {}
    for defer in (False, True):
        eng = TrainEngine(ARCH, torch.device("cuda"), seed=5, optim=OptimConfig(lr=1e-3), offload="on",
                          offload_gpu_bytes=budget)
        us = eng.sharded.units
        on_gpu = lambda u: [t.is_cuda for t in [u.lo] + [t for t in u.state.values() if t is not None]]
        assert all(on_gpu(us[-1])) and all(on_gpu(us[0]))      # root, then block 0
        assert not any(on_gpu(us[-2]))                          # the last block streams
        eng.defer_optimizer = defer
        losses = []
        for step in range(3):
            losses.append(eng.forward_backward(b).item())
            eng.grad_norm()
            eng.optimizer_step()
        eng.flush_updates()
        torch.cuda.synchronize()
        res[defer] = (losses, [u.hi.float().cpu().clone() for u in us])
        del eng
    assert res[False][0] == res[True][0]
    for a, c in zip(res[False][1], res[True][1]):
        assert torch.equal(a, c)


@pytest.mark.parametrize("mode", ["keep_attention", "no_recompute"])
def test_checkpointing_modes_give_the_recompute_gradients(mode):
    """Kept-attention checkpointing (the recompute skips the attention forward) and no activation
    checkpointing give the gradients of full per-block recomputation on the B200."""
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    with torch.device("meta"):
        shape_model = PanVideoDiffusionTransformer(**ARCH)
    batch, _ = tiny_batch(shape_model)
    b = _dev(batch)
    res = []
    for m in ("recompute", mode):
        eng = TrainEngine(ARCH, torch.device("cuda"), seed=5, optim=OptimConfig(lr=1e-3), offload="off")
        if m == "keep_attention":
            eng.set_activation_checkpointing(True, keep_attention=True)
        elif m == "no_recompute":
            eng.set_activation_checkpointing(False)
        loss = eng.forward_backward(b)
        grads = [u.full_grad.float().clone() for u in eng.sharded.units]
        res.append((loss.item(), grads))
        del eng
        torch.cuda.empty_cache()
    (la, ga), (lb, gb) = res
    assert abs(la - lb) <= 1e-6 * abs(la) + 1e-7
    for x, y in zip(ga, gb):
        assert (x - y).abs().max().item() <= 2e-2 * (x.abs().max().item() + 1e-12)
