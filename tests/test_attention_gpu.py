"""sm_100a varlen attention (forward + backward) against a PyTorch fp32 reference."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def ref_attention(q, k, v, lens, scale):
    out = torch.zeros_like(q, dtype=torch.float32)
    lse = torch.zeros(q.shape[1], q.shape[0])
    start = 0
    for n in lens:
        qs, ks, vs = (t[start:start + n].float().transpose(0, 1) for t in (q, k, v))
        s = qs @ ks.transpose(-1, -2) * scale
        lse[:, start:start + n] = torch.logsumexp(s, -1)
        out[start:start + n] = (torch.softmax(s, -1) @ vs).transpose(0, 1)
        start += n
    return out, lse


@pytest.fixture(params=[1, 2, 0], ids=["fused_bwd", "pipelined_bwd", "two_pass_bwd"])
def bwd_variant(request):
    from pan2_b200.ops._ext import ext
    ext().attn_set_backward_variant(request.param)
    yield request.param
    ext().attn_set_backward_variant(1)


@pytest.mark.parametrize("lens", [[128], [300, 129, 1000, 64], [2048, 5, 700]])
def test_attention_forward_backward(lens, bwd_variant):
    from pan2_b200.ops.attention import varlen_attention
    from pan2_b200.ops._ext import ext
    torch.manual_seed(0)
    H, D = 4, 128
    L = sum(lens) + 9
    scale = 1 / math.sqrt(D)
    q, k, v = (torch.randn(L, H, D) * s for s in (1.0, 1.0, 1.0))
    qc, kc, vc = (t.to(torch.bfloat16).cuda().requires_grad_(True) for t in (q, k, v))
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    o = varlen_attention(qc, kc, vc, cu, lens)
    qr, kr, vr = (t.detach().cpu().float().requires_grad_(True) for t in (qc, kc, vc))
    o_ref, _ = ref_attention(qr, kr, vr, lens, scale)
    err = (o.float().cpu() - o_ref).abs().max().item()
    assert err < 2e-2, err
    assert o[sum(lens):].abs().max().item() == 0
    g = torch.randn(L, H, D)
    g[sum(lens):] = 0
    o.backward(g.to(torch.bfloat16).cuda())
    o_ref.backward(g.to(torch.bfloat16).float())
    for a, r, n in ((qc.grad, qr.grad, "dq"), (kc.grad, kr.grad, "dk"), (vc.grad, vr.grad, "dv")):
        e = (a.float().cpu() - r).abs().max().item() / (r.abs().max().item() + 1e-6)
        assert e < 3e-2, (n, e)
    torch.cuda.synchronize()
    assert ext().error_flag(True) == 0
