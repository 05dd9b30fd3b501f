"""sm_100a varlen attention (forward + backward) against a PyTorch fp32 reference."""
import math

import pytest
import torch

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


@pytest.fixture(params=[1, 0], ids=["inorder_fwd", "awaiting_fwd"])
def variants(request):
    from pan2_b200.ops._ext import ext
    E = ext()
    saved = E.attn_get_variant(0)
    E.attn_set_forward_variant(request.param)
    yield request.param
    E.attn_set_forward_variant(saved)


@pytest.mark.parametrize("lens", [[128], [300, 129, 1000, 64], [2048, 5, 700]])
def test_attention_forward_backward(lens, variants):
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


def test_attention_full_length_segment_sampled_rows():
    """One 18,992-token segment with 32 heads (the training bench's clip), checked on sampled rows
    against fp32: output and LSE of sampled query rows, dQ of sampled query rows, dK / dV of sampled
    key rows (the fp32 log-sum-exp and Delta of every query row are computed in chunks)."""
    from pan2_b200.ops._ext import ext
    from pan2_b200.ops.attention import work_items
    torch.manual_seed(1)
    S, H, D = 18992, 32, 128
    scale = 1 / math.sqrt(D)
    q, k, v, do = (torch.randn(S, H, D, device="cuda").to(torch.bfloat16) for _ in range(4))
    E = ext()
    o, lse = E.attn_fwd(q, k, v, work_items([S], 256, q.device), S, scale)
    items = work_items([S], 128, q.device)
    dq, dk, dv = E.attn_bwd(do, q, k, v, o, lse, items, items, S, scale)
    torch.cuda.synchronize()
    assert E.error_flag(True) == 0
    qf, kf, vf, dof = (t.float().transpose(0, 1).contiguous() for t in (q, k, v, do))  # [H, S, D]
    lse_ref = torch.empty(H, S, device="cuda")
    delta_ref = torch.empty(H, S, device="cuda")
    rows = torch.randperm(S, device="cuda")[:96].sort().values
    o_rows = None
    for r0 in range(0, S, 1024):
        s = torch.matmul(qf[:, r0:r0 + 1024], kf.transpose(1, 2)) * scale
        lse_ref[:, r0:r0 + 1024] = torch.logsumexp(s, -1)
        o_blk = torch.matmul(torch.softmax(s, -1), vf)
        delta_ref[:, r0:r0 + 1024] = (dof[:, r0:r0 + 1024] * o_blk).sum(-1)
        del s, o_blk
    s = torch.matmul(qf[:, rows], kf.transpose(1, 2)) * scale                  # [H, r, S]
    p = torch.exp(s - lse_ref[:, rows, None])
    o_rows = torch.matmul(p, vf)
    o_err = (o.float()[rows].transpose(0, 1) - o_rows).abs().max().item()
    assert o_err < 2e-2, o_err
    lse_err = (lse[:, rows] - lse_ref[:, rows]).abs().max().item()
    assert lse_err < 1e-2, lse_err
    dp = torch.matmul(dof[:, rows], vf.transpose(1, 2))
    dq_ref = torch.matmul(p * (dp - delta_ref[:, rows, None]), kf) * scale     # [H, r, D]
    e = (dq.float()[rows].transpose(0, 1) - dq_ref).abs().max().item() / dq_ref.abs().max().item()
    assert e < 3e-2, ("dq", e)
    st = torch.matmul(kf[:, rows], qf.transpose(1, 2)) * scale                 # rows of S^T: [H, r, S]
    pt = torch.exp(st - lse_ref[:, None, :])
    dv_ref = torch.matmul(pt, dof)
    dpt = torch.matmul(vf[:, rows], dof.transpose(1, 2))
    dk_ref = torch.matmul(pt * (dpt - delta_ref[:, None, :]), qf) * scale
    for got, ref, name in ((dk, dk_ref, "dk"), (dv, dv_ref, "dv")):
        e = (got.float()[rows].transpose(0, 1) - ref).abs().max().item() / ref.abs().max().item()
        assert e < 3e-2, (name, e)
