"""Numerics of the sm_100a kernels against plain PyTorch fp32 references (run on a B200)."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def ext():
    from pan2_b200.ops._ext import ext as _e
    return _e()


def assert_close(out, ref, tol, name=""):
    out, ref = out.float(), ref.float()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"{name}: max err {err:.3e} vs scale {scale:.3e}"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    torch.cuda.synchronize()
    assert ext().error_flag(True) == 0, "a kernel recorded a bounded-wait timeout"


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.fixture(params=[1, 2], ids=["cta1", "cta2"])
def cta_group(request):
    ext().gemm_force_cta_group(request.param)
    yield request.param
    ext().gemm_force_cta_group(0)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 200, 136), (1024, 768, 512), (77, 4096, 256),
                                   (2304, 2048, 1024), (1100, 16640, 256)])  # last: 16-tile N bands
def test_gemm_nt(M, N, K, cta_group):
    a, b = bf(M, K), bf(N, K)
    bias = bf(N)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(a, b, out, True, True, bias, None, False)
    ref = a.float() @ b.float().t() + bias.float()
    assert_close(out, ref, 1e-2, "nt")


@pytest.mark.parametrize("M,N,K", [(256, 128, 256), (300, 200, 136), (512, 1024, 768), (1300, 1536, 512),
                                   (700, 16640, 128)])
def test_gemm_nn(M, N, K, cta_group):
    a, b = bf(M, K), bf(K, N)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(a, b, out, True, False, None, None, False)
    assert_close(out, a.float() @ b.float(), 1e-2, "nn")


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (200, 136, 300), (768, 512, 1000), (1024, 2048, 640)])
def test_gemm_tn_fp32_accumulate(M, N, K, cta_group):
    a, b = bf(K, M), bf(K, N)
    out = torch.randn(M, N, device="cuda")
    base = out.clone()
    ext().gemm(a, b, out, False, False, None, None, True)
    assert_close(out, base + a.float().t() @ b.float(), 1e-2, "tn")


def test_gemm_gelu_and_dgelu(cta_group):
    M, N, K = 384, 512, 256
    a, b, bias = bf(M, K), bf(N, K, scale=0.1), bf(N)
    pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(a, b, out, True, True, bias, pre, False)
    ref_pre = a.float() @ b.float().t() + bias.float()
    assert_close(pre, ref_pre, 1e-2, "pre")
    assert_close(out, F.gelu(ref_pre, approximate="tanh"), 2e-2, "gelu")
    # dgelu: dpre = (dY @ Wd) * gelu'(pre), post = gelu(pre)
    dY, Wd = bf(M, 128), bf(128, N)
    dpre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    post = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm_dgelu(dY, Wd, pre, dpre, post)
    p = pre.float().requires_grad_(True)
    g = F.gelu(p, approximate="tanh")
    (gp,) = torch.autograd.grad(g, p, dY.float() @ Wd.float())
    assert_close(dpre, gp, 2e-2, "dpre")
    assert_close(post, g.detach(), 2e-2, "post")


def test_gemm_grouped_two_weights(cta_group):
    L, K = 700, 256
    x = bf(L, K)
    w = [bf(384, K), bf(256, K)]
    b = [bf(384), bf(256)]
    bounds = [0, 450, 650]
    out = torch.zeros(L, 384, device="cuda", dtype=torch.bfloat16)
    ext().gemm_grouped_nt(x, w, out, b, None, bounds)
    ref = torch.zeros(L, 384, device="cuda")
    ref[0:450] = x[0:450].float() @ w[0].float().t() + b[0].float()
    ref[450:650, :256] = x[450:650].float() @ w[1].float().t() + b[1].float()
    assert_close(out, ref, 1e-2, "grouped")
    assert out[650:].abs().max().item() == 0


def _ops_pair(fn_cuda, fn_cpu, inputs, grads_of, gout_shape=None):
    """Run an op on CUDA (bf16) and on CPU (fp32), compare output and input grads."""
    cu = [t.detach().cuda().requires_grad_(t.requires_grad) if isinstance(t, torch.Tensor) else t for t in inputs]
    cp = [t.detach().float().requires_grad_(t.requires_grad) if isinstance(t, torch.Tensor) and t.is_floating_point() else t
          for t in inputs]
    oc = fn_cuda(*cu)
    op = fn_cpu(*cp)
    oc0 = oc[0] if isinstance(oc, tuple) else oc
    op0 = op[0] if isinstance(op, tuple) else op
    g = torch.randn_like(op0)
    oc0.backward(g.to(oc0.dtype).cuda())
    op0.backward(g)
    return oc, op, cu, cp


def test_ln_modulate_and_gate_ops():
    from pan2_b200.ops import packed as P
    torch.manual_seed(0)
    L, C = 300, 512
    bounds = [0, 100, 220, 280]
    x = (torch.randn(L, C) * 2 + 0.5).to(torch.bfloat16)
    stats = P.ln_stats_of(x.float(), 280)
    shift = (torch.randn(3, C) * 0.1).to(torch.bfloat16).requires_grad_(True)
    scale = (torch.randn(3, C) * 0.1).to(torch.bfloat16).requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    oc, op, cu, cp = _ops_pair(lambda a, s, h, sc: P.ln_modulate(a, s, h, sc, bounds),
                               lambda a, s, h, sc: P.ln_modulate(a, s, h, sc, bounds),
                               [xr, stats, shift, scale], None)
    assert_close(oc.cpu(), op, 2e-2, "ln_modulate")
    assert_close(cu[0].grad.cpu(), cp[0].grad, 3e-2, "ln_modulate dx")
    assert_close(cu[2].grad.cpu(), cp[2].grad, 2e-2, "dshift")
    assert_close(cu[3].grad.cpu(), cp[3].grad, 3e-2, "dscale")

    y = torch.randn(L, C).to(torch.bfloat16).requires_grad_(True)
    gate = (torch.randn(3, C)).to(torch.bfloat16).requires_grad_(True)
    res = torch.randn(L, C).to(torch.bfloat16).requires_grad_(True)
    oc, op, cu, cp = _ops_pair(lambda a, g, r: P.gate_residual(a, g, r, bounds),
                               lambda a, g, r: P.gate_residual(a, g, r, bounds), [y, gate, res], None)
    assert_close(oc[0].cpu(), op[0], 2e-2, "gate out")
    assert_close(oc[1].cpu(), op[1], 2e-2, "gate stats")
    assert_close(cu[0].grad.cpu(), cp[0].grad, 2e-2, "gate dy")
    assert_close(cu[1].grad.cpu(), cp[1].grad, 2e-2, "dgate")
    assert_close(cu[2].grad.cpu(), cp[2].grad, 1e-2, "dres")


def test_concat_mse_segment_sum():
    from pan2_b200.ops import packed as P
    torch.manual_seed(1)
    C = 256
    vid = torch.randn(130, C).to(torch.bfloat16).requires_grad_(True)
    txt = torch.randn(70, C).to(torch.bfloat16).requires_grad_(True)
    ttv = torch.randn(C).to(torch.bfloat16).requires_grad_(True)
    oc, op, cu, cp = _ops_pair(lambda v, t, e: P.simple_concat(v, t, 215, e),
                               lambda v, t, e: P.simple_concat(v, t, 215, e), [vid, txt, ttv], None)
    assert_close(oc[0].cpu(), op[0], 1e-2, "concat")
    assert_close(oc[1].cpu(), op[1], 2e-2, "concat stats")
    assert_close(cu[2].grad.cpu(), cp[2].grad, 2e-2, "dttv")
    pred = torch.randn(215, 192).to(torch.bfloat16)
    tgt = torch.randn(130, 192).to(torch.bfloat16)
    pc = pred.cuda().requires_grad_(True)
    sums = P.concat_mse_sums(pc, tgt.cuda(), 130)
    ref = (pred[:130].float() - tgt.float()).pow(2).sum()
    assert abs(sums[0].item() - ref.item()) / ref.item() < 1e-4
    assert sums[1].item() == 130 * 192
    (sums[0] / sums[1]).backward()
    gref = 2 * (pred[:130].float() - tgt.float()) / (130 * 192)
    assert_close(pc.grad[:130].cpu(), gref, 1e-2, "mse grad")
    assert pc.grad[130:].abs().max().item() == 0
    x = torch.randn(500, 512).to(torch.bfloat16)
    s = P.segment_sum(x.cuda(), [0, 200, 450])
    ref = torch.stack([x[:200].float().sum(0), x[200:450].float().sum(0)])
    assert_close(s.cpu(), ref, 1e-3, "segment_sum")


def test_qkv_project_matches_reference():
    from pan2_b200.ops.qkv import qkv_project
    from pan2_b200.models.packed import layout_permutations
    torch.manual_seed(2)
    heads, D = 4, 128
    hidden = heads * D
    vl, cl = [90, 60], [20, 30]
    L = sum(vl) + sum(cl) + 5
    itc, _ = layout_permutations(vl, cl, L)
    bounds = [0, sum(vl), sum(vl) + sum(cl)]
    x = (torch.randn(L, hidden) * 0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(2, 3 * hidden, hidden) / math.sqrt(hidden)).requires_grad_(True)
    b = (torch.randn(2, 3 * hidden) * 0.1).requires_grad_(True)
    qw = (1 + 0.1 * torch.randn(2 * D)).requires_grad_(True)
    kw = (1 + 0.1 * torch.randn(2 * D)).requires_grad_(True)
    ang = torch.randn(L, D // 2)
    cos = ang.cos().repeat_interleave(2, 1)
    sin = ang.sin().repeat_interleave(2, 1)
    itc32 = itc.to(torch.int32)

    def run(dev, dt):
        args = [t.detach().to(dev, dt if t.dtype == torch.bfloat16 else torch.float32).requires_grad_(True)
                for t in (x, w, b, qw, kw)]
        q, k, v = qkv_project(args[0], args[1], args[2], args[3], args[4], cos.to(dev), sin.to(dev),
                              itc32.to(dev), bounds, heads)
        gq = torch.ones_like(q) * 0.01 + torch.linspace(-1, 1, q.numel(), device=dev).view_as(q).to(q.dtype)
        (q.float() * gq.float() + k.float() * gq.float().flip(0) + v.float() * gq.float()).sum().backward()
        return (q, k, v), [a.grad for a in args]

    (qc, kc, vc), gc = run("cuda", torch.bfloat16)
    (qr, kr, vr), gr = run("cpu", torch.float32)
    for a, r, n in ((qc, qr, "q"), (kc, kr, "k"), (vc, vr, "v")):
        assert_close(a.cpu(), r, 2e-2, n)
    for a, r, n in zip(gc, gr, ["dx", "dw", "db", "dqw", "dkw"]):
        assert_close(a.cpu(), r, 3e-2, n)


def test_ln_modulate_forward_wide_rows_many_segments():
    """Bench-width rows (C = 4096, two column slabs), several segments per CTA row run, padding
    rows at the end: equal to the fp32 formula."""
    from pan2_b200.ops._ext import ext
    from pan2_b200.ops.packed import _bounds_tensor, ln_stats_of
    torch.manual_seed(3)
    L, C = 5003, 4096
    bounds = [0, 7, 1500, 1501, 3333, 4990]
    x = (torch.randn(L, C, device="cuda") * 1.5 + 0.3).to(torch.bfloat16)
    stats = ln_stats_of(x)
    shift = (torch.randn(5, C, device="cuda") * 0.1).to(torch.bfloat16)
    scale = (torch.randn(5, C, device="cuda") * 0.1).to(torch.bfloat16)
    y = ext().ln_modulate_fwd(x, stats, shift, scale, _bounds_tensor(bounds, x.device), 5)
    xf = x.float()
    mean = stats[:, 0:1] / C
    rstd = torch.rsqrt((stats[:, 1:2] / C - mean * mean).clamp_min(0) + 1e-6)
    ref = torch.zeros(L, C, device="cuda")
    for s in range(5):
        a, b = bounds[s], bounds[s + 1]
        ref[a:b] = (xf[a:b] - mean[a:b]) * rstd[a:b] * (1 + scale[s].float()) + shift[s].float()
    assert (y.float() - ref).abs().max().item() < 3e-2
    assert y[bounds[-1]:].abs().max().item() == 0


@pytest.mark.parametrize("B,M", [(1, 5120), (3, 200), (4, 36)])
def test_newton_schulz_normalise_and_rescale(B, M):
    """The two per-element Newton-Schulz passes equal the fp32 formulas rounded once to bf16:
    Rn = bf16(R / max(tr R, eps^2)) and Q <- bf16(Q / sqrt(max(tr R, eps^2)))."""
    E = ext()
    torch.manual_seed(B * M)
    eps = 1e-7
    R = torch.randn(B, M, M, device="cuda")
    norm2 = torch.empty(B, device="cuda")
    E.ns_trace(R, norm2)
    ref_n2 = torch.diagonal(R, dim1=-2, dim2=-1).sum(-1)
    assert torch.allclose(norm2, ref_n2, rtol=1e-4, atol=1e-3)
    norm2.abs_()
    Rn = torch.empty(B, M, M, device="cuda", dtype=torch.bfloat16)
    E.ns_gram_normalize(R, norm2, eps, Rn)
    den = norm2.clamp_min(eps * eps).view(-1, 1, 1)
    assert torch.equal(Rn, (R * (1.0 / den)).to(torch.bfloat16))
    Q = bf(B, M, M)
    want = (Q.float() * torch.rsqrt(den)).to(torch.bfloat16)
    E.ns_scale_by_invnorm(Q, norm2, eps)
    assert (Q.float() - want.float()).abs().max().item() <= 2 ** -7 * want.float().abs().max().item()
