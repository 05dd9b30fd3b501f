"""Kernel micro-benchmarks of the 29B training step's hot ops, against the measured roofline.

    python bench_kernels.py                       # every case at the bench shapes
    python bench_kernels.py --case gemm --small   # one small case per kernel (for profiler captures)

Each case prints one JSON line: the shape, the median device time over ``--iters`` launches (CUDA
events on the launching stream, one pair per launch, an L2 flush of 256 MiB between launches so no
launch reads the previous one's operands from L2), the achieved TFLOP/s or GB/s and the fraction of
the measured peak (``MEASURED_PEAKS.json``: copy bandwidth and cuBLAS bf16 burst throughput; the
earlier pool measurements 6650 GB/s and 1590 TFLOP/s when it is absent).  GEMM and attention cases
also time the library kernel of the same op (cuBLAS through ``torch.matmul``, cuDNN / flash through
``scaled_dot_product_attention``) unless ``--no-library``.

Shapes are the 29B model's (hidden 4096, 32 heads of 128, FFN 32768) on the training bench's
packed batch (5 clips of 18,992 joint tokens; 94,976 rows in total).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics

import torch

from pan2_b200.ops._ext import ext
from pan2_b200.ops.attention import work_items
from pan2_b200.ops.packed import _bounds_tensor, ln_stats_of

HIDDEN, HEADS, HEAD_DIM, FFN = 4096, 32, 128, 32768
GEMM_BAND_MB = 0  # the GEMM tile-order setting restored after a --gemm-band-mb sweep
CLIPS, CLIP_TOKENS = 5, 18992


def measured_peaks():
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


class Timer:
    """Median per-launch device time with an L2 flush between launches.  With ``sustain_s`` > 0 the
    op first runs back to back for that long (clocks settle under the power cap).  The SM clock is
    sampled during the timed launches (``last_clock``: median MHz and throttle reasons)."""

    def __init__(self, iters: int, warmup: int, sustain_s: float = 0.0):
        self.iters, self.warmup, self.sustain_s = iters, warmup, sustain_s
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.last_clock = None

    def __call__(self, fn) -> float:
        import time
        from pan2_b200.utils.clocks import ClockSampler
        for _ in range(self.warmup):
            fn()
        if self.sustain_s > 0:
            torch.cuda.synchronize()
            t0 = time.time()
            while time.time() - t0 < self.sustain_s:
                for _ in range(4):
                    fn()
                torch.cuda.synchronize()
        sampler = ClockSampler(interval_ms=50)
        sampler.start()
        times = []
        torch.cuda.synchronize()
        for _ in range(self.iters):
            self.flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            times.append((s, e))
        torch.cuda.synchronize()
        clk = sampler.stop(gpus=[torch.cuda.current_device()])
        self.last_clock = {"sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons")}
        return statistics.median(s.elapsed_time(e) for s, e in times)

    def clock_fields(self, prefix: str, ms: float) -> dict:
        """Median SM clock of the last timing and time x clock (the clock-normalised cost)."""
        c = self.last_clock or {}
        mhz = c.get("sm_mhz")
        out = {f"{prefix}sm_mhz": mhz, f"{prefix}reasons": c.get("reasons")}
        if mhz:
            out[f"{prefix}ms_x_ghz"] = round(ms * mhz / 1000.0, 4)
        return out


def gemm_cases(small: bool, only=None, rows=None):
    """The step's GEMM shapes; ``only`` keeps the named ones, ``rows`` overrides the token rows."""
    rows = rows or (8192 if small else CLIPS * CLIP_TOKENS)
    # (name, M, N, K, layout): NT = x @ w^T (forward), NN = dy @ w (input grad), TN = x^T @ dy (weight grad)
    cases = [("qkv_fwd", rows, 3 * HIDDEN, HIDDEN, "NT"), ("ffn_up_fwd", rows, FFN, HIDDEN, "NT"),
             ("ffn_down_fwd", rows, HIDDEN, FFN, "NT"), ("ffn_down_dgrad", rows, FFN, HIDDEN, "NN"),
             ("ffn_up_wgrad", FFN, HIDDEN, rows, "TN")]
    if only:
        return [c for c in cases if c[0] in only]
    return cases[:1] if small else cases


def run_gemm(name, M, N, K, layout, timer, library, peaks, band_mbs=(None,), probes=(None,), band_ns=(None,)):
    E = ext()
    dev = "cuda"
    a = torch.randn(K, M, device=dev, dtype=torch.bfloat16) if layout == "TN" else \
        torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) if layout == "NT" else \
        torch.randn(K, N, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=dev, dtype=torch.float32 if layout == "TN" else torch.bfloat16)
    fn = lambda: E.gemm(a, b, out, layout != "TN", layout == "NT", None, None, False)
    fl = 2.0 * M * N * K
    recs = []
    for band, probe, bn in [(b, pr, w) for b in band_mbs for pr in probes for w in band_ns]:
        E.gemm_tuning(6, int(probe or 0), GEMM_BAND_MB if band is None else int(band), int(bn or 0))
        ms = timer(fn)
        rec = dict(case=f"gemm_{name}", shape=[M, N, K], layout=layout, out_dtype=str(out.dtype).split(".")[-1],
                   ms=round(ms, 4), tflops=round(fl / ms / 1e9, 1), frac_of_peak=round(fl / ms / 1e9 / peaks[1], 3))
        if band is not None:
            rec["band_mb"] = int(band)
        if probe:
            rec["probe"] = int(probe)
        if bn:
            rec["band_n"] = int(bn)
        rec.update(timer.clock_fields("", ms))
        recs.append(rec)
    E.gemm_tuning(6, 0, GEMM_BAND_MB, 0)
    if library:
        ao = a.t() if layout == "TN" else a
        bo = b.t() if layout == "NT" else b
        lib_out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ms_l = timer(lambda: torch.matmul(ao, bo, out=lib_out))
        for rec in recs:
            rec["cublas_bf16_out_ms"] = round(ms_l, 4)
            rec["cublas_tflops"] = round(fl / ms_l / 1e9, 1)
            rec.update(timer.clock_fields("cublas_", ms_l))
    for rec in recs:
        rec["error_flag"] = E.error_flag(True)
    return recs


def run_attention(small, timer, library, peaks, which, fwd_variants=(None,)):
    E = ext()
    lens = [8192] if small else [CLIP_TOKENS] * CLIPS
    L = sum(lens)
    q, k, v = (torch.randn(L, HEADS, HEAD_DIM, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    scale = 1 / math.sqrt(HEAD_DIM)
    it_f, it_b = work_items(lens, 256, q.device), work_items(lens, 128, q.device)
    fl = sum(4.0 * s * s * HEAD_DIM * HEADS for s in lens)
    default_f = E.attn_get_variant(0)
    out = []
    o, lse = E.attn_fwd(q, k, v, it_f, L, scale)
    lib_f = None
    if "fwd" in which:
        for var in fwd_variants:
            E.attn_set_forward_variant(default_f if var is None else int(var))
            ms = timer(lambda: E.attn_fwd(q, k, v, it_f, L, scale))
            rec = dict(case="attn_fwd", segments=lens, heads=HEADS, head_dim=HEAD_DIM,
                       variant=E.attn_get_variant(0), ms=round(ms, 4), tflops=round(fl / ms / 1e9, 1),
                       frac_of_peak=round(fl / ms / 1e9 / peaks[1], 3))
            rec.update(timer.clock_fields("", ms))
            if library:
                lib_f = lib_f or _sdpa(q, lens, timer, fl, backward=False)
                rec.update(lib_f)
            out.append(rec)
        E.attn_set_forward_variant(default_f)
    if "bwd" in which:
        o, lse = E.attn_fwd(q, k, v, it_f, L, scale)
        do = torch.randn_like(o)
        flb = 2.5 * fl  # dV, dP, dQ, dK GEMMs plus the S recompute
        ms = timer(lambda: E.attn_bwd(do, q, k, v, o, lse, it_b, it_b, L, scale))
        rec = dict(case="attn_bwd", segments=lens, heads=HEADS, head_dim=HEAD_DIM, ms=round(ms, 4),
                   tflops=round(flb / ms / 1e9, 1), frac_of_peak=round(flb / ms / 1e9 / peaks[1], 3))
        rec.update(timer.clock_fields("", ms))
        if library:
            rec.update(_sdpa(q, lens, timer, flb, backward=True))
        out.append(rec)
    for r in out:
        r["error_flag"] = E.error_flag(True)
    return out


def _sdpa(q, lens, timer, fl, backward):
    """The library attention on the same work: one dense call per segment (no varlen packing)."""
    import torch.nn.functional as F
    try:
        segs = []
        start = 0
        for s in lens:
            x = q[start:start + s].transpose(0, 1).unsqueeze(0).contiguous().requires_grad_(backward)
            segs.append(x)
            start += s
        if not backward:
            ms = timer(lambda: [F.scaled_dot_product_attention(x, x, x) for x in segs])
            return {"sdpa_ms": round(ms, 4), "sdpa_tflops": round(fl / ms / 1e9, 1)}
        outs = [F.scaled_dot_product_attention(x, x, x) for x in segs]
        grads = [torch.randn_like(o) for o in outs]

        def bwd():
            for x, o, g in zip(segs, outs, grads):
                torch.autograd.grad(o, x, g, retain_graph=True)
        ms = timer(bwd)
        return {"sdpa_bwd_ms": round(ms, 4), "sdpa_bwd_tflops": round(fl / ms / 1e9, 1)}
    except RuntimeError as err:  # a backend without this shape
        return {"sdpa_error": str(err).splitlines()[0][:200]}


def run_elementwise(small, timer, peaks, which):
    E = ext()
    L = 8192 * 4 if small else CLIPS * CLIP_TOKENS
    x = torch.randn(L, HIDDEN, device="cuda", dtype=torch.bfloat16)
    bounds = [i * (L // CLIPS) for i in range(CLIPS)] + [L]
    bt = _bounds_tensor(bounds, x.device)
    shift = torch.randn(CLIPS, HIDDEN, device="cuda", dtype=torch.bfloat16)
    scl = torch.randn(CLIPS, HIDDEN, device="cuda", dtype=torch.bfloat16)
    stats = ln_stats_of(x)
    out = []
    nbytes = x.numel() * 2
    if "ln_modulate" in which:
        ms = timer(lambda: E.ln_modulate_fwd(x, stats, shift, scl, bt, CLIPS))
        moved = 2 * nbytes + L * 8
        out.append(dict(case="ln_modulate_fwd", shape=[L, HIDDEN], ms=round(ms, 4),
                        gbs=round(moved / ms / 1e6, 1), frac_of_peak=round(moved / ms / 1e6 / peaks[0], 3)))
    if "gate_residual" in which:
        res = torch.randn_like(x)
        ms = timer(lambda: E.gate_residual_fwd(x, shift, res, bt, CLIPS))
        moved = 3 * nbytes + L * 8
        out.append(dict(case="gate_residual_fwd", shape=[L, HIDDEN], ms=round(ms, 4),
                        gbs=round(moved / ms / 1e6, 1), frac_of_peak=round(moved / ms / 1e6 / peaks[0], 3)))
    for r in out:
        r["error_flag"] = E.error_flag(True)
    return out


def _ns_library(G, coeffs=(3.4445, -4.7750, 2.0315), steps=5, eps=1e-7, reset=2):
    """The same Gram Newton-Schulz recurrence on cuBLAS (torch bf16 batched matmuls; the Gram of the
    input from bf16 operands with an fp32 result, as the fused Gram kernel forms it): the library
    baseline of the tcgen05 chain."""
    a, b, c = coeffs
    X = G.transpose(-1, -2) if G.shape[-2] > G.shape[-1] else G
    R32 = torch.bmm(X, X.transpose(-1, -2), out_dtype=torch.float32)
    n2 = torch.diagonal(R32, dim1=-2, dim2=-1).sum(-1).clamp(min=eps * eps).view(-1, 1, 1)
    R = (R32 / n2).to(torch.bfloat16)
    eye = torch.eye(R.shape[-1], device=G.device, dtype=torch.bfloat16)
    Q, first = None, True
    for i in range(steps):
        if i == reset and Q is not None:
            if first:
                Q = (Q / n2.sqrt()).to(torch.bfloat16)
                first = False
            X = torch.matmul(Q, X)
            R = torch.matmul(X, X.transpose(-1, -2))
            Q = None
        Z = c * torch.matmul(R, R) + b * R
        Q = a * eye + Z if Q is None else torch.matmul(Q, Z) + a * Q
        if i < steps - 1 and (i + 1) != reset:
            RZ = torch.matmul(R, Z) + a * R
            R = torch.matmul(Z, RZ) + a * RZ
    if first:
        Q = (Q / n2.sqrt()).to(torch.bfloat16)
    return torch.matmul(Q, X)


def run_muon_ns(timer, library):
    """Gram Newton-Schulz of the 29B block's Muon matrices: the QKV weight as its 192 per-head row
    chunks and the video FFN up-projection (orthogonalised through its 4096-row side)."""
    from pan2_b200.optim.muon import gram_newton_schulz
    out = []
    for name, shape in (("qkv_chunks", (192, 128, 4096)), ("ffn_up_video", (1, 32768, 4096)),
                        ("out_proj_chunks", (2, 4096, 4096))):
        G = torch.randn(*shape, device="cuda").to(torch.bfloat16)
        ms = timer(lambda: gram_newton_schulz(G))
        rec = dict(case=f"muon_ns_{name}", shape=list(shape), ms=round(ms, 4))
        if library:
            ms_l = timer(lambda: _ns_library(G))
            rec["library_bmm_ms"] = round(ms_l, 4)
        out.append(rec)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", default=".*",
                    help="regex over gemm, attn_fwd, attn_bwd, ln_modulate, gate_residual, muon_ns")
    ap.add_argument("--small", action="store_true", help="one small case per kernel (operands still above L2)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-library", action="store_true", help="skip the cuBLAS / SDPA comparisons")
    ap.add_argument("--attn-fwd-variant", default=None,
                    help="comma list of attention forward variants (1: in-order MMA issue, the default; 0: PV "
                         "completion awaited before the next score GEMM)")
    ap.add_argument("--gemm-band-mb", default=None,
                    help="comma list of GEMM M-band budgets in MB (0 = N bands only)")
    ap.add_argument("--gemm-shape", default=None,
                    help="comma list of GEMM cases to run (qkv_fwd, ffn_up_fwd, ffn_down_fwd, ffn_down_dgrad, ffn_up_wgrad)")
    ap.add_argument("--rows", type=int, default=None, help="token rows of the GEMM cases (default: the step's)")
    ap.add_argument("--gemm-band-n", default=None,
                    help="comma list of GEMM N-band widths in tiles (0 = the default of 8)")
    ap.add_argument("--gemm-probe", default=None,
                    help="comma list of GEMM probe bits (timing experiments: 1 skips the epilogue stores, 2 "
                         "re-reads k-block 0)")
    ap.add_argument("--sustain-s", type=float, default=0.0,
                    help="run each op back to back this long before timing (clocks settle under the power cap)")
    args = ap.parse_args()
    pat = re.compile(args.case)
    lst = lambda s: [int(x) for x in s.split(",")] if s else [None]
    peaks = measured_peaks()
    timer = Timer(args.iters, args.warmup, args.sustain_s)
    library = not args.no_library
    if pat.search("gemm"):
        only = args.gemm_shape.split(",") if args.gemm_shape else None
        for c in gemm_cases(args.small, only, args.rows):
            for rec in run_gemm(*c, timer=timer, library=library, peaks=peaks, band_mbs=lst(args.gemm_band_mb),
                                probes=lst(args.gemm_probe), band_ns=lst(args.gemm_band_n)):
                print(json.dumps(rec), flush=True)
    which = [w for w in ("fwd", "bwd") if pat.search("attn_" + w)]
    if which:
        for r in run_attention(args.small, timer, library, peaks, which, lst(args.attn_fwd_variant)):
            print(json.dumps(r), flush=True)
    which = [w for w in ("ln_modulate", "gate_residual") if pat.search(w)]
    if which:
        for r in run_elementwise(args.small, timer, peaks, which):
            print(json.dumps(r), flush=True)
    if pat.search("muon_ns"):
        for r in run_muon_ns(timer, library):
            print(json.dumps(r), flush=True)
    print(json.dumps({"peaks": {"hbm_gbs": peaks[0], "bf16_tflops": peaks[1], "source": peaks[2]}}))


if __name__ == "__main__":
    main()
