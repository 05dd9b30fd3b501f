"""Muon for PAN 2: parameter split, learning-rate adjustment and the Gram Newton-Schulz step.

* Parameter split (pan/optim/muon.py:12-92): Muon for 2-D hidden weights; AdamW for 1-D tensors,
  embeddings, the output head, the timestep encoder, the patch embedding and every modulation.
* ``adjust_lr`` = torch.optim.Muon's ``match_rms_adamw``: ``lr * 0.2 * sqrt(max(A, B))`` of the
  (chunk) shape; chunked weights (QKV: one chunk per (modality, q/k/v, head); out-proj: one per
  modality) are orthogonalised as independent row blocks (patch_muon.py:71-143).
* Nesterov momentum, coefficients (3.4445, -4.7750, 2.0315), 5 steps, eps 1e-7 (torch defaults).
* Newton-Schulz runs on the Gram matrix ``R = X X^T`` of the small side with a reset at iteration 2,
  exactly the recurrence of the reference's ``_gram_newtonschulz_local`` (patch_muon.py:275-334):
  ``Z = b R + c R^2``; ``Q = a I + Z`` (first) or ``Q = Q Z + a Q``; ``R <- (aI+Z) R (aI+Z)``; at the
  reset ``X <- Q X`` and ``R = X X^T``; finally ``X <- Q X``.  The Frobenius normalisation is folded
  through ``trace(R)``: the first ``Q`` is scaled by ``1/||X||`` instead of rescaling ``X``.

On CUDA every product is a batched call of the tcgen05 GEMM (``alpha * A B^T + beta * C`` epilogue)
over all chunks of one shape at once; wide matrices are orthogonalised through their transpose using
MN-major operands, so nothing is transposed in memory.
"""
from __future__ import annotations

import math
from typing import Dict, Sequence, Tuple

import torch

from ..ops._ext import ext

NS_COEFFS = (3.4445, -4.7750, 2.0315)
NS_STEPS = 5
NS_EPS = 1e-7
NS_RESET = 2


def looks_like_embedding_or_head(name: str) -> bool:
    """Parameters that stay on AdamW under Muon (pan/optim/muon.py:12-51)."""
    lower = name.lower()
    generic = ("embedding", "embed_tokens", "token_embed", "token_emb", "pos_embed", "position_embed",
               "lm_head", "output_head", "classifier")
    if any(p in lower for p in generic):
        return True
    if ".modulation." in lower or "text_modulation" in lower:
        return True
    return lower.startswith(("output_head.", "timestep_encoder.", "text_type_embedding", "patch_embed."))


def use_muon_for(name: str, shape: Sequence[int]) -> bool:
    return len(shape) == 2 and not looks_like_embedding_or_head(name)


def muon_chunks(module: torch.nn.Module) -> Dict[str, Tuple[int, int]]:
    """``{name: (dim, n_chunks)}`` from the ``_muon_chunks_dim_*`` hints on parameters."""
    out = {}
    for name, p in module.named_parameters():
        for dim in (0, 1):
            n = getattr(p, f"_muon_chunks_dim_{dim}", None)
            if n is not None:
                out[name] = (dim, int(n))
                break
    return out


def adjust_lr_scale(shape: Sequence[int], fn: str = "match_rms_adamw") -> float:
    """Multiplier on the learning rate for a (chunk) shape ``(A, B)``."""
    A, B = shape[:2]
    if fn in (None, "original"):
        return math.sqrt(max(1.0, A / B))
    if fn == "match_rms_adamw":
        return 0.2 * math.sqrt(max(A, B))
    return 1.0


# ---------------------------------------------------------------------------------------------
# Gram Newton-Schulz
# ---------------------------------------------------------------------------------------------

def _ns_cpu(X: torch.Tensor, coeffs, steps, eps, reset, round_bf16: bool = False) -> torch.Tensor:
    """The same recurrence on the CPU in fp32; ``round_bf16`` rounds every product to bf16 the way
    the tcgen05 path stores it (fp32 accumulation, one rounding per output).  X is [B, M, N], M <= N."""
    a, b, c = coeffs
    rd = (lambda t: t.to(torch.bfloat16).float()) if round_bf16 else (lambda t: t)
    X = rd(X.float())
    R32 = X @ X.transpose(-1, -2)
    n2 = torch.diagonal(R32, dim1=-2, dim2=-1).sum(-1).clamp(min=eps * eps).view(-1, 1, 1)
    R = rd(R32 / n2)
    Q = None
    first = True
    I = torch.eye(X.shape[1]).expand_as(R)
    for i in range(steps):
        if i == reset and Q is not None:
            if first:
                Q = rd(Q / n2.sqrt())
                first = False
            X = rd(Q @ X)
            R = rd(X @ X.transpose(-1, -2))
            Q = None
        Z = rd(c * (R @ R) + b * R)
        Q = rd(a * I + Z) if Q is None else rd(Q @ Z + a * Q)
        if i < steps - 1 and (i + 1) != reset:
            RZ = rd(R @ Z + a * R)
            R = rd(Z @ RZ + a * RZ)
    if first:
        Q = rd(Q / n2.sqrt())
    return rd(Q @ X)


def gram_newton_schulz(G: torch.Tensor, coeffs=NS_COEFFS, steps: int = NS_STEPS, eps: float = NS_EPS,
                       reset: int = NS_RESET) -> torch.Tensor:
    """Orthogonalise each matrix of ``G`` ``[B, R, C]`` (bf16 on CUDA); returns the same layout.

    The Gram matrix is taken over the smaller side: ``X = G`` when ``R <= C`` else ``X = G^T``.
    """
    if G.dim() == 2:
        return gram_newton_schulz(G.unsqueeze(0), coeffs, steps, eps, reset)[0]
    Bn, Rr, Cc = G.shape
    transpose = Rr > Cc
    if not G.is_cuda:
        X = G.transpose(-1, -2) if transpose else G
        out = _ns_cpu(X, coeffs, steps, eps, reset)
        return (out.transpose(-1, -2) if transpose else out).to(G.dtype)
    E = ext()
    a, b, c = coeffs
    G = G.to(torch.bfloat16).contiguous()
    M = Cc if transpose else Rr
    dev = G.device
    R32 = torch.empty(Bn, M, M, device=dev, dtype=torch.float32)
    if transpose:  # R = G^T G  (both operands MN-major views of G)
        E.gemm_batched(G, G, R32, False, False, 1.0, 0.0, None)
    else:          # R = G G^T
        E.gemm_batched(G, G, R32, True, True, 1.0, 0.0, None)
    norm2 = torch.empty(Bn, device=dev, dtype=torch.float32)
    E.ns_trace(R32, norm2)
    R = torch.empty(Bn, M, M, device=dev, dtype=torch.bfloat16)
    E.ns_gram_normalize(R32, norm2, eps, R)
    del R32
    Z = torch.empty_like(R)
    RZ = torch.empty_like(R)
    Rn = torch.empty_like(R)
    Q = None
    first_segment = True
    X = G

    def apply_q(Qm, Xm):
        out = torch.empty_like(Xm)
        if transpose:   # X^T <- X^T Q^T  (= (Q X)^T)
            E.gemm_batched(Xm, Qm, out, True, True, 1.0, 0.0, None)
        else:           # X <- Q X       (X as an MN-major B operand)
            E.gemm_batched(Qm, Xm, out, True, False, 1.0, 0.0, None)
        return out

    for i in range(steps):
        if i == reset and Q is not None:
            if first_segment:
                E.ns_scale_by_invnorm(Q, norm2, eps)
                first_segment = False
            X = apply_q(Q, X)
            if transpose:
                E.gemm_batched(X, X, R, False, False, 1.0, 0.0, None)
            else:
                E.gemm_batched(X, X, R, True, True, 1.0, 0.0, None)
            Q = None
        # M x M products use B as an MN-major operand (true A @ B): the Gram iterates are only
        # symmetric up to rounding, and A @ B^T would feed that asymmetry back every step
        E.gemm_batched(R, R, Z, True, False, c, b, R)          # Z = c R R + b R
        if Q is None:
            Q = Z.clone()
            E.ns_add_diag(Q, a)                                  # Q = a I + Z
        else:
            Qn = torch.empty_like(Q)
            E.gemm_batched(Q, Z, Qn, True, False, 1.0, a, Q)    # Q = Q Z + a Q
            Q = Qn
        if i < steps - 1 and (i + 1) != reset:
            E.gemm_batched(R, Z, RZ, True, False, 1.0, a, R)    # RZ = R Z + a R
            E.gemm_batched(Z, RZ, Rn, True, False, 1.0, a, RZ)  # R = Z RZ + a RZ
            R, Rn = Rn, R
    if first_segment:
        E.ns_scale_by_invnorm(Q, norm2, eps)
    return apply_q(Q, X)


# ---------------------------------------------------------------------------------------------
# grouping of Muon work
# ---------------------------------------------------------------------------------------------

def chunk_view(t: torch.Tensor, n_chunks: int) -> torch.Tensor:
    """``[R, C]`` -> ``[n_chunks, R / n_chunks, C]`` (dim-0 chunks)."""
    R, C = t.shape
    if R % n_chunks:
        raise ValueError(f"{R} rows are not divisible into {n_chunks} chunks")
    return t.view(n_chunks, R // n_chunks, C)
