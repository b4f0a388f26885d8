"""Quintic Newton-Schulz orthogonalisation for Muon, batched over same-shape matrices.

Iteration (Keller Jordan's Muon; reference aurora/muon.py:25-39 and aurora/ns_triton.py:63-81):
    X <- G / (||G||_F + 1e-7) (bf16, transposed so that rows <= cols)
    5 x:  A = X X^T ;  B = b A + c A A ;  X = a X + B X         (a, b, c) = (3.4445, -4.7750, 2.0315)

On CUDA every product is one launch of the tcgen05 GEMM (csrc/gemm.cu) with the affine terms fused into its
epilogue (``alpha * acc + beta * D``): A A is formed as A A^T (A is symmetric), and B X reads X MN-major, so no
transposes are materialised inside the loop. The two symmetric products (X X^T and c A A^T + b A) run in the
GEMM's symmetric mode (``gemm_syrk``): only the 256-row tile blocks on and below the diagonal are computed and
each off-diagonal block is stored twice, which halves their tensor work (reference aurora/ns_triton.py:20-48
computes the lower triangle the same way).
"""
import torch

from ..ops.gemm import gemm

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def zeropower_reference(G, steps=5):
    """fp32-or-bf16 PyTorch version (CPU path and test oracle); works batched."""
    a, b, c = NS_COEFFS
    X = G.bfloat16()
    transposed = G.size(-2) > G.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    if transposed:
        X = X.mT
    return X


def zeropower(G, steps=5, out=None, scratch_ok=False):
    """Orthogonalise the last two dims of G (B, m, n) or (m, n); returns bf16 (written into `out` when given).
    scratch_ok: G is a contiguous bf16 buffer the caller does not need afterwards, so the Frobenius normalisation
    happens in place (one fp32-accumulated norm pass and one scaling pass over the bf16 data)."""
    if not G.is_cuda:
        X = zeropower_reference(G, steps)
        return out.copy_(X) if out is not None else X
    a, b, c = NS_COEFFS
    squeeze = G.dim() == 2
    X = G.unsqueeze(0) if squeeze else G
    transposed = X.size(-2) > X.size(-1)
    if scratch_ok and X.dtype == torch.bfloat16 and X.is_contiguous():
        norm = torch.linalg.vector_norm(X, dim=(-2, -1), keepdim=True, dtype=torch.float32)
        X.mul_(1.0 / (norm + 1e-7))  # fp32 math, one rounding to bf16 (the transpose comes free below)
        if transposed:
            X = X.mT.contiguous()
    else:
        if transposed:
            X = X.mT
        norm = X.float().norm(dim=(-2, -1), keepdim=True)
        X = (X.float() / (norm + 1e-7)).to(torch.bfloat16).contiguous()
    n, m, k = X.shape
    A = torch.empty(n, m, m, device=X.device, dtype=torch.bfloat16)
    Bm = torch.empty_like(A)
    final = None
    if out is not None and not transposed:
        final = out.view(n, m, k)
    Y = torch.empty_like(X)
    from ..ops._ext import err_buf, ext
    err = err_buf(X.device)
    for i in range(steps):
        ext().gemm_syrk(X, A, None, 1.0, 0.0, err)     # A = X X^T            (symmetric)
        ext().gemm_syrk(A, Bm, A, c, b, err)           # B = c A A^T + b A    (symmetric)
        dst = final if (final is not None and i == steps - 1) else Y
        gemm(Bm, X, out=dst, b_mn=True, d=X, alpha=1.0, beta=a)  # X = B X + a X
        X, Y = dst, X
    if transposed:
        X = X.mT
    if out is not None:
        if final is None:
            out.view(X.shape).copy_(X)
        return out
    return X.squeeze(0) if squeeze else X


def rownorm(G, eps=1e-7):
    """Row-wise step of periodic row-wise Muon (arXiv:2608.20818, reference aurora/muon.py:42-52): in the wide
    orientation every row is scaled to unit norm. Works batched; returns bf16."""
    X = G.float()
    transposed = X.size(-2) > X.size(-1)
    if transposed:
        X = X.mT
    X = X / X.norm(dim=-1, keepdim=True).clamp_min(eps)
    if transposed:
        X = X.mT
    return X.bfloat16()
