"""bf16 GEMMs on the tcgen05 kernel (csrc/gemm.cu), in the three layouts a Linear layer needs.

Reference: every nn.Linear of aurora/model.py:102-188 runs as a cuBLAS GEMM under bf16 autocast; the weight
gradient is accumulated into fp32 ``param.grad``. Here the forward and both gradients call the same kernel with
different operand majors, and the weight gradient is written (or accumulated) in fp32 directly by the epilogue.
"""
import torch

from ._ext import err_buf, ext


def gemm(a, b, out=None, a_mn=False, b_mn=False, d=None, alpha=1.0, beta=0.0, accumulate=False, out_dtype=None):
    """C = alpha * op(A) @ op(B)^T (+ beta * D).

    a: (M, K) if not a_mn else (K, M); b: (N, K) if not b_mn else (K, N); optional leading batch dim on all.
    """
    if not a.is_cuda:
        A = a.float().mT if a_mn else a.float()
        B = b.float() if b_mn else b.float().mT
        c = alpha * (A @ B)
        if d is not None:
            c = c + beta * d.float()
        if out is not None:
            if accumulate:
                out += c.to(out.dtype)
            else:
                out.copy_(c)
            return out
        return c.to(out_dtype or a.dtype)
    M = a.shape[-1] if a_mn else a.shape[-2]
    N = b.shape[-1] if b_mn else b.shape[-2]
    if out is None:
        out = torch.empty(*a.shape[:-2], M, N, device=a.device, dtype=out_dtype or torch.bfloat16)
    ext().gemm(a, b, out, a_mn, b_mn, d, float(alpha), float(beta), accumulate, err_buf(a.device))
    return out


def linear_fwd(x2d, w):
    """y = x @ w^T; x (M, K) bf16, w (N, K) bf16."""
    return gemm(x2d, w)


def linear_dgrad(dy2d, w):
    """dx = dy @ w; dy (M, N), w (N, K) -> (M, K)."""
    return gemm(dy2d, w, b_mn=True)


def linear_wgrad(dy2d, x2d, out=None, accumulate=False):
    """dW = dy^T @ x in fp32; dy (M, N), x (M, K) -> (N, K). accumulate: out += dW."""
    if out is None:
        out = torch.empty(dy2d.shape[-1], x2d.shape[-1], device=dy2d.device, dtype=torch.float32)
    return gemm(dy2d, x2d, out=out, a_mn=True, b_mn=True, accumulate=accumulate)


def gemm_grouped(a, b, offsets, b_mn=False, row_scale=None):
    """Grouped GEMM: rows [offsets[g], offsets[g + 1]) of a (M, K) times group g of b (G, N, K) (b_mn: (G, K, N))
    -> (M, N). On CUDA one persistent tcgen05 launch whose tile schedule is derived from ``offsets`` on the device
    (reference aurora/moe_triton.py:13-107: grouped expert GEMM with a device-built block schedule); row_scale (M,)
    multiplies the output rows (routing weights)."""
    G = b.shape[0]
    N = b.shape[-1] if b_mn else b.shape[-2]
    if not a.is_cuda:
        out = torch.zeros(a.shape[0], N, dtype=torch.float32)
        off = [int(v) for v in offsets.tolist()]
        for g in range(G):
            lo, hi = off[g], off[g + 1]
            if hi > lo:
                w = b[g].float() if b_mn else b[g].float().T
                out[lo:hi] = a[lo:hi].float() @ w
        if row_scale is not None:
            out *= row_scale.float()[:, None]
        return out.to(a.dtype)
    out = torch.empty(a.shape[0], N, device=a.device, dtype=torch.bfloat16)
    ext().gemm_grouped(a.contiguous(), b.contiguous(), offsets.to(device=a.device, dtype=torch.int32).contiguous(),
                       out, b_mn, None if row_scale is None else row_scale.float().contiguous(), err_buf(a.device))
    return out
