"""Per-kernel micro-benchmark of the fused sm_100a ops on the 1.24B DiT shapes, with a library baseline per op.

    python -m trenowanie_generatora_obrazkow_b200.ops.microbench --op all
    python -m trenowanie_generatora_obrazkow_b200.ops.microbench --op gemm_qkv --small --iters 2 --warmup 1

Every op is timed with CUDA events on the launching stream, one event pair per launch, after ``--warmup`` untimed
launches; a 256 MiB buffer (twice the L2) is rewritten between timed launches so each launch starts cold. The report
is one JSON line per op: median milliseconds, achieved TFLOP/s (contractions) or GB/s (bandwidth-bound ops, counted
as the algorithmic bytes: every input read once, every output written once), the fraction of the measured peaks in
MEASURED_PEAKS.json (copy bandwidth, cuBLAS bf16 burst) when that file is found, and the same figures for the library
path that computes the same result (cuBLAS through torch.matmul, cuDNN / flash SDPA, eager PyTorch elementwise).
``--small`` shrinks the batch to keep a single launch short (for profiler captures). The reference has no counterpart
(its kernels are Triton / torch.compile generated).
"""
import argparse
import json
import os
import statistics

import torch
import torch.nn.functional as F

from . import reference as R
from ._ext import err_buf, ext

HERE = os.path.dirname(os.path.abspath(__file__))


def measured_peaks():
    for d in (os.getcwd(), os.path.dirname(os.path.dirname(HERE))):
        p = os.path.join(d, "MEASURED_PEAKS.json")
        if os.path.exists(p):
            with open(p) as f:
                return json.load(f)
    return {}


_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def time_op(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def _bf16(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


# ------------------------------------------------------------------------------------------------------------------
# op builders: each returns (ours, library, flops, bytes)
# ------------------------------------------------------------------------------------------------------------------
def gemm_case(M, N, K, a_mn=False, b_mn=False, accumulate=False):
    """C[M, N] = op(A) op(B)^T; a_mn / b_mn: the operand is stored K-rows (MN-major), as in dgrad / wgrad;
    accumulate: fp32 C += (the weight-gradient epilogue)."""
    a = _bf16(K, M) if a_mn else _bf16(M, K)
    b = _bf16(K, N) if b_mn else _bf16(N, K)
    out = torch.zeros(M, N, dtype=torch.float32 if accumulate else torch.bfloat16, device="cuda")
    err = err_buf(a.device)
    A = a.t() if a_mn else a
    B = b if b_mn else b.t()

    def ours():
        ext().gemm(a, b, out, a_mn, b_mn, None, 1.0, 0.0, accumulate, err)

    def lib():
        if accumulate:
            out.add_(torch.matmul(A, B))
        else:
            torch.matmul(A, B, out=out)

    return ours, lib, 2.0 * M * N * K, 2 * (M * K + N * K) + out.element_size() * M * N * (2 if accumulate else 1)


def gemm_i8_case(M, N, K):
    """W8A8: our kind::i8 GEMM with the scales in its epilogue vs torch._int_mm + the scaling (the reference's
    teacher path); counted as 2 M N K integer operations."""
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
    sa, sb = torch.rand(M, device="cuda"), torch.rand(N, device="cuda")
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    err = err_buf(a.device)
    bt = b.T

    def ours():
        ext().gemm_i8(a, b, c, sa, sb, err)

    def lib():
        (torch._int_mm(a, bt).float() * sa[:, None] * sb[None, :]).to(torch.bfloat16)

    return ours, lib, 2.0 * M * N * K, M * K + N * K + 2 * M * N


def attn_case(B, T, H, hd, backward, Tk=None):
    Tk = Tk or T
    q = _bf16(B, T, H, hd)
    k, v = (_bf16(B, Tk, H, hd) for _ in range(2))
    kv_len = torch.full((B,), Tk, dtype=torch.int32, device="cuda")
    scale = hd ** -0.5
    err = err_buf(q.device)
    o, lse = ext().attention_fwd(q, k, v, kv_len, scale, None, err)
    do = _bf16(B, T, H, hd)
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    qt, kt, vt = (x.transpose(1, 2).contiguous().requires_grad_(backward) for x in (q, k, v))
    fl = 4.0 * B * H * T * Tk * hd
    if not backward:
        def ours():
            ext().attention_fwd(q, k, v, kv_len, scale, o, err)

        def lib():
            F.scaled_dot_product_attention(qt, kt, vt, scale=scale)

        return ours, lib, fl, 2 * (2 * B * T + 2 * B * Tk) * H * hd

    ot = F.scaled_dot_product_attention(qt, kt, vt, scale=scale)
    dot = do.transpose(1, 2).contiguous()

    def ours():
        ext().attention_bwd(q, k, v, o, lse, do, kv_len, scale, dq, dk, dv, err)

    def lib():
        torch.autograd.grad(ot, (qt, kt, vt), dot, retain_graph=True)

    return ours, lib, 2.5 * fl, 2 * 8 * B * T * H * hd


def swiglu_gemm_case(M, D, H):
    """Up projection + SwiGLU in one GEMM (sampling path) vs the library GEMM followed by silu * up."""
    x = _bf16(M, D)
    w = _bf16(2 * H, D, scale=D ** -0.5)
    out = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)

    def ours():
        ext().gemm_swiglu(x, w, out, err_buf(x.device))

    def lib():
        ab = x @ w.T
        F.silu(ab[:, :H]) * ab[:, H:]

    return ours, lib, 2.0 * M * 2 * H * D, 2 * (M * D + 2 * H * D + M * H)


def grouped_gemm_case(M, N, K, groups):
    """Grouped GEMM with the device-side tile schedule (uneven groups) vs one library GEMM per group."""
    from .gemm import gemm_grouped
    a = _bf16(M, K)
    b = _bf16(groups, N, K, scale=K ** -0.5)
    g = torch.Generator().manual_seed(3)
    cuts = torch.sort(torch.randint(0, M, (groups - 1,), generator=g)).values
    off = torch.cat([torch.tensor([0]), cuts, torch.tensor([M])]).to(torch.int32)
    offd = off.cuda()
    bounds = off.tolist()

    def ours():
        gemm_grouped(a, b, offd)

    def lib():
        for e in range(groups):
            a[bounds[e]:bounds[e + 1]] @ b[e].T

    return ours, lib, 2.0 * M * N * K, 2 * (M * K + groups * N * K + M * N)


def adanorm_case(B, T, D, backward):
    x, y = _bf16(B, T, D), _bf16(B, T, D)
    gate, shift, scale = (torch.randn(B, D, device="cuda", dtype=torch.bfloat16) * 0.1 for _ in range(3))
    w = torch.ones(D, device="cuda")
    x_new, h, rstd = ext().adanorm_fwd(x, y, gate, w, shift, scale, T, R.EPS)
    dh, dxn = _bf16(B, T, D), _bf16(B, T, D)
    dw = torch.zeros_like(w)
    if not backward:
        def ours():
            ext().adanorm_fwd(x, y, gate, w, shift, scale, T, R.EPS)

        def lib():
            xn = x + gate[:, None] * y
            (F.rms_norm(xn.float(), (D,), w, R.EPS) * (1 + scale[:, None]) + shift[:, None]).to(torch.bfloat16)

        return ours, lib, 0.0, 2 * 4 * B * T * D

    def ours():
        ext().adanorm_bwd(dh, dxn, x_new, rstd, w, dw, scale, y, gate, T)

    xr = x_new.float().requires_grad_(True)
    hr = F.rms_norm(xr, (D,), w, R.EPS) * (1 + scale[:, None].float()) + shift[:, None].float()

    def lib():
        torch.autograd.grad(hr, xr, dh.float(), retain_graph=True)

    return ours, lib, 0.0, 2 * 6 * B * T * D


def swiglu_case(M, H, backward):
    ab = _bf16(M, 2 * H)
    dg = _bf16(M, H)
    if not backward:
        return (lambda: ext().swiglu_fwd(ab)), (lambda: R.swiglu(ab)), 0.0, 2 * 3 * M * H
    abr = ab.detach().requires_grad_(True)
    g = R.swiglu(abr)
    return ((lambda: ext().swiglu_bwd(ab, dg)), (lambda: torch.autograd.grad(g, abr, dg, retain_graph=True)), 0.0,
            2 * 5 * M * H)


def qknorm_case(B, T, H, hd, backward, dq_f32=False):
    C = 3 * H * hd
    qkv = _bf16(B * T, C)
    qw, kw = torch.ones(hd, device="cuda"), torch.ones(hd, device="cuda")
    cos, sin = R.rope_1d_table(T, hd, device="cuda")
    q, k, rq, rk = ext().qknorm_rope_fwd(qkv, H, H, hd, qw, kw, cos, sin, T, R.EPS)
    dq, dk = torch.randn_like(q), torch.randn_like(k)
    if dq_f32:  # the training path: the attention backward's fp32 dq accumulator read directly
        dq = dq.float()
    dqkv = torch.empty_like(qkv)
    dwq, dwk = torch.zeros_like(qw), torch.zeros_like(kw)
    qv = qkv[:, :2 * H * hd].view(B, T, 2 * H, hd)
    if not backward:
        def lib():
            R.apply_rope(F.rms_norm(qv.float(), (hd,), qw, R.EPS), cos, sin).to(torch.bfloat16)

        return ((lambda: ext().qknorm_rope_fwd(qkv, H, H, hd, qw, kw, cos, sin, T, R.EPS)), lib, 0.0,
                2 * 4 * B * T * H * hd)

    def ours():
        ext().qknorm_rope_bwd(qkv, H, H, hd, qw, kw, cos, sin, T, rq, rk, dq, dk, dqkv, dwq, dwk)

    xr = qv.float().requires_grad_(True)
    nr = F.rms_norm(xr, (hd,), qw, R.EPS)

    def lib():
        torch.autograd.grad(nr, xr, torch.cat([dq.view(B, T, H, hd), dk.view(B, T, H, hd)], 2).float(), retain_graph=True)

    return ours, lib, 0.0, (2 * 9 + (4 if dq_f32 else 0)) * B * T * H * hd


def euler_case(B, side, C):
    T = side * side
    z = torch.randn(B, C, side, side, device="cuda")
    v = _bf16(2 * B, T, C)

    def ours():
        ext().euler_cfg(v, z, 0.02, 3.0)

    def lib():
        vu, vc = v.float().chunk(2)
        z.add_((vu + 3.0 * (vc - vu)).transpose(1, 2).reshape(z.shape), alpha=0.02)

    return ours, lib, 0.0, 4 * 2 * B * C * T + 2 * 2 * B * T * C


def ns_case(batch, m, n, steps=5):
    """Muon's quintic Newton-Schulz on a shape bucket: ours with the symmetric GEMM mode for X X^T and A A^T, the
    'library' column the same loop with full products (the symmetric mode switched off). FLOPs: the full math,
    2 m^2 n + 2 m^3 + 2 m^2 n per iteration, so the symmetric saving shows as higher TFLOP/s."""
    from ..optim.newton_schulz import zeropower
    g = torch.randn(batch, m, n, device="cuda")

    def ours():
        zeropower(g, steps)

    def lib():
        ext().set_gemm_syrk(False)
        try:
            zeropower(g, steps)
        finally:
            ext().set_gemm_syrk(True)

    return ours, lib, steps * batch * (4 * m * m * n + 2 * m ** 3), 0


def cases(small):
    B = 8 if small else 32
    T, D, H, hd, MLP = 1024, 2048, 16, 128, 5504
    M = B * T
    return {
        "gemm_qkv": lambda: gemm_case(M, 3 * D, D),
        "gemm_out": lambda: gemm_case(M, D, D),
        "gemm_mlp_up": lambda: gemm_case(M, 2 * MLP, D),
        "gemm_mlp_down": lambda: gemm_case(M, D, MLP),
        "gemm_i8": lambda: gemm_i8_case(M, 3 * D, D),  # W8A8 teacher projection (qkv shape)
        "dgrad_qkv": lambda: gemm_case(M, D, 3 * D, b_mn=True),
        "wgrad_qkv": lambda: gemm_case(3 * D, D, M, a_mn=True, b_mn=True, accumulate=True),
        "wgrad_mlp_down": lambda: gemm_case(D, MLP, M, a_mn=True, b_mn=True, accumulate=True),
        "wgrad_out": lambda: gemm_case(D, D, M, a_mn=True, b_mn=True, accumulate=True),
        "attn_fwd": lambda: attn_case(B, T, H, hd, False),
        "attn_bwd": lambda: attn_case(B, T, H, hd, True),
        "attn_fwd_4k": lambda: attn_case(4 if small else 16, 4096, H, hd, False),  # 1024 px sampling (CFG batch)
        "attn_cross_4k": lambda: attn_case(4 if small else 16, 4096, H, hd, False, Tk=128),  # text cross-attention
        "attn_cross_bwd": lambda: attn_case(B, T, H, hd, True, Tk=128),  # training cross-attention backward
        "adanorm_fwd": lambda: adanorm_case(B, T, D, False),
        "adanorm_bwd": lambda: adanorm_case(B, T, D, True),
        "qknorm_rope_fwd": lambda: qknorm_case(B, T, H, hd, False),
        "qknorm_rope_bwd": lambda: qknorm_case(B, T, H, hd, True),
        "qknorm_rope_bwd_f32dq": lambda: qknorm_case(B, T, H, hd, True, dq_f32=True),
        "swiglu_fwd": lambda: swiglu_case(M, MLP, False),
        "swiglu_bwd": lambda: swiglu_case(M, MLP, True),
        "euler_cfg": lambda: euler_case(8, 64, 128),
        "gemm_swiglu": lambda: swiglu_gemm_case(M, D, MLP),
        "gemm_grouped": lambda: grouped_gemm_case(M, 8192, D, 8),  # MoE experts: up projection of hidden 4096
        # Newton-Schulz buckets of the 1.24B model on one GPU: 2048 x 2048 (q, k, v, out, cross q / out of 24
        # blocks) and 2048 x 5504 (SwiGLU gate / up / down)
        "ns_2048": lambda: ns_case(24 if small else 144, D, D),
        "ns_2048x5504": lambda: ns_case(12 if small else 72, D, MLP),
    }


def report(name, fn_ours, fn_lib, flops, nbytes, iters, warmup, peaks, library=True):
    row = {"op": name}
    for tag, fn in (("ours", fn_ours), ("library", fn_lib if library else None)):
        if fn is None:
            continue
        ms = time_op(fn, iters, warmup)
        r = {"ms": round(ms, 4)}
        if flops:
            tf = flops / ms / 1e9
            r["tflops"] = round(tf, 1)
            if peaks.get("bf16_tflops"):
                r["frac_of_measured_bf16"] = round(tf / peaks["bf16_tflops"], 3)
        else:
            gbs = nbytes / ms / 1e6
            r["gbs"] = round(gbs, 1)
            if peaks.get("hbm_gbs"):
                r["frac_of_measured_hbm"] = round(gbs / peaks["hbm_gbs"], 3)
        row[tag] = r
    return row


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--op", default="all", help="comma-separated op names, or 'all'")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--small", action="store_true")
    p.add_argument("--no-library", action="store_true", help="time only our kernels (profiler captures)")
    p.add_argument("--gemm-pair", type=int, default=-1, help="1 / 0: force the 2-CTA GEMM on / off")
    p.add_argument("--gemm-tma-epilogue", type=int, default=-1, help="1 / 0: force the 2-CTA GEMM's TMA epilogue "
                   "on / off (per-row global stores)")
    p.add_argument("--qknorm-bwd-unroll", type=int, default=0, help="2 / 4: q/k-norm backward heads in flight")
    p.add_argument("--gemm-splitk", type=int, default=-1, help="1 / 0: split-K of the accumulating GEMMs on / off")
    p.add_argument("--gemm-tail", default="", help="comma-separated 1 / 0: the 2-CTA GEMM's tail split on / off; "
                   "every op runs once per setting")
    p.add_argument("--attn-pingpong", default="", help="comma-separated 0 / 1: attention forward softmax groups "
                   "alternate their exponential phases; every op runs once per setting (and per --attn-emu)")
    p.add_argument("--attn-emu", default="", help="comma-separated settings of the attention forward's FMA-pipe "
                   "exponentials (eighths of the key pairs: 0, 2, 3, 4); every op runs once per setting")
    p.add_argument("--attn-poll", default="", help="comma-separated masks (0..7) of attention barrier waits that "
                   "poll instead of suspending (1 MMA thread, 2 softmax / dQ drain, 4 TMA producer); every op runs "
                   "once per mask")
    p.add_argument("--gemm-poll", default="", help="comma-separated masks (0..7) of GEMM barrier waits that poll "
                   "(1 MMA thread, 2 epilogue, 4 TMA producer); every op runs once per mask")
    p.add_argument("--attn-dq-store", default="", help="comma-separated 1 / 0: attention backward with one key block "
                   "stores final dQ tiles (1) or reduce-adds into a zeroed accumulator (0); every op runs per setting")
    p.add_argument("--adanorm-bwd-rows", default="", help="comma-separated 1 / 2: adanorm backward rows per block "
                   "reduction; every op runs once per setting")
    a = p.parse_args(argv)
    torch.manual_seed(0)
    if a.gemm_pair >= 0:
        ext().set_gemm_pair(bool(a.gemm_pair))
    if a.gemm_tma_epilogue >= 0:
        ext().set_gemm_tma_epilogue(bool(a.gemm_tma_epilogue))
    if a.qknorm_bwd_unroll:
        ext().set_qknorm_bwd_unroll(a.qknorm_bwd_unroll)
    if a.gemm_splitk >= 0:
        ext().set_gemm_splitk(bool(a.gemm_splitk))
    peaks = measured_peaks()
    table = cases(a.small)
    names = list(table) if a.op == "all" else a.op.split(",")
    rows = []
    settings = [int(v) for v in a.attn_emu.split(",")] if a.attn_emu else [None]
    pps = [int(v) for v in a.attn_pingpong.split(",")] if a.attn_pingpong else [None]
    polls = [int(v) for v in a.attn_poll.split(",")] if a.attn_poll else [None]
    gpolls = [int(v) for v in a.gemm_poll.split(",")] if a.gemm_poll else [None]
    arows = [int(v) for v in a.adanorm_bwd_rows.split(",")] if a.adanorm_bwd_rows else [None]
    tails = [int(v) for v in a.gemm_tail.split(",")] if a.gemm_tail else [None]
    stores = [int(v) for v in a.attn_dq_store.split(",")] if a.attn_dq_store else [None]
    for emu, pp, poll, gpoll, arow, tail, store in [(e, q, w, g, r, t, d) for d in stores for t in tails for r in arows
                                                    for g in gpolls for w in polls for q in pps for e in settings]:
        if store is not None:
            ext().set_attention_dq_store(bool(store))
        if tail is not None:
            ext().set_gemm_tail_split(bool(tail))
        if arow is not None:
            ext().set_adanorm_bwd_rows(arow)
        if gpoll is not None:
            ext().set_gemm_poll(gpoll)
        if poll is not None:
            ext().set_attention_poll(poll)
        if emu is not None:
            ext().set_attention_fwd_emu(emu)
        if pp is not None:
            ext().set_attention_fwd_pingpong(bool(pp))
        for n in names:
            ours, lib, flops, nbytes = table[n]()
            row = report(n, ours, lib, flops, nbytes, a.iters, a.warmup, peaks, not a.no_library)
            if emu is not None:
                row["attn_emu"] = emu
            if pp is not None:
                row["attn_pingpong"] = pp
            if poll is not None:
                row["attn_poll"] = poll
            if gpoll is not None:
                row["gemm_poll"] = gpoll
            if arow is not None:
                row["adanorm_bwd_rows"] = arow
            if tail is not None:
                row["gemm_tail"] = tail
            if store is not None:
                row["attn_dq_store"] = store
            from ._ext import check_errors
            check_errors()
            print(json.dumps(row), flush=True)
            rows.append(row)
            torch.cuda.empty_cache()
    return rows


if __name__ == "__main__":
    main()
