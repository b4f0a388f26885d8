"""Fused sm_100a ops (forward and backward) vs fp32 PyTorch references of the same math."""
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.ops import fused as Fz
from trenowanie_generatora_obrazkow_b200.ops import reference as R

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("D,T,with_res,with_gate,with_mod", [(2048, 256, True, True, True), (576, 64, True, False, False),
                                                             (1024, 128, False, False, True), (3072, 96, True, True, True)])
def test_adanorm(D, T, with_res, with_gate, with_mod):
    torch.manual_seed(0)
    B = 3
    x = torch.randn(B, T, D, device="cuda").bfloat16().requires_grad_()
    y = torch.randn(B, T, D, device="cuda").bfloat16().requires_grad_() if with_res else None
    mod = (0.3 * torch.randn(B, 6, D, device="cuda")).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(D, device="cuda")).requires_grad_()
    gout = [torch.randn(B, T, D, device="cuda").bfloat16(), torch.randn(B, T, D, device="cuda").bfloat16()]

    def run(x, y, mod, w, cuda):
        gate = mod[:, 2] if with_gate else None
        shift, scale = (mod[:, 0], mod[:, 1]) if with_mod else (None, None)
        if cuda:
            return Fz.adanorm(x, y, gate, w, shift, scale)
        xf = x.float()
        xn = xf if y is None else xf + (y.float() if gate is None else gate.float()[:, None] * y.float())
        h = R.rmsnorm(xn, w)
        if with_mod:
            h = h * (1 + scale.float()[:, None]) + shift.float()[:, None]
        return xn, h

    ins = [x, y, mod, w]
    xs = [t.detach().clone().requires_grad_() if t is not None else None for t in ins]
    outs = run(*xs, True)
    if with_res:
        torch.autograd.backward(list(outs), gout)
    else:
        torch.autograd.backward([outs[1]], [gout[1]])
    xr = [t.detach().clone().requires_grad_() if t is not None else None for t in ins]
    refs = run(*xr, False)
    if with_res:
        torch.autograd.backward(list(refs), [g.float() for g in gout])
    else:
        torch.autograd.backward([refs[1]], [gout[1].float()])
    assert rel(outs[1], refs[1]) < 1.5e-2
    if with_res:
        assert rel(outs[0], refs[0]) < 1e-2
    for a, b in zip(xs, xr):
        if a is None or b.grad is None:
            continue
        assert a.grad is not None
        assert rel(a.grad, b.grad) < 3e-2, (a.shape, rel(a.grad, b.grad))


@pytest.mark.parametrize("hd,hq,hkv,norm,rope,T,kv_mask", [(128, 4, 4, True, True, 256, False),
                                                          (64, 6, 2, False, True, 77, True),
                                                          (128, 2, 2, True, False, 130, False),
                                                          (64, 9, 3, False, True, 64, True),
                                                          (64, 16, 4, False, True, 128, True)])  # the refiner
def test_self_attention_core(hd, hq, hkv, norm, rope, T, kv_mask):
    torch.manual_seed(1)
    B = 2
    C = (hq + 2 * hkv) * hd
    qkv = torch.randn(B, T, C, device="cuda").bfloat16()
    qw = (1 + 0.1 * torch.randn(hd, device="cuda")) if norm else None
    kw = (1 + 0.1 * torch.randn(hd, device="cuda")) if norm else None
    cos, sin = R.rope_1d_table(T, hd, device="cuda") if rope else (None, None)
    kv_len = torch.tensor([T, max(1, T // 3)], device="cuda", dtype=torch.int32) if kv_mask else None
    do = torch.randn(B, T, hq * hd, device="cuda").bfloat16()

    a = qkv.clone().requires_grad_()
    qa = qw.clone().requires_grad_() if norm else None
    ka = kw.clone().requires_grad_() if norm else None
    o = Fz.self_attention_core(a, hq, hkv, hd, qa, ka, cos, sin, kv_len)
    o.backward(do)

    b = qkv.float().cpu().requires_grad_()
    qb = qw.cpu().requires_grad_() if norm else None
    kb = kw.cpu().requires_grad_() if norm else None
    ref = Fz.self_attention_core(b, hq, hkv, hd, qb, kb,
                                 None if cos is None else cos.cpu(), None if sin is None else sin.cpu(),
                                 None if kv_len is None else kv_len.cpu())
    ref.backward(do.float().cpu())
    assert rel(o.cpu(), ref) < 2e-2
    assert rel(a.grad.cpu(), b.grad) < 4e-2
    if norm:
        assert rel(qa.grad.cpu(), qb.grad) < 4e-2
        assert rel(ka.grad.cpu(), kb.grad) < 4e-2


@pytest.mark.parametrize("D,heads,T,L", [(2048, 16, 256, 128), (576, 9, 100, 40)])
def test_cross_attention_core(D, heads, T, L):
    torch.manual_seed(2)
    B = 3
    q = torch.randn(B, T, D, device="cuda").bfloat16()
    kv = torch.randn(B, L, 2 * D, device="cuda").bfloat16()
    kv_len = torch.tensor([L, 1, L // 2], device="cuda", dtype=torch.int32)
    do = torch.randn(B, T, D, device="cuda").bfloat16()
    qa, kva = q.clone().requires_grad_(), kv.clone().requires_grad_()
    o = Fz.cross_attention_core(qa, kva, heads, kv_len)
    o.backward(do)
    qb, kvb = q.float().cpu().requires_grad_(), kv.float().cpu().requires_grad_()
    ref = Fz.cross_attention_core(qb, kvb, heads, kv_len.cpu())
    ref.backward(do.float().cpu())
    assert rel(o.cpu(), ref) < 2e-2
    assert rel(qa.grad.cpu(), qb.grad) < 4e-2
    assert rel(kva.grad.cpu(), kvb.grad) < 4e-2


def test_swiglu():
    torch.manual_seed(3)
    ab = torch.randn(4, 100, 2 * 1536, device="cuda").bfloat16()
    dg = torch.randn(4, 100, 1536, device="cuda").bfloat16()
    a = ab.clone().requires_grad_()
    g = Fz.swiglu(a)
    g.backward(dg)
    b = ab.float().clone().requires_grad_()
    gr = R.swiglu(b)
    gr.backward(dg.float())
    assert rel(g, gr) < 1e-2
    assert rel(a.grad, b.grad) < 2e-2


def test_linear_grad_accumulates_fp32():
    torch.manual_seed(4)
    lin = torch.nn.Linear(256, 384, bias=False).cuda()
    x = torch.randn(2, 64, 256, device="cuda").bfloat16().requires_grad_()
    for _ in range(2):
        y = Fz.linear(x, lin)
        y.float().square().mean().backward()
    xr = x.detach().float().requires_grad_()
    wr = lin.weight.detach().clone().requires_grad_()
    for _ in range(2):
        (xr @ wr.T).square().mean().backward()
    assert lin.weight.grad.dtype == torch.float32
    assert rel(lin.weight.grad, wr.grad) < 2e-2
    assert rel(x.grad, xr.grad) < 2e-2


@pytest.mark.parametrize("hd,hq,hkv,lens,causal", [(64, 12, 12, [37, 300, 1, 129, 512], True),
                                                    (128, 8, 2, [256, 3, 77, 400], True),
                                                    (128, 4, 4, [100, 260, 17], False)])
def test_varlen_attention(hd, hq, hkv, lens, causal):
    """Packed variable-length (causal) tcgen05 attention against the fp32 per-sequence oracle."""
    torch.manual_seed(0)
    T = sum(lens)
    cu = torch.tensor([0] + lens).cumsum(0).to(torch.int32)
    qkv = torch.randn(T, hq + 2 * hkv, hd, device="cuda").bfloat16()
    q, k, v = qkv.split([hq, hkv, hkv], dim=1)
    out = Fz.varlen_attention(q, k, v, cu.cuda(), causal=causal)
    ref = R.varlen_attention(q.float(), k.float(), v.float(), cu, causal=causal, scale=hd ** -0.5)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


def test_slayer_packed_states_gpu():
    """The frozen Slayer LM packed on the GPU (varlen kernel) matches its padded causal-SDPA states."""
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD, SlayerFrozenLM
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    torch.manual_seed(0)
    gpt = GPT(GPTConfig(vocab=1000, n_layer=2, n_embd=256, n_head=4, block=128))
    lm = SlayerFrozenLM(None, model=gpt, device="cuda", packed=False)
    ids = torch.randint(0, 1000, (3, 96), device="cuda")
    lens = [96, 40, 7]
    for r, n in enumerate(lens):
        ids[r, n:] = LM_PAD
    a = lm.states(ids)
    b = lm.states_packed(ids)
    for r, n in enumerate(lens):
        d = (a[r, :n].float() - b[r, :n].float()).abs().max().item()
        assert d < 0.1 * a[r, :n].float().abs().max().item(), (r, d)


@pytest.mark.parametrize("M,D,H", [(300, 512, 384), (4096, 2048, 5504)])
def test_up_swiglu_fused_matches_separate_ops(M, D, H):
    """Up projection + SwiGLU in one GEMM epilogue (inference) against the GEMM followed by the SwiGLU kernel."""
    torch.manual_seed(0)
    layer = torch.nn.Linear(D, 2 * H, bias=False).cuda()
    x = torch.randn(M, D, device="cuda").bfloat16()
    with torch.no_grad():
        fused = Fz.up_swiglu(x, layer)
        ref = Fz.swiglu(Fz.linear(x, layer))
    err = ((fused.float() - ref.float()).norm() / ref.float().norm()).item()
    assert fused.shape == (M, H) and err < 1e-2, err


@pytest.mark.parametrize("emu,pingpong", [(0, False), (2, False), (3, False), (4, False), (0, True), (3, True)])
@pytest.mark.parametrize("hd,T,logit_scale", [(128, 640, 1.0), (128, 300, 6.0), (64, 520, 3.0)])
def test_attention_fwd_fma_exponentials(emu, pingpong, hd, T, logit_scale):
    """tcgen05 forward with `emu` eighths of its exponentials as FMA-pipe polynomials (and optionally the two
    softmax groups taking turns), against the fp32 oracle: masked keys (-inf logits), wide logit ranges
    (running-max rescales, probabilities that underflow)."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, err_buf, ext
    torch.manual_seed(5)
    B, H = 2, 3
    q = (logit_scale * torch.randn(B, T, H, hd, device="cuda")).bfloat16()
    k = torch.randn(B, T, H, hd, device="cuda").bfloat16()
    v = torch.randn(B, T, H, hd, device="cuda").bfloat16()
    kv_len = torch.tensor([T, T // 2 + 7], device="cuda", dtype=torch.int32)
    scale = hd ** -0.5
    ext().set_attention_fwd_emu(emu)
    ext().set_attention_fwd_pingpong(pingpong)
    try:
        o, lse = ext().attention_fwd(q, k, v, kv_len, scale, None, err_buf(q.device))
        torch.cuda.synchronize()
        check_errors()
    finally:
        ext().set_attention_fwd_emu(-1)  # back to the defaults
        ext().set_attention_fwd_pingpong(False)
    ref = R.attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), kv_len.cpu(), scale)
    assert torch.isfinite(o).all()
    assert rel(o.cpu(), ref) < 1.5e-2


def test_fm_inputs_and_forward_tokens():
    """Fused flow-matching input / target kernel against the eager formulas, and the denoiser fed the token-major
    input against the latent-layout forward."""
    from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig
    from trenowanie_generatora_obrazkow_b200.models.dit import Denoiser
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    torch.manual_seed(7)
    x0 = torch.randn(3, 128, 12, 10, device="cuda")
    eps = torch.randn_like(x0)
    t = torch.rand(3, device="cuda")
    z_tok, target = Fz.fm_inputs(x0, eps, t)
    torch.cuda.synchronize()
    check_errors()
    tt = t.view(-1, 1, 1, 1)
    tok = lambda a: a.flatten(2).transpose(1, 2)
    z_ref = tok((1 - tt) * x0 + tt * eps)
    assert z_tok.dtype == torch.bfloat16 and z_tok.shape == (3, 120, 128)
    assert rel(z_tok, z_ref) < 5e-3
    assert torch.allclose(target, tok(eps - x0), atol=1e-6)
    den = Denoiser(DenoiserConfig(dim=256, depth=2, heads=2, mlp_hidden=704, text_dim=256, latent_size=12)).cuda()
    den.init_weights()
    with torch.no_grad():
        for p in den.parameters():  # non-zero output layers, so the comparison is not trivially exact
            p.add_(0.02 * torch.randn_like(p))
    text = torch.randn(3, 16, 256, device="cuda")
    valid = torch.ones(3, 16, dtype=torch.bool, device="cuda")
    with torch.no_grad():
        v_tok = den.forward_tokens(z_tok, (12, 10), t, text, valid)
        v_ref = den((1 - tt) * x0 + tt * eps, t, text, valid, tokens_out=True)
    assert v_tok.shape == v_ref.shape
    assert rel(v_tok, v_ref) < 1e-2


def _fp32_self_attention(qkv, hq, hkv, hd, qw, kw, cos, sin):
    """fp32 oracle on the GPU (the production shapes are too large for the CPU)."""
    B, T, _ = qkv.shape
    q, k, v = qkv.float().split([hq * hd, hkv * hd, hkv * hd], dim=-1)
    q, k, v = q.view(B, T, hq, hd), k.view(B, T, hkv, hd), v.view(B, T, hkv, hd)
    q, k = R.apply_rope(R.rmsnorm(q, qw), cos, sin), R.apply_rope(R.rmsnorm(k, kw), cos, sin)
    return R.attention(q, k, v, None, hd ** -0.5).reshape(B, T, hq * hd)


def test_self_attention_production_shape():
    """B 4 x T 4096 x 16 heads x 128 (1024 work items of 256 query rows > 148 persistent CTAs: barrier phases and the
    O hand-off between one item's epilogue and the next item's P V are exercised), 2-D RoPE, q/k norm."""
    torch.manual_seed(5)
    B, T, H, hd = 4, 4096, 16, 128
    qkv = torch.randn(B, T, 3 * H * hd, device="cuda").bfloat16()
    qw, kw = 1 + 0.1 * torch.randn(hd, device="cuda"), 1 + 0.1 * torch.randn(hd, device="cuda")
    cos, sin = R.rope_2d_table(64, 64, hd, 0, "cuda")
    do = torch.randn(B, T, H * hd, device="cuda").bfloat16()
    a = qkv.clone().requires_grad_()
    qa, ka = qw.clone().requires_grad_(), kw.clone().requires_grad_()
    o = Fz.self_attention_core(a, H, H, hd, qa, ka, cos, sin)
    o.backward(do)
    b = qkv.float().requires_grad_()
    qb, kb = qw.clone().requires_grad_(), kw.clone().requires_grad_()
    ref = _fp32_self_attention(b, H, H, hd, qb, kb, cos, sin)
    ref.backward(do.float())
    assert rel(o, ref) < 2e-2
    assert rel(a.grad, b.grad) < 4e-2
    assert rel(qa.grad, qb.grad) < 4e-2 and rel(ka.grad, kb.grad) < 4e-2


def test_cross_attention_sampling_shape():
    """16 x 4096 queries against 128 text tokens with per-sample key lengths (the sampling step's cross-attention)."""
    torch.manual_seed(6)
    B, T, D, heads, L = 16, 4096, 2048, 16, 128
    q = torch.randn(B, T, D, device="cuda").bfloat16()
    kv = torch.randn(B, L, 2 * D, device="cuda").bfloat16()
    kv_len = torch.randint(1, L + 1, (B,), device="cuda", dtype=torch.int32)
    with torch.no_grad():
        o = Fz.cross_attention_core(q, kv, heads, kv_len)
        k, v = kv.float().chunk(2, dim=-1)
        ref = R.attention(q.float().view(B, T, heads, D // heads), k.view(B, L, heads, D // heads),
                          v.view(B, L, heads, D // heads), kv_len, (D // heads) ** -0.5).reshape(B, T, D)
    assert rel(o, ref) < 2e-2


def test_ops_from_a_fresh_thread():
    """A thread whose first CUDA work is this extension (an autograd worker thread whose first backward node is the
    attention, a server thread): tensor-map kernels run there and match the main thread's results."""
    import threading
    from trenowanie_generatora_obrazkow_b200.ops._ext import err_buf, ext
    torch.manual_seed(7)
    B, T, H, hd = 2, 256, 4, 128
    q, k, v, do = (torch.randn(B, T, H, hd, device="cuda").bfloat16() for _ in range(4))
    a = torch.randn(512, 256, device="cuda").bfloat16()
    w = torch.randn(384, 256, device="cuda").bfloat16()
    err = err_buf(q.device)

    def run():
        o, lse = ext().attention_fwd(q, k, v, None, hd ** -0.5, None, err)
        dq = torch.empty(q.shape, device="cuda", dtype=torch.float32)
        dk, dv = torch.empty_like(k), torch.empty_like(v)
        ext().attention_bwd(q, k, v, o, lse, do, None, hd ** -0.5, dq, dk, dv, err)
        c = torch.empty(512, 384, device="cuda", dtype=torch.bfloat16)
        ext().gemm(a, w, c, False, False, err=err)
        torch.cuda.synchronize()
        return [o, dq, dk, dv, c]

    out = {}
    t = threading.Thread(target=lambda: out.setdefault("thread", run()))
    t.start()
    t.join()
    main = run()
    assert "thread" in out and err.sum().item() == 0
    for x, y in zip(out["thread"], main):
        torch.testing.assert_close(x, y, rtol=0, atol=1e-3)


def test_cross_attention_backward_single_key_block_and_empty_text():
    """Keys <= 128: the backward stores each dQ tile directly (no accumulator); a sample with no text keys
    (kv_len 0) gets zero output and exactly zero dQ, the others match the fp32 reference."""
    torch.manual_seed(8)
    B, T, D, heads, L = 3, 320, 1024, 8, 96
    q = torch.randn(B, T, D, device="cuda").bfloat16()
    kv = torch.randn(B, L, 2 * D, device="cuda").bfloat16()
    kv_len = torch.tensor([L, 0, 17], device="cuda", dtype=torch.int32)
    do = torch.randn(B, T, D, device="cuda").bfloat16()
    qa, kva = q.clone().requires_grad_(), kv.clone().requires_grad_()
    o = Fz.cross_attention_core(qa, kva, heads, kv_len)
    o.backward(do)
    torch.cuda.synchronize()
    assert torch.count_nonzero(o[1]).item() == 0 and torch.count_nonzero(qa.grad[1]).item() == 0
    keep = torch.tensor([0, 2])
    qb, kvb = q[keep].float().cpu().requires_grad_(), kv[keep].float().cpu().requires_grad_()
    ref = Fz.cross_attention_core(qb, kvb, heads, kv_len[keep].cpu())
    ref.backward(do[keep].float().cpu())
    assert rel(o[keep].cpu(), ref) < 2e-2
    assert rel(qa.grad[keep].cpu(), qb.grad) < 4e-2
    assert rel(kva.grad[keep].cpu(), kvb.grad) < 4e-2
