"""Fused optimizer tail on the GPU: on-device gradient norm + clip coefficient, multi-tensor AdamW with the clip
coefficient, bf16 shadows and the EMA fused in, and the EMA fused into the Muon apply, against torch's
clip_grad_norm_ / AdamW / lerp."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(512, 256), (1000,), (3, 77), (256,), (2048, 64), (5,)]


def _params_and_flat_grads(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ps = [torch.nn.Parameter(torch.randn(*s, device="cuda", generator=g) * 0.1) for s in SHAPES]
    total = sum(p.numel() for p in ps) + 3
    flat = torch.zeros(total, device="cuda")
    o = 1  # odd offsets: some gradient views are not 16-byte aligned (scalar path)
    for p in ps:
        p.grad = flat[o:o + p.numel()].view_as(p)
        p.grad.copy_(torch.randn(p.shape, device="cuda", generator=g))
        o += p.numel()
    return ps, flat


def test_grad_norm_and_coefficient():
    from trenowanie_generatora_obrazkow_b200.optim.adamw import GradNorm
    ps, flat = _params_and_flat_grads(0)
    gn = GradNorm("cuda")
    for clip in (1.0, 1e6):
        norm, coef = gn([p.grad for p in ps], clip)
        want = torch.linalg.vector_norm(torch.cat([p.grad.reshape(-1) for p in ps]))
        torch.testing.assert_close(norm, want, rtol=1e-5, atol=0)
        torch.testing.assert_close(coef[0], (clip / (want + 1e-6)).clamp(max=1.0), rtol=1e-5, atol=0)
    norm2, _ = gn([flat], 1.0)  # the accumulator and counter were reset by the previous launch
    torch.testing.assert_close(norm2, torch.linalg.vector_norm(flat), rtol=1e-5, atol=0)


def test_fused_adamw_with_coef_shadow_and_ema():
    from trenowanie_generatora_obrazkow_b200.ops.fused import bf16_weight
    from trenowanie_generatora_obrazkow_b200.optim.adamw import FusedAdamW
    from trenowanie_generatora_obrazkow_b200.optim.groups import EMA
    pa, _ = _params_and_flat_grads(1)
    pb = [torch.nn.Parameter(p.detach().clone()) for p in pa]
    groups = lambda ps: [dict(params=ps[:3], lr=1e-3, weight_decay=0.1), dict(params=ps[3:], lr=3e-4, weight_decay=0.0)]
    fa = FusedAdamW(groups(pa), betas=(0.9, 0.95), eps=1e-8)
    ref = torch.optim.AdamW(groups(pb), betas=(0.9, 0.95), eps=1e-8, foreach=False)
    ema_a, ema_b = EMA(pa, 0.999), EMA(pb, 0.999)
    for p in pa:
        if p.ndim == 2:
            bf16_weight(p)
    g = torch.Generator(device="cuda").manual_seed(5)
    for step in range(1, 4):
        for a, b in zip(pa, pb):
            a.grad.copy_(torch.randn(a.shape, device="cuda", generator=g))
            b.grad = a.grad.clone()
        coef = torch.tensor([0.5], device="cuda")
        rate = 1 - ema_a.decay_at(step)
        fa.step(coef=coef, ema=ema_a, ema_rate=rate)
        ema_a.update(step)  # nothing left to do: the fused launch covered every parameter
        torch._foreach_mul_([b.grad for b in pb], 0.5)
        ref.step()
        ema_b.update(step)
    torch.cuda.synchronize()
    for a, b, ea, eb in zip(pa, pb, ema_a.shadow, ema_b.shadow):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(fa.state[a]["exp_avg_sq"], ref.state[b]["exp_avg_sq"], rtol=1e-5, atol=1e-9)
        torch.testing.assert_close(ea, eb, rtol=1e-5, atol=1e-6)
        if a.ndim == 2:
            assert torch.equal(bf16_weight(a), a.detach().bfloat16())
    sd = fa.state_dict()  # torch's layout: loads into a plain AdamW
    torch.optim.AdamW(groups([torch.nn.Parameter(p.detach().clone()) for p in pa])).load_state_dict(sd)


def test_muon_apply_updates_the_ema():
    from trenowanie_generatora_obrazkow_b200.optim.groups import EMA
    from trenowanie_generatora_obrazkow_b200.optim.muon import Muon
    torch.manual_seed(0)
    init = [torch.randn(256, 128, device="cuda") * 0.05, torch.randn(384, 128, device="cuda") * 0.05]
    pa = [torch.nn.Parameter(t.clone()) for t in init]
    opt = Muon(pa, lr=0.02, shard=False, splits={pa[1]: [128, 128, 128]})
    ema = EMA(pa, 0.99)
    before = [s.clone() for s in ema.shadow]
    for p in pa:
        p.grad = torch.randn_like(p)
    opt.step(ema=ema, ema_rate=0.25)
    ema.update(1)
    torch.cuda.synchronize()
    for p, s, s0 in zip(pa, ema.shadow, before):
        torch.testing.assert_close(s, s0 + 0.25 * (p.detach() - s0), rtol=1e-5, atol=1e-7)
