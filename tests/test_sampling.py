"""Euler / CFG sampler: CPU path against an explicit re-statement of the update, fused CUDA step against torch."""
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig, build_models
from trenowanie_generatora_obrazkow_b200.sampling.euler import encode_prompts, sample, sample_latents, time_grid


def tiny(device="cpu"):
    den = DenoiserConfig(dim=128, depth=2, heads=2, mlp_hidden=256, text_dim=128, latent_channels=32, latent_size=8)
    te = LMEncoderConfig(lm_dim=64, dim=128, depth=1, heads=2, kv_heads=1, head_dim=64, mlp_hidden=256, max_tokens=16,
                         backend="states")
    torch.manual_seed(0)
    te_m, den_m = build_models(den, te, device=device)
    with torch.no_grad():  # non-zero head so the velocity is not identically zero
        den_m.patch_out.weight.normal_(0, 0.05)
        for b in den_m.blocks:
            b.cross.out.weight.normal_(0, 0.05)
    return te_m, den_m


def test_time_grid_shift():
    ts = time_grid(4, 3.0)
    u = torch.linspace(1, 0, 5)
    assert torch.allclose(ts, 3 * u / (1 + 2 * u))
    assert ts[0] == 1 and ts[-1] == 0


def test_cpu_sampler_matches_explicit_loop():
    te, den = tiny()
    states = torch.randn(3, 16, 64)
    text, lens, null, nlen = encode_prompts(te, lm_states=states)
    noise = torch.randn(3, 32, 8, 8)
    z = sample_latents(den, text, lens, null, nlen, steps=3, cfg=2.5, shift=2.0, noise=noise)
    ref = noise.clone()
    ts = time_grid(3, 2.0)
    for k in range(3):
        tt = torch.full((3,), ts[k].item())
        vu = den(ref, tt, null.expand(3, -1, -1), text_len=nlen.expand(3))
        vc = den(ref, tt, text, text_len=lens)
        ref = ref + (ts[k + 1] - ts[k]) * (vu + 2.5 * (vc - vu))
    assert torch.allclose(z, ref, atol=1e-4, rtol=1e-4)


def test_sample_is_seeded_per_prompt_batch():
    te, den = tiny()
    states = torch.randn(4, 16, 64)
    a = sample(te, den, steps=2, cfg=3.0, seed=5, batch=2, lm_states=states)
    b = sample(te, den, steps=2, cfg=3.0, seed=5, batch=2, lm_states=states)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_fused_euler_cfg_matches_torch():
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    torch.manual_seed(0)
    B, C, H, W = 3, 128, 16, 24
    out = torch.randn(2 * B, H * W, C, device="cuda").bfloat16()
    z = torch.randn(B, C, H, W, device="cuda")
    ref = z + 0.1 * (lambda v: v[:B] + 3.0 * (v[B:] - v[:B]))(out.float().transpose(1, 2).reshape(2 * B, C, H, W))
    ext().euler_cfg(out, z, 0.1, 3.0)
    assert torch.allclose(z, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.gpu
def test_gpu_sampler_close_to_cpu():
    te, den = tiny()
    states = torch.randn(2, 16, 64)
    te_g, den_g = tiny("cuda")
    den_g.load_state_dict(den.state_dict())
    te_g.load_state_dict(te.state_dict())
    # CPU and GPU generators draw different noise: share one noise tensor
    text, lens, null, nlen = encode_prompts(te, lm_states=states)
    tg, lg, ng, nlg = encode_prompts(te_g, lm_states=states.cuda())
    noise = torch.randn(2, 32, 8, 8)
    a = sample_latents(den, text, lens, null, nlen, steps=4, cfg=3.0, noise=noise)
    b = sample_latents(den_g, tg, lg, ng, nlg, steps=4, cfg=3.0, noise=noise.cuda())
    assert ((a - b.cpu()).norm() / a.norm()) < 3e-2
