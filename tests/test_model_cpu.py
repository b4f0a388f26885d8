"""Denoiser / refiner on the CPU oracle path: shapes, parameter layout and numerics vs the reference modules."""
import os
import sys

import pytest
import torch

from trenowanie_generatora_obrazkow_b200.models import (SIZES, DenoiserConfig, LMEncoderConfig, benchmark_configs,
                                                        build_models)
from trenowanie_generatora_obrazkow_b200.train.flow import FlowModel

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _ref_model():
    if not os.path.isdir(os.path.join(REF, "aurora")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF not in sys.path:  # appended: the repository's own same-named scripts keep priority
        sys.path.append(REF)
    import aurora.model as am
    return am


def small_cfgs():
    den = DenoiserConfig(dim=128, depth=2, heads=2, mlp_hidden=256, text_dim=128, latent_channels=32, latent_size=8)
    te = LMEncoderConfig(lm_dim=96, dim=128, depth=2, heads=2, kv_heads=1, head_dim=64, mlp_hidden=256, max_tokens=16,
                         backend="states")
    return den, te


def test_denoiser_matches_reference_forward():
    am = _ref_model()
    torch.manual_seed(0)
    cfg = DenoiserConfig(dim=128, depth=2, heads=2, mlp_hidden=256, text_dim=96, latent_channels=32, latent_size=8,
                         rope_ref=16, micro_cond=256)
    from trenowanie_generatora_obrazkow_b200.models.dit import Denoiser
    ours = Denoiser(cfg)
    ref = am.Denoiser(am.DenoiserConfig(**{k: getattr(cfg, k) for k in am.DenoiserConfig.__dataclass_fields__}))
    ref.init_weights()
    # randomise everything (the zero inits would hide mistakes)
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.05)
    missing = ours.load_state_dict(ref.state_dict(), strict=True)
    z = torch.randn(3, 32, 8, 8)
    t = torch.rand(3)
    text = torch.randn(3, 10, 96)
    valid = torch.ones(3, 10, dtype=torch.bool)
    valid[1, 4:] = False
    valid[2, 1:] = False
    a = ours(z, t, text, valid)
    b = ref(z, t, text, valid)
    assert torch.allclose(a, b, atol=1e-4, rtol=1e-4), (a - b).abs().max()
    a2, ha = ours(z, t, text, valid, hidden_at=1)
    b2, hb = ref(z, t, text, valid, hidden_at=1)
    assert torch.allclose(ha, hb, atol=1e-4, rtol=1e-4)


def test_refiner_matches_reference_forward():
    am = _ref_model()
    import aurora.slayer as asl
    torch.manual_seed(1)
    _, te_cfg = small_cfgs()
    from trenowanie_generatora_obrazkow_b200.models.text import LM_NULL, LM_PAD, LMTextEncoder
    ours = LMTextEncoder(te_cfg)
    ref = asl.LMTextEncoder(te_cfg, with_lm=False)
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.05)
    ours.load_state_dict(ref.state_dict(), strict=True)
    ids = torch.randint(0, 1000, (3, 16))
    ids[1, 9:] = LM_PAD
    ids[2, :] = LM_PAD
    ids[2, 0] = LM_NULL
    states = torch.randn(3, 16, 96)
    a, va = ours(ids, lm_states=states)
    b, vb = ref(ids, lm_states=states)
    assert torch.equal(va, vb)
    # padded query rows differ only through masked-out keys: compare the valid rows
    assert torch.allclose(a[va], b[vb], atol=1e-4, rtol=1e-4)


def test_param_layout_matches_reference_presets():
    am = _ref_model()
    from trenowanie_generatora_obrazkow_b200.models.dit import Denoiser
    for name in ("50m", "116m"):
        assert ({k: v.shape for k, v in Denoiser(SIZES[name]).state_dict().items()}
                == {k: v.shape for k, v in am.Denoiser(am.SIZES[name]).state_dict().items()})
    den_cfg, te_cfg = benchmark_configs("tiny")
    te, den = build_models(den_cfg, te_cfg)
    ref = am.Denoiser(am.DenoiserConfig(**{k: getattr(den_cfg, k) for k in am.DenoiserConfig.__dataclass_fields__}))
    assert {k: v.shape for k, v in den.state_dict().items()} == {k: v.shape for k, v in ref.state_dict().items()}


def test_every_param_gets_gradient_after_steps():
    """Port of the dead-branch check: after a few optimizer steps every trainable parameter has a non-zero grad."""
    torch.manual_seed(0)
    den_cfg, te_cfg = small_cfgs()
    te, den = build_models(den_cfg, te_cfg)
    model = FlowModel(te, den)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    for _ in range(4):  # gated / zero-init branches need a few steps before every grad is non-zero
        x0 = torch.randn(2, 32, 8, 8)
        eps = torch.randn_like(x0)
        t = torch.rand(2)
        states = torch.randn(2, 16, 96)
        valid = torch.ones(2, 16, dtype=torch.bool)
        opt.zero_grad()
        loss, fm, _, _ = model(x0, t, eps, lm_states=states, valid=valid, is_null=torch.tensor([False, True]))
        loss.backward()
        opt.step()
    dead = [n for n, p in model.named_parameters() if p.grad is None or p.grad.abs().max() == 0]
    assert not dead, dead


def test_tiny_baseline_config_train_step():
    """The tiny headline config on CPU: tiny DiT (576 x 12, 9 heads), 256 tokens, text [4, 64, 1024]: one step with
    Muon (5 NS steps) on the hidden matrices and AdamW elsewhere; the loss is finite and the weights move."""
    from trenowanie_generatora_obrazkow_b200.optim import build_optimizers
    torch.manual_seed(0)
    den_cfg, te_cfg = benchmark_configs("tiny")
    te, den = build_models(den_cfg, te_cfg)
    n = sum(p.numel() for p in den.parameters())
    assert 40e6 < n < 80e6, n
    model = FlowModel(te, den)
    named = [(pre, name, p) for pre, mod in (("te", te), ("den", den)) for name, p in mod.named_parameters()]
    opts, counts = build_optimizers(named, shard=False)
    x0 = torch.randn(4, 128, 16, 16)
    eps = torch.randn_like(x0)
    t = torch.sigmoid(torch.randn(4))
    states = torch.randn(4, 64, 1024)
    before = den.blocks[0].attn.qkv.weight.detach().clone()
    loss, fm, _, _ = model(x0, t, eps, lm_states=states)
    loss.backward()
    for o in opts:
        o.step()
    assert torch.isfinite(loss)
    assert not torch.equal(before, den.blocks[0].attn.qkv.weight)


def test_slayer_gpt_matches_reference():
    """models/slayer.GPT loads the reference GPT's state dict strictly and gives the same hidden states."""
    import os
    import sys
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "aurora")):
        pytest.skip("reference not installed")
    sys.path.insert(0, ref)
    try:
        from types import SimpleNamespace

        from aurora.slayer import GPT as RefGPT
    finally:
        sys.path.remove(ref)
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    cfg = GPTConfig(vocab=512, n_layer=3, n_embd=96, n_head=4, block=64)
    torch.manual_seed(0)
    ref_model = RefGPT(cfg.vocab, cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.block, SimpleNamespace(**vars(cfg)))
    with torch.no_grad():
        for n, p in ref_model.named_parameters():
            if n.endswith("vr_lambda"):
                p.fill_(0.3)
    ours = GPT(cfg)
    ours.load_state_dict(ref_model.state_dict(), strict=True)
    idx = torch.randint(0, cfg.vocab, (2, 17))
    with torch.no_grad():
        a, b = ref_model.hidden(idx, 2), ours.hidden(idx, 2)
    assert torch.allclose(a, b, atol=1e-5), (a - b).abs().max()


def test_slayer_packed_states_match_padded():
    """Packed captions (varlen causal attention, positions restarting per caption) give the padded LM's states for
    every real token, zeros at pads and on null-prompt rows."""
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_NULL, LM_PAD, SlayerFrozenLM
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    torch.manual_seed(0)
    cfg = GPTConfig(vocab=300, n_layer=3, n_embd=64, n_head=4, block=64)
    gpt = GPT(cfg)
    with torch.no_grad():
        for blk in gpt.blocks[1:]:
            blk.vr_lambda.fill_(0.25)
    lm_pad = SlayerFrozenLM(None, skip_last=1, model=gpt, dtype=torch.float32, packed=False)
    lm_pack = SlayerFrozenLM(None, skip_last=1, model=gpt, dtype=torch.float32, packed=True, max_tokens=20)
    ids = torch.randint(0, 300, (4, 12))
    lens = [12, 5, 1, 9]
    for r, n in enumerate(lens):
        ids[r, n:] = LM_PAD
    ids[2, 0] = LM_NULL  # a null prompt: not run
    a, b = lm_pad.states(ids), lm_pack.states(ids)
    assert b.shape == a.shape
    for r, n in enumerate(lens):
        if r == 2:
            assert b[r].abs().max() == 0
            continue
        assert torch.allclose(a[r, :n], b[r, :n], atol=1e-5), (r, (a[r, :n] - b[r, :n]).abs().max())
        assert n == ids.shape[1] or b[r, n:].abs().max() == 0


def test_varlen_attention_oracle_matches_per_sequence_sdpa():
    from trenowanie_generatora_obrazkow_b200.ops import reference as R
    torch.manual_seed(1)
    lens = [7, 1, 13]
    cu = torch.tensor([0, 7, 8, 21], dtype=torch.int32)
    q, k, v = torch.randn(21, 4, 16), torch.randn(21, 2, 16), torch.randn(21, 2, 16)
    out = R.varlen_attention(q, k, v, cu, causal=True, scale=0.25)
    for (a, n) in zip([0, 7, 8], lens):
        qs, ks, vs = q[a:a + n], k[a:a + n].repeat_interleave(2, 1), v[a:a + n].repeat_interleave(2, 1)
        s = torch.einsum("qhd,khd->hqk", qs, ks) * 0.25
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
        ref = torch.einsum("hqk,khd->qhd", s.softmax(-1), vs)
        assert torch.allclose(out[a:a + n], ref, atol=1e-5)
