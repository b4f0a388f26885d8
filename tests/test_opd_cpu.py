"""On-policy distillation pieces on CPU: grid, picks, rollout states, state weights, resolution schedule, and a
learner step (fresh batch then replay) against a frozen teacher."""
import torch

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig, build_models
from trenowanie_generatora_obrazkow_b200.ops.reference import valid_to_len
from trenowanie_generatora_obrazkow_b200.train.opd import (DiTTeacher, OPDLearner, batch_resolution, dance_picks,
                                                            opd_grid, rollout, state_weights, token_batch_multiplier)

DEN = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16, latent_size=4)
TE = LMEncoderConfig(lm_dim=32, dim=64, depth=1, heads=1, kv_heads=1, head_dim=64, mlp_hidden=128, max_tokens=8,
                     backend="states")


def _models(seed):
    torch.manual_seed(seed)
    te, den = build_models(DEN, TE)
    with torch.no_grad():
        for p in den.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return te, den


def test_grid_and_picks():
    ts = opd_grid(8, 6.0, 0.3)
    assert ts[0] == 1 and ts[-1] == 0 and (ts[1:] <= ts[:-1]).all()
    p = dance_picks(5, 3, 8, (5.0, 2.0), 0, 0, 1)
    assert p.shape == (5, 3) and p.min() >= 0 and p.max() <= 7
    assert torch.equal(p, dance_picks(5, 3, 8, (5.0, 2.0), 0, 0, 1))


def test_rollout_states_follow_euler():
    te, den = _models(0)
    z = torch.randn(2, 16, 4, 4)
    st = torch.randn(2, 8, 32)
    text, v = te(lm_states=st)
    lens = valid_to_len(v)
    ts = opd_grid(4, 2.0, 0.5)
    picks = torch.tensor([[0, 2], [1, 3]])
    out = rollout(den, text, lens, z, ts, picks, mb=2)
    ref = [z.clone()]
    x = z.clone()
    with torch.no_grad():
        for k in range(3):
            x = x + (ts[k + 1] - ts[k]) * den(x, ts[k].expand(2), text, text_len=lens)
            ref.append(x.clone())
    for b in range(2):
        for j in range(2):
            assert torch.allclose(out[b, j], ref[picks[b, j]][b], atol=1e-5)


def test_state_weights_balanced():
    torch.manual_seed(0)
    err = torch.rand(64)
    t = torch.rand(64)
    w = state_weights(err, t)
    assert w.min() >= 0.5 - 1e-6 and w.max() <= 1.5 + 1e-6
    bins = (t * 4).long().clamp(0, 3)
    for b in range(4):
        if (bins == b).sum() >= 4:
            assert abs(w[bins == b].mean().item() - 1.0) < 1e-5


def test_resolution_schedule():
    rs = [batch_resolution(0, s, (256, 512, 1024)) for s in range(20)]
    assert rs == [batch_resolution(0, s, (256, 512, 1024)) for s in range(20)] and len(set(rs)) > 1
    assert token_batch_multiplier(256, 1024) == 16 and token_batch_multiplier(1024, 1024) == 1


def test_learner_fresh_then_replay():
    te, den = _models(1)
    tte, tden = _models(2)
    teacher = DiTTeacher(tte, tden, cfg=3.0)
    learner = OPDLearner(te, den, teacher, K=4, m=2, method="dance", shift=2.0, mb=2, reuse=2, weighting=True)
    st = torch.randn(2, 8, 32)
    valid = torch.ones(2, 8, dtype=torch.bool)
    noise = torch.randn(2, 16, 4, 4)
    l1 = learner.step_grads(0, st, valid, noise)
    first = learner.cache
    assert any(p.grad is not None and p.grad.abs().sum() > 0 for p in den.parameters())
    l2 = learner.step_grads(1, st, valid, noise)  # replay of the cached targets
    assert learner.cache is first and torch.isfinite(torch.as_tensor(l1)) and torch.isfinite(torch.as_tensor(l2))
    learner.step_grads(2, st, valid, noise)  # reuse exhausted: fresh batch
    assert learner.cache is not first


def test_installed_cache_with_deferred_teacher_matches_the_direct_path():
    """The prefetch path (rollout_states, a deferred teacher request computed in chunks, install) trains on the same
    states and targets as a fresh batch prepared inside step_grads, and a replay step needs no batch."""
    grads = []
    for deferred in (False, True):
        te, den = _models(1)
        tte, tden = _models(2)
        teacher = DiTTeacher(tte, tden, cfg=3.0)
        learner = OPDLearner(te, den, teacher, K=4, m=2, method="dance", shift=2.0, mb=2, reuse=2)
        st = torch.randn(3, 8, 32, generator=torch.Generator().manual_seed(5))
        valid = torch.ones(3, 8, dtype=torch.bool)
        noise = torch.randn(3, 16, 4, 4, generator=torch.Generator().manual_seed(6))
        if deferred:
            states, t, kw = learner.rollout_states(0, st, valid, noise, 2.0)
            learner.install(states, t, teacher.collect(teacher.request(states, t, kw, chunks=4)), kw)
            assert not learner.needs_fresh
            learner.step_grads(0)
        else:
            learner.step_grads(0, st, valid, noise, 2.0)
        grads.append([p.grad.clone() for p in den.parameters() if p.grad is not None])
        for p in den.parameters():
            p.grad = None
        learner.step_grads(1)  # replay: no batch arguments
        assert learner.needs_fresh
    for a, b in zip(*grads):
        assert torch.allclose(a, b, rtol=1e-4, atol=1e-6)
