"""On-policy distillation (OPD): the student regresses a frozen teacher's velocity at states of its OWN Euler
trajectories.

Behaviour of the reference (train_pp.py:782-997, aurora/opd_resolution.py):
* Trajectory grid: K Euler steps on u = [1, 1 - (k - d) / K for k = 1..K-1, 0] with one random offset d ~ U(0, 1)
  per update (so the trained t cover [0, 1], not K fixed values), shifted t = s u / (1 + (s - 1) u).
* Which states are trained: DanceOPD picks floor(Beta(A, B) K) (clamped to K - 1) per state, DiffusionOPD m distinct
  step indices per trajectory.
* Rollout: conditional student velocity (no CFG), stopping each micro-batch at its deepest queried state.
* Targets: the teacher's CFG velocity at the picked (state, t) pairs; the loss is the MSE of the student's
  velocity there. Targets are detached and may be replayed for ``reuse`` updates (fresh student graphs each time).
* State weighting: priorities in [0.5, 1.5] from the previous update's per-state errors, balanced to mean 1 within
  four t bins.
* Resolution schedule: one resolution per fresh batch, drawn identically on every learner from
  Random(seed * 1_000_003 + step * 1009 + 739), with a per-resolution time shift and a token-balanced batch
  multiplier round((res_max / res)^2).
Seeds follow the reference's (seed * 1_000_003 + replica * 1009 + step + 7 for grids and picks).
"""
import math
import random

import numpy as np
import torch
import torch.nn.functional as F


# ------------------------------------------------------------------------------------------------------------------
# grids, picks, weights, resolution schedule
# ------------------------------------------------------------------------------------------------------------------
def opd_grid(K, shift, d, device=None):
    u = torch.cat([torch.ones(1), 1 - (torch.arange(1, K) - d) / K, torch.zeros(1)]).clamp(0, 1).to(device)
    return shift * u / (1 + (shift - 1) * u)


def dance_picks(B, m, K, beta, seed, replica, step):
    u = np.random.default_rng([seed, replica, step, 52]).beta(*beta, size=(B, m))
    return torch.from_numpy((u * K).astype(np.int64)).clamp(max=K - 1)


def diffusion_picks(B, m, K, generator):
    return torch.stack([torch.randperm(K, generator=generator)[:m] for _ in range(B)])


@torch.no_grad()
def state_weights(errors, times):
    """Priorities in [0.5, 1.5] with mean 1 per quarter of t: above-median errors up, below-median down."""
    errors, times = errors.detach().float(), times.detach().float()
    w = torch.ones_like(errors)
    bins = (times * 4).long().clamp(0, 3)
    for b in range(4):
        idx = (bins == b).nonzero(as_tuple=True)[0]
        if idx.numel() < 4:
            continue
        e = errors[idx]
        if not torch.isfinite(e).all():
            continue
        med = e.quantile(0.5)
        lo, hi = e < med, e > med
        nl, nh = lo.sum().float(), hi.sum().float()
        den = torch.maximum(nl, nh).clamp_min(1)
        w[idx] = 1 + 0.5 * (hi.float() * nl - lo.float() * nh) / den
    return w


def batch_resolution(seed, step, resolutions, weights=None, default=256):
    if not resolutions:
        return default
    return random.Random(seed * 1_000_003 + step * 1009 + 739).choices(list(resolutions), weights=weights, k=1)[0]


def resolution_shift(resolution, resolutions=(), shifts=(), shift_ref=0.0, t_shift=1.0, res_max=None):
    if resolutions and shifts:
        return shifts[list(resolutions).index(resolution)]
    if shift_ref:
        return resolution / shift_ref
    if resolutions and res_max:
        return t_shift * resolution / res_max
    return t_shift


def token_batch_multiplier(resolution, res_max):
    """Equal image-token count per batch: round((res_max / res)^2) base batches at a lower resolution."""
    return max(1, round((res_max / resolution) ** 2))


# ------------------------------------------------------------------------------------------------------------------
# teachers
# ------------------------------------------------------------------------------------------------------------------
class DiTTeacher:
    """A frozen denoiser (+ text encoder) as the teacher: CFG velocity v_u + w (v_c - v_u)."""

    def __init__(self, te, den, cfg=3.0):
        self.te, self.den, self.cfg = te.eval().requires_grad_(False), den.eval().requires_grad_(False), cfg

    def request(self, x, t, text_kw, chunks=1, deferred=False):
        """Same interface as a remote teacher's deferred request: computed here (in ``chunks`` row chunks),
        returned by ``collect``."""
        from ..parallel.roles import chunked_velocity
        return chunked_velocity(self, x, t, text_kw, chunks)

    def collect(self, handle):
        return handle

    @torch.no_grad()
    def velocity(self, x, t, text_kw):
        from ..sampling.euler import encode_prompts
        text, lens, null, nlen = encode_prompts(self.te, **text_kw)
        B = x.shape[0]
        v = self.den(torch.cat([x, x]), torch.cat([t, t]), torch.cat([null.expand(B, -1, -1), text]),
                     text_len=torch.cat([nlen.expand(B), lens]).to(torch.int32)).float()
        vu, vc = v.chunk(2)
        return vu + self.cfg * (vc - vu)


# ------------------------------------------------------------------------------------------------------------------
# rollout and training on the states
# ------------------------------------------------------------------------------------------------------------------
@torch.no_grad()
def rollout(den, text, text_len, z, ts, picks, mb):
    """Student's own conditional Euler trajectories from noise z (B, C, h, w) on the grid ts (K + 1); returns the
    states (B, m, C, h, w) at step indices picks (B, m). Each micro-batch stops at its deepest queried state."""
    B, m = picks.shape
    out = torch.empty(B, m, *z.shape[1:], device=z.device)
    z = z.clone().float()
    lasts = [int(picks[j:j + mb].max()) for j in range(0, B, mb)]
    for k in range(int(picks.max()) + 1):
        bi, ri = (picks == k).nonzero(as_tuple=True)
        if len(bi):
            out[bi.to(z.device), ri.to(z.device)] = z[bi.to(z.device)]
        for c, j in enumerate(range(0, B, mb)):
            if k >= lasts[c]:
                continue
            sl = slice(j, j + mb)
            t = ts[k].expand(z[sl].shape[0])
            v = den(z[sl], t, text[sl], text_len=text_len[sl]).float()
            z[sl] = z[sl] + (ts[k + 1] - ts[k]) * v
    return out


def train_on_states(te, den, x, t, target, text_kw, mb, weights=None, errors=None):
    """One backward per micro-batch of (state, t, target); returns the summed unweighted MSE and the count."""
    total, count = 0.0, 0
    for j in range(0, x.shape[0], mb):
        sl = slice(j, j + mb)
        kw = {k: (v[sl] if torch.is_tensor(v) else v) for k, v in text_kw.items()}
        text, valid = te(**kw)
        pred = den(x[sl], t[sl], text, valid).float()
        per = (pred - target[sl]).square().flatten(1).mean(1)
        if errors is not None:
            errors.append(per.detach())
        loss = (per * weights[sl]).mean() if weights is not None else per.mean()
        loss.backward()
        total += per.mean().detach()
        count += 1
    return total, count


class OPDLearner:
    """Fresh OPD batches (rollout -> teacher -> train) and replays of the cached targets."""

    def __init__(self, te, den, teacher, K=8, m=2, method="dance", beta=(5.0, 2.0), shift=6.0, mb=4, reuse=1,
                 weighting=False, seed=0, replica=0):
        self.te, self.den, self.teacher = te, den, teacher
        self.K, self.m, self.method, self.beta, self.shift, self.mb = K, m, method, beta, shift, mb
        self.reuse, self.weighting, self.seed, self.replica = reuse, weighting, seed, replica
        self.cache = None
        self.uses = 0

    def rollout_states(self, step, lm_states, valid, noise, shift):
        """The student's own states of a fresh batch: (states (B m, C, h, w), t (B m), text_kw repeated per state)."""
        B = noise.shape[0]
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + self.replica * 1009 + step + 7)
        if self.method == "dance":
            picks = dance_picks(B, self.m, self.K, self.beta, self.seed, self.replica, step)
        else:
            picks = diffusion_picks(B, self.m, self.K, g)
        d = torch.rand((), generator=g).item()
        ts = opd_grid(self.K, shift, d, noise.device)
        with torch.no_grad():
            text, v = self.te(lm_states=lm_states, valid=valid)
        from ..ops.reference import valid_to_len
        states = rollout(self.den, text, valid_to_len(v), noise, ts, picks, self.mb).flatten(0, 1)
        t = ts[picks.to(noise.device)].flatten()
        rep = lambda a: a.repeat_interleave(self.m, dim=0)
        return states, t, dict(lm_states=rep(lm_states), valid=rep(valid))

    @property
    def needs_fresh(self):
        return self.cache is None or self.uses >= self.reuse

    def install(self, states, t, target, text_kw):
        """A fresh cache (states, times, teacher targets) for the next ``reuse`` updates."""
        self.cache = dict(x=states, t=t, target=target, text_kw=text_kw, errors=None)
        self.uses = 0

    def _prepare(self, step, lm_states, valid, noise, shift):
        states, t, text_kw = self.rollout_states(step, lm_states, valid, noise, shift)
        self.install(states, t, self.teacher.velocity(states, t, text_kw), text_kw)

    def step_grads(self, step, lm_states=None, valid=None, noise=None, shift=None):
        """Accumulate the gradient of one OPD update (fresh batch or replay); returns the mean MSE. The batch
        arguments are only read when a fresh cache is due and none was installed."""
        if self.needs_fresh:
            assert noise is not None, "a fresh OPD batch is due: pass its noise and text states (or install one)"
            self._prepare(step, lm_states, valid, noise, shift or self.shift)
        c = self.cache
        weights = state_weights(torch.cat(c["errors"]), c["t"]) if (self.weighting and c["errors"]) else None
        errors = [] if self.weighting else None
        total, count = train_on_states(self.te, self.den, c["x"], c["t"], c["target"], c["text_kw"], self.mb,
                                       weights, errors)
        c["errors"] = errors
        self.uses += 1
        grads = [p.grad for p in list(self.te.parameters()) + list(self.den.parameters()) if p.grad is not None]
        if grads:
            torch._foreach_div_(grads, count)
        return total / count
