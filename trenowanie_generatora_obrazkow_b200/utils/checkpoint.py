"""Checkpoint files compatible with the reference's layout.

``latest.pt`` (reference train.py:819-831, train_pp.py:1749-1785) holds: step, samples, den_config, te_config,
te / den state dicts (fp32, CPU), opts (optimizer state dicts, or None when they live in per-stage files), ema (a
flat list: text-encoder parameters then denoiser parameters, in ``parameters()`` order), args, outer (DiLoCo outer
optimizer) and repa_proj. ``snap_<step>.pt`` keeps weights + EMA; ``merge/step_<step>.pt`` keeps raw weights for
WSM merging. Pipeline runs write one ``opt_stage{s}.pt`` per stage and commit in two phases (all ``.tmp`` files
first, then the renames), so a failed write leaves the previous state intact. Every write is ``.tmp`` +
``os.replace``.
"""
import os
from dataclasses import asdict

import torch


def _sd(module):
    return {k: v.detach().cpu() for k, v in module.state_dict().items()}


def atomic_save(obj, path):
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)


def ema_list(te, den, ema):
    """The EMA as the reference's flat list (te params then den params). ``ema``: an optim.EMA over
    list(te.parameters()) + list(den.parameters()) or None (then the live weights are used)."""
    if ema is None:
        return [p.detach().float().cpu() for p in list(te.parameters()) + list(den.parameters())]
    return [s.detach().float().cpu() for s in ema.shadow]


def save_latest(path, step, samples, den_cfg, te_cfg, te, den, opts, ema, args=None, outer=None, repa_proj=None,
                extra=None):
    ck = dict(step=step, samples=samples, den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=_sd(te),
              den=_sd(den), opts=None if opts is None else [o.state_dict() for o in opts],
              ema=ema_list(te, den, ema), args=dict(args or {}), outer=outer,
              repa_proj=_sd(repa_proj) if repa_proj is not None else None)
    if extra:
        ck.update(extra)
    atomic_save(ck, path)
    return ck


def save_snapshot(out_dir, step, den_cfg, te_cfg, te, den, ema):
    path = os.path.join(out_dir, f"snap_{step:07d}.pt")
    atomic_save(dict(step=step, den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=_sd(te), den=_sd(den),
                     ema=ema_list(te, den, ema)), path)
    return path


def save_merge(out_dir, step, total_steps, den_cfg, te_cfg, te, den):
    """WSM: raw (non-EMA) fp32 weights for merge.py."""
    d = os.path.join(out_dir, "merge")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"step_{step:07d}.pt")
    atomic_save(dict(step=step, total_steps=total_steps, den_config=asdict(den_cfg), te_config=asdict(te_cfg),
                     te=_sd(te), den=_sd(den)), path)
    return path


def two_phase_commit(writes, barrier=None):
    """writes: [(obj, path)] written to .tmp; after ``barrier()`` (every rank's temporaries are complete) all are
    renamed. A crash before the renames leaves every previous file untouched."""
    for obj, path in writes:
        torch.save(obj, path + ".tmp")
    if barrier is not None:
        barrier()
    for _, path in writes:
        os.replace(path + ".tmp", path)


def keep_hardlink(path, step, out_dir):
    """Keep ``latest.pt`` of this step as step_<step>.pt without copying (hard link; latest.pt is replaced
    atomically later, so the linked inode stays intact)."""
    kept = os.path.join(out_dir, f"step_{step:07d}.pt")
    if os.path.exists(kept + ".tmp"):
        os.remove(kept + ".tmp")
    os.link(path, kept + ".tmp")
    os.replace(kept + ".tmp", kept)
    return kept


def load(path, map_location="cpu"):
    return torch.load(path, map_location=map_location, weights_only=False, mmap=True)


def load_opt_state(opt, state):
    """Restore optimizer state but keep the current hyper-parameters (reference train.py:540-546)."""
    fresh = [{k: v for k, v in g.items() if k != "params"} for g in opt.param_groups]
    opt.load_state_dict(state)
    for g, f in zip(opt.param_groups, fresh):
        g.update(f)


@torch.no_grad()
def load_weights(ck, te, den, strict=True, use_ema=False):
    """Load te / den from a checkpoint dict; use_ema: copy the flat EMA list instead of the raw weights."""
    if use_ema and ck.get("ema"):
        params = list(te.parameters()) + list(den.parameters())
        assert len(params) == len(ck["ema"]), "checkpoint EMA does not match the model"
        for p, e in zip(params, ck["ema"]):
            p.copy_(e.to(p.device, p.dtype))
        return
    te.load_state_dict(ck["te"], strict=strict)
    den.load_state_dict(ck["den"], strict=strict)
