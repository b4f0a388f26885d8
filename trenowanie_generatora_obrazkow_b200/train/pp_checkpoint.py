"""Checkpoints of a PP x DP flow-matching run in the single-model layout.

Save (reference train_pp.py:1749-1785): replica 0's stages send their parameters and EMA (under the unsplit model's
names) to global rank 0 over a Gloo group; rank 0 writes ``latest.pt`` in the layout train.py, sample_ckpt.py,
export.py and merge.py read (te / den state dicts, the flat EMA list in the unsplit model's ``parameters()``
order). Every learner rank writes its optimizer state to ``opt_stage{s}_rep{r}.pt`` together with the pipeline
layout it belongs to. The commit is two-phase (every ``.tmp`` first, then the renames), so a crash mid-save leaves
the previous checkpoint intact; the ranks agree on the outcome of phase 1 (a rank whose write fails makes every rank
drop its temporaries and raise), and a resume first finishes or undoes a commit a crash interrupted between its phases
(utils/checkpoint.recover_commit).

Resume (reference train_pp.py:1453-1500): any pipeline layout loads the weights and the EMA of ``latest.pt`` by
name; the optimizer state only when the rank's file exists and its layout matches (pp, dp, the stage's block
range) and it was written at the step of ``latest.pt``; otherwise the run stops, unless ``resume_opt_mismatch`` asks
for fresh optimizer state.
"""
import os
from dataclasses import asdict

import torch
import torch.distributed as dist

from ..models import build_models
from ..parallel.pipeline import stage_ranges
from ..utils import checkpoint as ckpt


def layout(tr):
    return dict(pp=tr.pp, dp=tr.dp, stage=tr.stage, blocks=list(stage_ranges(tr.den_cfg.depth, tr.pp,
                                                                             tr.te_cost)[tr.stage]))


def opt_path(out, tr):
    return os.path.join(out, f"opt_stage{tr.stage}_rep{tr.replica}.pt")


def _unsplit_order(den_cfg, te_cfg):
    """[(prefix, name)] of the unsplit model in parameters() order (text encoder first), built on the meta device."""
    with torch.device("meta"):
        te, den = build_models(den_cfg, te_cfg)
    return [("te", n) for n, _ in te.named_parameters()] + [("den", n) for n, _ in den.named_parameters()]


def save(tr, out, step, samples, args, save_group, learner_group, keep=False, extra=None):
    """Collective over the learner ranks. save_group: Gloo group of replica 0's stages (ranks 0 .. pp - 1);
    ``extra``: a dict kept in latest.pt under "extra" (``resume`` puts it on ``tr.ckpt_extra``)."""
    os.makedirs(out, exist_ok=True)
    if hasattr(tr, "before_save"):
        tr.before_save()  # sharded optimizer state into the optimizers (collective over the stage group)
    writes = [(dict(layout=layout(tr), step=step, opts=[o.state_dict() for o in tr.opts]), opt_path(out, tr))]
    latest = os.path.join(out, "latest.pt")
    if tr.replica == 0:
        trainable = [(pre, n) for pre, n, p in tr.named if p.requires_grad]
        payload = dict(params={(pre, n): p.detach().float().cpu() for pre, n, p in tr.named},
                       ema={k: s.detach().float().cpu() for k, s in zip(trainable, tr.ema.shadow)})
        got = [None] * tr.pp if dist.get_rank() == 0 else None
        dist.gather_object(payload, got, dst=0, group=save_group)
        if dist.get_rank() == 0:
            params, ema = {}, {}
            for part in got:
                params.update(part["params"])
                ema.update(part["ema"])
            order = _unsplit_order(tr.den_cfg, tr.te_cfg)
            missing = [k for k in order if k not in params]
            assert not missing, f"pipeline checkpoint: parameters owned by no stage: {missing[:4]}"
            ck = dict(step=step, samples=samples, den_config=asdict(tr.den_cfg), te_config=asdict(tr.te_cfg),
                      te={n: params[(pre, n)] for pre, n in order if pre == "te"},
                      den={n: params[(pre, n)] for pre, n in order if pre == "den"},
                      opts=None, ema=[ema.get(k, params[k]) for k in order], args=dict(args or {}),
                      outer=None, repa_proj=None, pp_layout=dict(pp=tr.pp, dp=tr.dp), extra=dict(extra or {}))
            writes.append((ck, latest))
    ckpt.two_phase_commit(writes, agree=ckpt.agree_all(learner_group))
    if keep and dist.get_rank() == 0:
        ckpt.keep_hardlink(latest, step, out)
    dist.barrier(group=learner_group)


@torch.no_grad()
def resume(tr, out, resume_opt_mismatch=False, log=print, group=None):
    """Load latest.pt (if any) into this rank's stage. Returns (step, samples) or (0, 0) without a checkpoint.
    Collective over ``group`` (the learner ranks) when it is given: global rank 0 first repairs an interrupted commit
    and the others wait for it."""
    if group is not None:
        if dist.get_rank() == 0 and os.path.isdir(out):
            ckpt.recover_commit(out, log)
        dist.barrier(group=group)
    latest = os.path.join(out, "latest.pt")
    if not os.path.exists(latest):
        return 0, 0
    ck = ckpt.load(latest)
    tr.ckpt_extra = dict(ck.get("extra") or {})
    order = _unsplit_order(tr.den_cfg, tr.te_cfg)
    ema_by_name = dict(zip(order, ck["ema"])) if ck.get("ema") and len(ck["ema"]) == len(order) else {}
    for pre, n, p in tr.named:
        p.copy_(ck[pre][n].to(p.device, p.dtype))
    if tr.ema is not None:
        trainable = [(pre, n) for pre, n, p in tr.named if p.requires_grad]
        for k, s in zip(trainable, tr.ema.shadow):
            s.copy_(ema_by_name.get(k, ck[k[0]][k[1]]).to(s.device, s.dtype))
    path = opt_path(out, tr)
    opt = ckpt.load(path) if os.path.exists(path) else None
    same_step = opt is not None and int(opt.get("step", -1)) == int(ck.get("step", 0))
    if opt is not None and opt.get("layout") == layout(tr) and len(opt["opts"]) == len(tr.opts) and same_step:
        for o, st in zip(tr.opts, opt["opts"]):
            ckpt.load_opt_state(o, st)
        if hasattr(tr, "after_load"):
            tr.after_load()
    elif resume_opt_mismatch:
        log(f"[stage {tr.stage} replica {tr.replica}] optimizer state of {path} does not match this pipeline "
            "layout: starting it fresh (--resume-opt-mismatch)")
    else:
        why = ("missing" if opt is None else "written at another step than latest.pt" if not same_step else
               "written by another pipeline layout")
        raise RuntimeError(f"{path}: optimizer state {why}; pass --resume-opt-mismatch to resume the weights with "
                           "fresh optimizer state")
    step = int(ck.get("step", 0))
    tr.step_idx = step
    return step, int(ck.get("samples", 0))


# ---------------------------------------------------------------------------------------------------------------
# WSM merge checkpoints and EMA evaluation of the unsplit model (reference train_pp.py:2450-2462)
# ---------------------------------------------------------------------------------------------------------------
def gather_unsplit(tr, save_group, ema=False):
    """Replica 0's stages send their tensors (``ema``: the EMA where there is one) to global rank 0 under the unsplit
    names. Collective over ``save_group``; returns (te state, den state) on global rank 0, None elsewhere."""
    if tr.replica != 0:
        return None
    trainable = [(pre, n) for pre, n, p in tr.named if p.requires_grad]
    part = {(pre, n): p.detach().float().cpu() for pre, n, p in tr.named}
    if ema and tr.ema is not None:
        part.update({k: s.detach().float().cpu() for k, s in zip(trainable, tr.ema.shadow)})
    got = [None] * tr.pp if dist.get_rank() == 0 else None
    dist.gather_object(part, got, dst=0, group=save_group)
    if dist.get_rank() != 0:
        return None
    merged = {}
    for g in got:
        merged.update(g)
    order = _unsplit_order(tr.den_cfg, tr.te_cfg)
    return ({n: merged[(pre, n)] for pre, n in order if pre == "te"},
            {n: merged[(pre, n)] for pre, n in order if pre == "den"})


def merge_save(tr, out, step, total_steps, save_group):
    """WSM: the raw fp32 weights as merge/step_<step>.pt in train.py's layout (utils/checkpoint.save_merge), written
    by global rank 0. Collective over replica 0's stages."""
    got = gather_unsplit(tr, save_group, ema=False)
    if got is None:
        return None
    path = os.path.join(out, "merge", f"step_{step:07d}.pt")
    os.makedirs(os.path.dirname(path), exist_ok=True)
    ckpt.atomic_save(dict(step=step, total_steps=total_steps, den_config=asdict(tr.den_cfg),
                          te_config=asdict(tr.te_cfg), te=got[0], den=got[1]), path)
    return path


def ema_eval(tr, save_group, val, device):
    """Validation loss of the EMA weights (train/evaluate.py: 4 t buckets and the t in 0.9-1.0 slice) on the unsplit
    model rebuilt on global rank 0. Collective over replica 0's stages; the result dict on rank 0, else None."""
    got = gather_unsplit(tr, save_group, ema=True)
    if got is None or val is None:
        return None
    from .evaluate import evaluate
    te, den = build_models(tr.den_cfg, tr.te_cfg, device=device)
    te.load_state_dict(got[0])
    den.load_state_dict(got[1])
    res = evaluate(te, den, val, device)
    del te, den
    return res

