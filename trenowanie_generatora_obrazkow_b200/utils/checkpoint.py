"""Checkpoint files compatible with the reference's layout.

``latest.pt`` (reference train.py:819-831, train_pp.py:1749-1785) holds: step, samples, den_config, te_config,
te / den state dicts (fp32, CPU), opts (optimizer state dicts, or None when they live in per-stage files), ema (a
flat list: text-encoder parameters then denoiser parameters, in ``parameters()`` order), args, outer (DiLoCo outer
optimizer) and repa_proj. ``snap_<step>.pt`` keeps weights + EMA; ``merge/step_<step>.pt`` keeps raw weights for
WSM merging. Pipeline runs write one ``opt_stage{s}.pt`` per stage and commit in two phases (all ``.tmp`` files
first, then the renames), so a failed write leaves the previous state intact. Every write is ``.tmp`` +
``os.replace``.

Failures (the reference stops on them and is rerun; train.py:819-831, train_pp.py:1749-1785): a write that fails
(a full disk, a killed process) removes its partial ``.tmp`` and re-raises; in a multi-rank commit every rank learns
through ``agree`` whether all parts were written, so a failure on one rank makes every rank drop its temporaries and
raise instead of waiting at a barrier for a rank that will not come. ``recover_commit`` (run before a resume)
finishes or undoes a commit that was interrupted between or during its phases, and an unreadable checkpoint (a
truncated file) raises ``CheckpointError`` naming the file and the checkpoints that are still there.
"""
import glob
import os
import pickle
from dataclasses import asdict

import torch


class CheckpointError(RuntimeError):
    pass


def _remove(path):
    try:
        os.remove(path)
    except FileNotFoundError:
        pass


def _sd(module):
    return {k: v.detach().cpu() for k, v in module.state_dict().items()}


def atomic_save(obj, path):
    """torch.save to ``path`` + ".tmp", then an atomic rename; on any failure the partial temporary is removed and
    the previous ``path`` is left as it was."""
    tmp = path + ".tmp"
    try:
        torch.save(obj, tmp)
        os.replace(tmp, path)
    except BaseException:
        _remove(tmp)
        raise


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


def two_phase_commit(writes, barrier=None, agree=None):
    """writes: [(obj, path)] written to .tmp (phase 1), then all renamed (phase 2). A crash before the renames leaves
    every previous file untouched.

    agree(ok) -> bool (every rank's phase 1 succeeded; a collective, see ``agree_all``) replaces ``barrier``: when any
    rank failed, every rank removes its temporaries and raises (the failing rank its own error, the others
    CheckpointError), so no rank is left waiting and nothing is committed. Without ``agree`` a failing rank removes
    its temporaries and raises before the barrier."""
    err = None
    try:
        for obj, path in writes:
            torch.save(obj, path + ".tmp")
    except Exception as e:  # a full disk, an unpicklable object, ...
        err = e
    ok = agree(err is None) if agree is not None else err is None
    if not ok:
        for _, path in writes:
            _remove(path + ".tmp")
        if err is not None:
            raise err
        raise CheckpointError("checkpoint not committed: another rank failed to write its part (the previous "
                              "checkpoint is kept)")
    if agree is None and barrier is not None:
        barrier()
    for _, path in writes:
        os.replace(path + ".tmp", path)


def agree_all(group=None):
    """``agree`` for two_phase_commit: an all-reduce of the ranks' failure flags over ``group`` (CPU tensor on
    Gloo, the current CUDA device on NCCL)."""
    import torch.distributed as dist

    def agree(ok):
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
        bad = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(bad, group=group)
        return int(bad.item()) == 0
    return agree


# files of the two-phase commit set: latest.pt and the per-rank optimizer files of pipeline runs
COMMIT_SET = ("latest.pt", "opt_stage*_rep*.pt")


def step_of(path):
    """The ``step`` recorded in a checkpoint file, or None when the file is missing or unreadable."""
    try:
        return int(torch.load(path, map_location="cpu", weights_only=False, mmap=True).get("step", -1))
    except Exception:
        return None


def recover_commit(out, log=print):
    """Finish or undo a two-phase commit in ``out`` that a crash interrupted; run once (one rank) before resuming.

    S = the newest step among readable commit-set temporaries. When some final file already holds step S, phase 2
    had begun, which happens only after every rank's temporary was complete: the temporaries of step S are renamed
    into place (roll forward). Otherwise the commit never reached phase 2: every temporary is removed and the
    previous checkpoint stays (roll back). Leftover temporaries of single-file saves (snap_, merge/, step_) are
    removed. Returns ("clean" | "forward" | "back", S)."""
    tmps = sorted({t for pat in COMMIT_SET for t in glob.glob(os.path.join(out, pat + ".tmp"))})
    for t in glob.glob(os.path.join(out, "*.pt.tmp")) + glob.glob(os.path.join(out, "merge", "*.pt.tmp")):
        if t not in tmps:
            _remove(t)
    if not tmps:
        return "clean", None
    tmp_steps = {t: step_of(t) for t in tmps}
    valid = [s for s in tmp_steps.values() if s is not None]
    S = max(valid) if valid else None
    finals = sorted({f for pat in COMMIT_SET for f in glob.glob(os.path.join(out, pat))})
    final_steps = [step_of(f) for f in finals]
    began = S is not None and S in final_steps and S >= max((s for s in final_steps if s is not None), default=S)
    if began:
        for t, s in tmp_steps.items():
            if s == S:
                os.replace(t, t[:-len(".tmp")])
            else:
                _remove(t)
        log(f"{out}: finished an interrupted checkpoint commit of step {S}")
        return "forward", S
    for t in tmps:
        _remove(t)
    log(f"{out}: removed the temporaries of an unfinished checkpoint commit (step {S}); the previous checkpoint "
        "is kept")
    return "back", S


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
    """torch.load of a checkpoint (memory-mapped). A truncated or corrupt file raises CheckpointError naming the
    checkpoints of its directory that remain."""
    try:
        return torch.load(path, map_location=map_location, weights_only=False, mmap=True)
    except FileNotFoundError:
        raise
    except (RuntimeError, EOFError, OSError, ValueError, pickle.UnpicklingError) as e:
        d = os.path.dirname(os.path.abspath(path))
        others = sorted(os.path.basename(f) for f in glob.glob(os.path.join(d, "*.pt"))
                        if os.path.abspath(f) != os.path.abspath(path))
        raise CheckpointError(f"{path}: unreadable checkpoint ({type(e).__name__}: {str(e)[:200]}); it may have been "
                              f"cut short by a crash or a full disk. Other checkpoints here: {others or 'none'}") from e


def load_opt_state(opt, state):
    """Restore optimizer state but keep the current hyper-parameters (reference train.py:540-546)."""
    fresh = [{k: v for k, v in g.items() if k != "params"} for g in opt.param_groups]
    opt.load_state_dict(state)
    for g, f in zip(opt.param_groups, fresh):
        g.update(f)


# output projections that start at zero in a block added by growth (each new block starts as the identity)
GROW_ZERO = ("attn.out.weight", "cross.out.weight", "mlp.out_proj.weight")


def _param_order(ck):
    """[(prefix, name)] of the checkpoint's own models in parameters() order (the flat EMA list's order)."""
    from ..models import build_models
    from ..models.config import configs_from_ckpt
    if "den_config" not in ck:
        return None
    den_cfg, te_cfg = configs_from_ckpt(ck)
    with torch.device("meta"):
        te, den = build_models(den_cfg, te_cfg)
    return [("te", n) for n, _ in te.named_parameters()] + [("den", n) for n, _ in den.named_parameters()]


@torch.no_grad()
def init_named(ck, named, log=print):
    """``--init`` (reference train.py:617-660, train_pp.py:1272-1426): the weights of checkpoint ``ck`` -- its EMA
    when it has one, else the raw weights -- copied by name into ``named`` = [(prefix "te" | "den", name, tensor)]
    (a whole model or one pipeline stage's part of it).

    Growth (SANA-1.5 style): denoiser blocks past the checkpoint's depth keep their fresh initialisation with
    attn.out, cross.out and mlp.out_proj zeroed, so each new block starts as the identity. A text encoder of another
    shape stays fresh (a new text encoder on a trained denoiser). Any other denoiser tensor that the checkpoint lacks
    or holds in another shape is an error. Returns dict(loaded, grown (block indices), fresh (names))."""
    src = {"te": dict(ck.get("te") or {}), "den": dict(ck["den"])}
    if ck.get("ema"):
        order = _param_order(ck)
        if order is not None and len(order) == len(ck["ema"]):
            for (pre, n), e in zip(order, ck["ema"]):
                src[pre][n] = e
        else:
            log("init: the checkpoint's EMA list does not match its configuration; using its raw weights")
    old_depth = 1 + max((int(k.split(".")[1]) for k in src["den"] if k.startswith("blocks.")), default=-1)
    loaded, fresh, grown = 0, [], set()
    for pre, n, t in named:
        w = src.get(pre, {}).get(n)
        if w is not None and tuple(w.shape) == tuple(t.shape):
            t.copy_(w.to(device=t.device, dtype=t.dtype))
            loaded += 1
        elif pre == "den" and n.startswith("blocks.") and int(n.split(".")[1]) >= old_depth:
            grown.add(int(n.split(".")[1]))
            if n.endswith(GROW_ZERO):
                t.zero_()
        elif pre == "den":
            raise ValueError(f"--init: denoiser tensor {n} is missing from the checkpoint or has another shape")
        else:
            fresh.append(f"{pre}.{n}")
    what = f"init: {loaded} tensors from step {ck.get('step')} ({'EMA' if ck.get('ema') else 'raw'} weights)"
    if grown:
        what += f"; blocks {min(grown)}-{max(grown)} grown as identity blocks"
    if fresh:
        what += f"; {len(fresh)} text-encoder tensors kept fresh"
    log(what)
    return dict(loaded=loaded, grown=sorted(grown), fresh=fresh)


@torch.no_grad()
def reset_ema(ema):
    """EMA shadows set to the current weights (after an --init load replaced the weights the EMA was made from)."""
    if ema is not None:
        for p, s in zip(ema.params, ema.shadow):
            s.copy_(p.detach().to(s.device, torch.float32))


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
