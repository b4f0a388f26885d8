"""Parameter grouping, LR schedule, EMA.

Grouping follows the reference (train.py:305-341): Muon takes the 2D hidden matrices inside ``.blocks.`` of the
text encoder and the denoiser; AdamW takes the token embedding (lr_emb, no decay), the other projections
(patch_in / patch_out / time_mlp / ada / refiner in/out projections, with decay) and everything else (norms,
mod tables, biases, the null vector; no decay). AdamW is (0.9, beta2), eps 1e-8.
LR schedule: linear warmup then constant or cosine (reference train.py:373-378).
EMA: fp32 copy, decay min(ema, step / (9 + step)) (reference train.py:951-966).
"""
import math

import torch

from .adamw import FusedAdamW
from .muon import Muon, muon_splits


def split_params(named):
    """(prefix, name, param) triples -> dict of lists: hidden (Muon), emb, proj, other."""
    hidden, emb, proj, other = [], [], [], []
    for prefix, name, p in named:
        if not p.requires_grad:
            continue
        full = f"{prefix}.{name}"
        if full == "te.token_embedding.weight":
            emb.append(p)
        elif prefix in ("te", "den") and ".blocks." in f".{name}" and p.ndim == 2 and not name.endswith("mod_table"):
            hidden.append(p)
        elif p.ndim == 2 and not name.endswith("mod_table"):
            proj.append(p)
        else:
            other.append(p)
    return dict(hidden=hidden, emb=emb, proj=proj, other=other)


def build_optimizers(named, optimizer="muon", lr_muon=1e-2, lr_emb=5e-4, lr_adam=3e-4, lr_hidden=None, lr_scale=1.0,
                     wd=0.01, beta2=None, momentum=0.95, ns_steps=5, cmuon=False, muon_period=1, muon_gamma=0.15,
                     momentum_dtype=None, shard=True, group=None, gather=None, fused_adam=None):
    """-> (list of optimizers, parameter counts per kind). Every group carries ``base_lr`` for the LR schedule."""
    parts = split_params(named)
    adam_groups = [
        dict(params=parts["emb"], base_lr=lr_emb * lr_scale, weight_decay=0.0),
        dict(params=parts["proj"], base_lr=lr_adam * lr_scale, weight_decay=wd),
        dict(params=parts["other"], base_lr=lr_adam * lr_scale, weight_decay=0.0),
    ]
    opts = []
    if optimizer == "muon":
        m = Muon([dict(params=parts["hidden"], base_lr=lr_muon)], lr=lr_muon, momentum=momentum, ns_steps=ns_steps,
                 weight_decay=wd, shard=shard, splits=muon_splits(named) if cmuon else None, period=muon_period,
                 gamma=muon_gamma, momentum_dtype=momentum_dtype, group=group, gather=gather)
        opts.append(m)
    else:
        adam_groups.append(dict(params=parts["hidden"], base_lr=(lr_hidden or 1e-4) * lr_scale, weight_decay=wd))
    adam_groups = [g for g in adam_groups if g["params"]]
    for g in adam_groups:
        g["lr"] = g["base_lr"]
    b2 = beta2 if beta2 is not None else (0.99 if optimizer == "adamw" else 0.95)
    if fused_adam is None:
        fused_adam = all(p.is_cuda for g in adam_groups for p in g["params"]) and bool(adam_groups)
    if fused_adam:  # one launch with the clip coefficient, bf16 shadows and the EMA (csrc/optim.cu)
        opts.append(FusedAdamW(adam_groups, betas=(0.9, b2), eps=1e-8))
    else:
        opts.append(torch.optim.AdamW(adam_groups, betas=(0.9, b2), eps=1e-8))
    counts = {k: sum(p.numel() for p in v) for k, v in parts.items()}
    return opts, counts


def lr_mult(step, total, warmup, schedule="constant"):
    if step < warmup:
        return (step + 1) / warmup
    if schedule == "constant":
        return 1.0
    return 0.5 * (1 + math.cos(math.pi * min(1.0, (step - warmup) / max(1, total - warmup))))


def set_lr(opts, mult):
    for opt in opts:
        for g in opt.param_groups:
            g["lr"] = g.get("base_lr", g["lr"]) * mult


class EMA:
    """fp32 exponential moving average of a list of parameters (optionally on the CPU, pinned).

    Fused optimizers may update the EMA of their own parameters inside their parameter-update launch: they call
    ``lookup(p)`` for the EMA tensor and ``mark_fused(p)``; ``update`` then skips those parameters for that step."""

    def __init__(self, params, decay, device=None):
        self.params = list(params)
        self.decay = decay
        self.shadow = [p.detach().float().clone().to(device or p.device) for p in self.params]
        if device is not None and str(device) == "cpu" and torch.cuda.is_available():
            self.shadow = [s.pin_memory() for s in self.shadow]
        self._index = {id(p): i for i, p in enumerate(self.params)}
        self._fused = set()

    def decay_at(self, step):
        return min(self.decay, step / (9 + step))

    def lookup(self, p):
        """The EMA tensor of p when it can be updated in place next to p (same device), else None."""
        i = self._index.get(id(p))
        if i is None or self.shadow[i].device != p.device:
            return None
        return self.shadow[i]

    def mark_fused(self, p):
        self._fused.add(id(p))

    @torch.no_grad()
    def update(self, step, decay=None):
        """Per-step update with decay min(ema, step / (9 + step)), or with an explicit ``decay`` (DiLoCo syncs).
        Parameters whose EMA a fused optimizer already updated this step are skipped."""
        d = decay if decay is not None else self.decay_at(step)
        todo = [(p, s) for p, s in zip(self.params, self.shadow) if id(p) not in self._fused]
        self._fused.clear()
        if not todo:
            return
        src = [p.detach().float() if p.device == s.device else p.detach().float().to(s.device, non_blocking=True)
               for p, s in todo]
        torch._foreach_lerp_([s for _, s in todo], src, 1 - d)

    def state_list(self):
        return [s.clone().cpu() for s in self.shadow]

    @torch.no_grad()
    def copy_to(self, params=None):
        for p, s in zip(params or self.params, self.shadow):
            p.copy_(s.to(p.device))
