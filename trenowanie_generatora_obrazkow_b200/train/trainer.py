"""Flow-matching trainer: one optimizer step over a global batch (micro-batches, gradient accumulation, gradient
reduction, clipping, LR schedule, Muon + AdamW, EMA).

Reference hot loop: train.py:906-966 (DDP) — per micro-batch logit-normal t, Gaussian noise, caption dropout to the
null prompt, forward/backward of loss / accum; then clip_grad_norm_, LR multiplier, optimizer steps, EMA lerp.
The public entry point is ``Trainer.step(batch)``; batch tensors may live in (pinned) host memory, in which case
they are copied to the device inside the step.
"""
import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..models import build_models
from ..optim import EMA, build_optimizers, lr_mult, set_lr
from ..parallel.ddp import GradBuckets
from .flow import FlowModel, drop_captions


@dataclass
class TrainConfig:
    global_batch: int = 256
    micro_batch: int = 32
    steps: int = 1000
    warmup: int = 0
    schedule: str = "constant"
    optimizer: str = "muon"
    lr_muon: float = 1e-2
    lr_emb: float = 5e-4
    lr_adam: float = 3e-4
    lr_hidden: float = None
    no_lr_batch_scaling: bool = False
    wd: float = 0.01
    beta2: float = None
    momentum: float = 0.95
    ns_steps: int = 5
    cmuon: bool = False
    muon_period: int = 1
    muon_gamma: float = 0.15
    muon_momentum_dtype: str = "fp32"
    clip: float = 1.0
    ema: float = None
    ema_on_all_ranks: bool = False
    cfg_drop: float = 0.1
    t_shift: float = 1.0
    grad_comm: str = "nccl_bf16"
    shard_muon: bool = True
    seed: int = 0
    act_checkpoint: bool = False

    def derived(self):
        ratio = self.global_batch / 256
        lr_scale = 1.0 if self.no_lr_batch_scaling else math.sqrt(ratio)
        ema = self.ema if self.ema is not None else 0.9995 ** ratio
        return lr_scale, ema


class Trainer:
    def __init__(self, den_cfg, te_cfg, cfg: TrainConfig, device, group=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.group = group
        assert cfg.global_batch % (cfg.micro_batch * self.world) == 0 or cfg.global_batch < cfg.micro_batch * self.world
        self.per_rank = cfg.global_batch // self.world
        self.micro = min(cfg.micro_batch, self.per_rank)
        self.accum = self.per_rank // self.micro
        torch.manual_seed(cfg.seed)  # identical init on every rank
        te, den = build_models(den_cfg, te_cfg, device=self.device)
        self.te, self.den = te, den
        self.den.checkpoint_blocks = cfg.act_checkpoint
        self.model = FlowModel(te, den)
        lr_scale, ema = self.cfg.derived()
        named = [(pre, n, p) for pre, mod in (("te", te), ("den", den)) for n, p in mod.named_parameters()]
        self.params = [p for _, _, p in named if p.requires_grad]
        self.buckets = GradBuckets(self.params, group=group, comm=cfg.grad_comm) if self.device.type == "cuda" \
            else None
        mdt = torch.bfloat16 if cfg.muon_momentum_dtype == "bf16" else None
        self.opts, self.counts = build_optimizers(
            named, optimizer=cfg.optimizer, lr_muon=cfg.lr_muon, lr_emb=cfg.lr_emb, lr_adam=cfg.lr_adam,
            lr_hidden=cfg.lr_hidden, lr_scale=lr_scale, wd=cfg.wd, beta2=cfg.beta2, momentum=cfg.momentum,
            ns_steps=cfg.ns_steps, cmuon=cfg.cmuon, muon_period=cfg.muon_period, muon_gamma=cfg.muon_gamma,
            momentum_dtype=mdt, shard=cfg.shard_muon, group=group)
        self.ema = EMA(self.params, ema) if (self.rank == 0 or cfg.ema_on_all_ranks) else None
        self.step_idx = 0
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(cfg.seed * 1000 + self.rank)
        self.last_gnorm = None

    def n_params(self):
        return sum(p.numel() for p in self.den.parameters()), sum(p.numel() for p in self.te.parameters())

    def _to_dev(self, t):
        if t is None:
            return None
        return t.to(self.device, non_blocking=True) if t.device != self.device else t

    def step(self, batch):
        """batch: dict with x0 (B, C, H, W) latents, lm_states (B, L, lm_dim), optional valid (B, L) bool and
        is_null (B,) bool; B = global_batch / world. Returns the mean flow-matching loss (device scalar)."""
        cfg = self.cfg
        x0_all = self._to_dev(batch["x0"])
        st_all = self._to_dev(batch["lm_states"])
        valid_all = self._to_dev(batch.get("valid"))
        null_all = self._to_dev(batch.get("is_null"))
        if self.buckets is not None:
            self.buckets.zero()
        else:
            for p in self.params:
                p.grad = None
        acc = torch.zeros((), device=self.device)
        for m in range(self.accum):
            sl = slice(m * self.micro, (m + 1) * self.micro)
            x0 = x0_all[sl].float()
            b = x0.shape[0]
            states = st_all[sl]
            valid = valid_all[sl] if valid_all is not None else torch.ones(b, states.shape[1], dtype=torch.bool,
                                                                         device=self.device)
            is_null = null_all[sl] if null_all is not None else None
            if cfg.cfg_drop > 0:
                is_null, valid = drop_captions(is_null, valid, cfg.cfg_drop, self.gen)
            t = torch.sigmoid(torch.randn(b, device=self.device, generator=self.gen))
            if cfg.t_shift != 1.0:
                t = cfg.t_shift * t / (1 + (cfg.t_shift - 1) * t)
            eps = torch.randn(x0.shape, device=self.device, generator=self.gen)
            if self.buckets is not None and m == self.accum - 1:
                self.buckets.arm()
            loss, l_fm, _, _ = self.model(x0, t, eps, lm_states=states, valid=valid, is_null=is_null)
            (loss / self.accum).backward()
            acc += l_fm / self.accum
        if self.buckets is not None:
            self.buckets.finish()
        self.last_gnorm = torch.nn.utils.clip_grad_norm_(self.params, cfg.clip, foreach=True)
        set_lr(self.opts, lr_mult(self.step_idx, cfg.steps, cfg.warmup, cfg.schedule))
        for o in self.opts:
            o.step()
        self.step_idx += 1
        if self.ema is not None:
            self.ema.update(self.step_idx)
        return acc
