"""PP x DP flow-matching trainer (reference train_pp.py main loop, 2082-2352, without the OPD / server roles).

Rank layout: rank = replica * pp + stage. Each rank builds only its stage (parallel/pipeline.py), the same seed on
every replica of a stage, and broadcasts its weights over the stage group. One ``step``:
  stage 0 draws t / noise / caption dropout for the M micro-batches, sends the targets to the last stage, the 1F1B
  schedule runs the forwards / backwards, gradients are reduced over the stage group (bucketed, overlapped with the
  backward), the clipping norm is all-reduced over the pipe, Muon (sharded over the stage group) + AdamW step, and
  replica 0 keeps the EMA of its stage.
"""
import math

import torch
import torch.distributed as dist

from ..models.text import LMTextEncoder
from ..optim import EMA, build_optimizers, lr_mult, set_lr
from ..parallel.ddp import GradBuckets
from ..parallel.pipeline import (OneFOneB, StageModel, clip_with_norm, direction_groups, grid_layout, pipe_grad_norm,
                                 recv_targets, send_targets, stage_ranges)
from ..ops import fused as Fz
from ..optim.adamw import FusedAdamW
from ..optim.muon import Muon
from .flow import drop_captions
from .trainer import TrainConfig


def pp_groups(world, pp):
    """Process groups of the PP x DP grid over learner ranks [0, world): (pipe group per replica, stage group per
    stage, one-direction links between adjacent stages). A collective over the default group: every rank calls it,
    service ranks too."""
    _, pipes, stages = grid_layout(world, pp)
    return [dist.new_group(r) for r in pipes], [dist.new_group(r) for r in stages], direction_groups(pipes)


class PPTrainer:
    """``world``: the learner ranks [0, world) (service ranks after them take no part); ``groups``: the result of
    ``pp_groups(world, pp)`` when the caller created them already (service ranks in the job)."""

    def __init__(self, den_cfg, te_cfg, cfg: TrainConfig, device, pp, microbatches, te_cost=1.0, world=None,
                 groups=None):
        self.cfg, self.device = cfg, torch.device(device)
        self.rank = dist.get_rank()
        self.world = world or dist.get_world_size()
        self.pp, self.M, self.te_cost = pp, microbatches, te_cost
        self.dp, pipes, stages = grid_layout(self.world, pp)
        self.stage, self.replica = self.rank % pp, self.rank // pp
        self.pipe = pipes[self.replica]
        pipe_groups, stage_groups, self.links = groups if groups is not None else pp_groups(self.world, pp)
        self.pipe_group, self.stage_group = pipe_groups[self.replica], stage_groups[self.stage]
        self.den_cfg, self.te_cfg = den_cfg, te_cfg
        lo, hi = stage_ranges(den_cfg.depth, pp, te_cost)[self.stage]
        self.first, self.last = self.stage == 0, self.stage == pp - 1
        self.model = StageModel(den_cfg, te_cfg, lo, hi, self.first, self.last, self.device,
                                seed=cfg.seed * 1000 + self.stage)
        for p in self.model.parameters():  # identical replicas of a stage
            dist.broadcast(p.data, src=stages[self.stage][0], group=self.stage_group)
        self.named = self.model.full_named_parameters()
        self.params = [p for _, _, p in self.named if p.requires_grad]
        ratio = cfg.global_batch / 256
        lr_scale = 1.0 if cfg.no_lr_batch_scaling else math.sqrt(ratio)
        self.opts, _ = build_optimizers(self.named, optimizer=cfg.optimizer, lr_muon=cfg.lr_muon, lr_emb=cfg.lr_emb,
                                        lr_adam=cfg.lr_adam, lr_hidden=cfg.lr_hidden, lr_scale=lr_scale, wd=cfg.wd,
                                        beta2=cfg.beta2, momentum=cfg.momentum, ns_steps=cfg.ns_steps,
                                        cmuon=cfg.cmuon, muon_period=cfg.muon_period, muon_gamma=cfg.muon_gamma,
                                        shard=cfg.shard_muon, group=self.stage_group)
        # Muon over the stage group: with replicas on CUDA, its gradients are reduce-scattered to the owners and
        # the updates gathered into the parameter update over peer memory (parallel/muon_comm.py); the other
        # gradients are all-reduced in buckets. Otherwise every gradient goes through the buckets.
        self.muon = next((o for o in self.opts if isinstance(o, Muon)), None)
        self.muon_comm = self.muon_buckets = None
        dense = self.params
        if (cfg.muon_comm == "sharded" and self.muon is not None and self.dp > 1 and self.device.type == "cuda"
                and self.muon.world == self.dp):
            from ..parallel.muon_comm import MuonShardedComm
            mids = {id(p) for g in self.muon.param_groups for p in g["params"]}
            transport = "p2p" if cfg.grad_comm == "p2p" else "torch"
            self.muon_comm = MuonShardedComm(self.muon, group=self.stage_group, device=self.device,
                                             transport=transport)
            self.muon_buckets = GradBuckets([p for p in dense if id(p) in mids], group=self.stage_group,
                                            comm="nccl_bf16", reducer=self.muon_comm.reduce_bucket)
            self.muon_comm.attach_buckets(self.muon_buckets)
            dense = [p for p in dense if id(p) not in mids]
        self.buckets = GradBuckets(dense, group=self.stage_group, comm=cfg.grad_comm)
        ema = cfg.ema if cfg.ema is not None else 0.9995 ** ratio
        self.ema = EMA(self.params, ema) if self.replica == 0 else None
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(cfg.seed * 1000 + self.replica)
        self.step_idx = 0
        self.sched = None

    def before_save(self):
        """Every learner rank: bring the owners' sharded Muon momentum into the optimizer state (collective over
        the stage group)."""
        if self.muon_comm is not None:
            self.muon_comm.export_momentum()

    def after_load(self):
        """Every learner rank, after the optimizers' load_state_dict: take this rank's momentum shards."""
        if self.muon_comm is not None:
            self.muon_comm.import_momentum()

    def _schedule(self, mb, side, L):
        dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        d = self.den_cfg
        shapes = dict(x=(mb, side * side, d.dim), t6=(mb, 6, d.dim), text=(mb, L, d.text_dim), dtype=dt)
        return OneFOneB(self.model, self.pipe, self.stage, shapes, self.device, links=self.links)

    def step(self, batch):
        """batch (stage 0 of every replica): x0 (M * mb, C, h, w) and lm_states (M * mb, L, D) [+ valid, is_null,
        cond (M * mb, 8) micro-conditions].
        Other stages pass the same keys with shapes only used for sizing (or None). Returns the loss on the last
        stage (device scalar), else None."""
        cfg, M = self.cfg, self.M
        x0_all = batch["x0"].to(self.device, non_blocking=True) if self.first else None
        n = batch["n"]
        mb = n // M
        side = batch["side"]
        L = batch["text_len"]
        C = self.den_cfg.latent_channels
        self.buckets.zero()
        if self.muon_buckets is not None:
            self.muon_buckets.zero()
            self.muon_comm.begin_step()
        inputs, targets = [], None
        if self.first:
            st_all = batch["lm_states"].to(self.device, non_blocking=True)
            targets = []
            for i in range(M):
                sl = slice(i * mb, (i + 1) * mb)
                x0 = x0_all[sl].float()
                t = torch.sigmoid(torch.randn(mb, device=self.device, generator=self.gen))
                if cfg.t_shift != 1.0:
                    t = cfg.t_shift * t / (1 + (cfg.t_shift - 1) * t)
                eps = torch.randn(x0.shape, device=self.device, generator=self.gen)
                valid = batch["valid"][sl].to(self.device) if batch.get("valid") is not None else \
                    torch.ones(mb, L, dtype=torch.bool, device=self.device)
                is_null = batch["is_null"][sl].to(self.device) if batch.get("is_null") is not None else None
                is_null, valid = drop_captions(is_null, valid, cfg.cfg_drop, self.gen)
                kw = dict(lm_states=st_all[sl], valid=valid, is_null=is_null, hw=tuple(x0.shape[2:]))
                if batch.get("cond") is not None:  # micro-conditions (crop windows) of the micro-batch
                    kw["cond"] = batch["cond"][sl].to(self.device)
                # token-major z_t (bf16 on CUDA) and eps - x0 (fp32) in one pass (the fused kernel on CUDA)
                z_tok, target = Fz.fm_inputs(x0, eps, t)
                inputs.append((z_tok, t, kw))
                targets.append(target.contiguous())
            if self.pp > 1:
                send_targets(targets, self.pipe)
                targets = None
        elif self.last:
            targets = recv_targets(M, (mb, side * side, C), torch.float32, self.device, self.pipe)
        if self.sched is None or self.sched.shapes["x"][:2] != (mb, side * side) or self.sched.shapes["text"][1] != L:
            self.sched = self._schedule(mb, side, L)
        def arm():
            self.buckets.arm()
            if self.muon_buckets is not None:
                self.muon_buckets.arm()

        loss = self.sched.step(M, (lambda i: inputs[i]) if self.first else None, targets, side, 1.0 / M,
                               before_last_backward=arm)
        self.buckets.finish()
        if self.muon_buckets is not None:
            self.muon_buckets.finish()
        # global norm over the pipe: this stage's squared norm (Muon part: the owners' all-reduced squares), summed
        # over the stages; the optimizers apply the clip coefficient themselves
        others = [p.grad for p in self.buckets.params if p.grad is not None]
        sq = torch.stack(torch._foreach_norm(others)).float().square().sum() if others else \
            torch.zeros((), device=self.device)
        if self.muon_comm is not None:
            sq = sq + self.muon_comm.owned_sumsq().reshape(())
        if self.pp > 1:
            dist.all_reduce(sq, group=self.pipe_group)
        norm = sq.sqrt()
        coef = (cfg.clip / (norm + 1e-6)).clamp(max=1.0)
        set_lr(self.opts, lr_mult(self.step_idx, cfg.steps, cfg.warmup, cfg.schedule))
        ema = self.ema
        rate = 1.0 - ema.decay_at(self.step_idx + 1) if ema is not None else 0.0
        for o in self.opts:
            if o is self.muon and self.muon_comm is not None:
                self.muon_comm.step(coef, ema=ema, ema_rate=rate)
            elif isinstance(o, (Muon, FusedAdamW)):
                o.step(coef=coef, ema=ema, ema_rate=rate)
            else:
                grads = [p.grad for g in o.param_groups for p in g["params"] if p.grad is not None]
                if grads:
                    torch._foreach_mul_(grads, coef)
                o.step()
        self.step_idx += 1
        if ema is not None:
            ema.update(self.step_idx)  # what the fused launches did not cover
        self.last_gnorm = norm
        return loss
