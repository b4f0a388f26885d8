"""Flow-matching trainer: one optimizer step over a global batch (micro-batches, gradient accumulation, gradient
reduction, clipping, LR schedule, Muon + AdamW, EMA, DiLoCo outer syncs).

Reference hot loop: train.py:906-966 (DDP) — per micro-batch logit-normal t, Gaussian noise, caption dropout to the
null prompt, MLM every mlm_every steps (from-scratch text encoder), forward/backward of loss / accum; then
clip_grad_norm_, LR multiplier, optimizer steps, EMA lerp; DiLoCo: an outer sync every H steps instead of a
per-step gradient all-reduce.
The public entry point is ``Trainer.step(batch)``. A batch holds ``x0`` latents and either ``ids`` (caption token
ids: a from-scratch text encoder, or a frozen-LM backend that turns them into states) or ``lm_states`` (optional
``valid`` / ``is_null``). Tensors may live in (pinned) host memory; they are copied inside the step.
"""
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..models import build_models
from ..models.frozen_lm import LM_NULL, LM_PAD, build_frozen_lm
from ..models.text import LMTextEncoder
from ..optim import EMA, build_optimizers, lr_mult, set_lr
from ..optim.adamw import FusedAdamW, GradNorm
from ..optim.muon import Muon
from ..parallel.ddp import GradBuckets
from . import diloco as D
from .flow import FlowModel, drop_captions, make_mlm


def trim_ids(ids, multiple):
    """Drop the all-padding tail columns of right-padded caption rows, keeping a multiple of ``multiple`` columns
    (reference aurora/slayer.py:276-281): the LM and the text attention then run on the real caption lengths."""
    n = int(ids.ne(LM_PAD).sum(1).max()) if ids.numel() else 1
    return ids[:, :min(ids.shape[1], max(multiple, -(-n // multiple) * multiple))]


def length_sorted(ids, parts, generator=None):
    """Row indices of ``parts`` micro-batches of similar caption length: sorted by length, shuffled inside each
    part (reference aurora/slayer.py:284-292). Gradient accumulation sums over all parts, so the step is the same."""
    order = ids.ne(LM_PAD).sum(1).argsort(stable=True)
    return [part[torch.randperm(len(part), generator=generator)] for part in order.chunk(parts)]


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
    ema_cpu: bool = False         # the EMA in pinned host memory (with DiLoCo: updated only at the outer syncs)
    ema_on_all_ranks: bool = False
    cfg_drop: float = 0.1
    t_shift: float = 1.0
    mlm_weight: float = 0.05
    mlm_every: int = 4
    mlm_prob: float = 0.15
    grad_comm: str = "nccl_bf16"
    shard_muon: bool = True
    muon_comm: str = "gather"     # "sharded": owner reduce-scatter + owner-only momentum/NS + fused update all-gather
    rope_random: bool = False     # RPE-2D: random sorted token positions of 0..rope_ref-1 per sample and axis
    t_shift_ref: float = 0.0      # > 0: resolution-dependent time shift s = res / t_shift_ref (overrides t_shift)
    repa_weight: float = 0.0      # > 0: REPA alignment of the block-repa_layer hidden state
    repa_layer: int = 0
    repa_frac: float = 0.25
    repa_until: float = 0.4
    repa_every: int = 1
    repa_target: str = "latent"   # "latent" (offline stand-in) or a FLUX.2 VAE directory (DINOv2 targets)
    irepa: bool = False
    powersgd_rank: int = 8        # grad_comm "powersgd": rank of the gradient approximation
    powersgd_start: int = 10      # plain averaging for this many steps first
    diloco: int = 0
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    outer_comm: str = "bf16"
    offload: bool = False
    seed: int = 0
    act_checkpoint: object = False  # False, "full" (or True) or "selective"
    random_lm: bool = False
    moe_experts: int = 0          # > 0: every moe_every-th block's MLP becomes an MoE layer
    moe_top_k: int = 2
    moe_hidden: int = 4096
    moe_every: int = 2
    moe_capacity: float = 1.25
    moe_aux_weight: float = 0.01
    moe_transport: str = "p2p"    # expert exchange: "p2p" (peer memory fused with the expert GEMMs) or "nccl"
    text_bucket: int = 0          # > 0: trim each micro-batch's caption tokens to its longest caption, rounded up
    length_sort: bool = False     # group the step's samples into micro-batches of similar caption length
    expert_parallel: bool = True  # experts sharded over the data-parallel group

    def derived(self, world=1):
        ratio = self.global_batch / 256
        lr_ratio = self.global_batch / world / 256 if self.diloco else ratio
        lr_scale = 1.0 if self.no_lr_batch_scaling else math.sqrt(lr_ratio)
        ema = self.ema if self.ema is not None else 0.9995 ** ratio
        return lr_scale, ema


class Trainer:
    def __init__(self, den_cfg, te_cfg, cfg: TrainConfig, device, group=None, models=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.group = group
        self.den_cfg, self.te_cfg = den_cfg, te_cfg
        self.per_rank = max(1, cfg.global_batch // self.world)
        self.micro = min(cfg.micro_batch, self.per_rank)
        self.accum = max(1, self.per_rank // self.micro)
        torch.manual_seed(cfg.seed)  # identical init on every rank
        te, den = models if models is not None else build_models(den_cfg, te_cfg, device=self.device)
        self.te, self.den = te.to(self.device), den.to(self.device)
        self.expert_params = []
        if cfg.moe_experts:
            from ..models.moe import MoEMLP, moe_denoiser
            ep_group = dist.group.WORLD if (cfg.expert_parallel and self.distributed and self.world > 1) else None
            # fully recomputed blocks would replay the peer exchange (its epochs): those use NCCL
            transport = cfg.moe_transport if cfg.act_checkpoint in (False, None, "", "selective") else "nccl"
            moe_denoiser(den, cfg.moe_experts, cfg.moe_top_k, cfg.moe_hidden, cfg.moe_every, cfg.moe_capacity, ep_group,
                         transport)
            torch.manual_seed(cfg.seed * 7919 + (self.rank if ep_group is not None else 0))
            for m in den.modules():  # each rank's experts are different experts
                if isinstance(m, MoEMLP):
                    m.reset_parameters()
                    with torch.no_grad():  # the router is replicated: same init everywhere
                        g = torch.Generator().manual_seed(cfg.seed + 17)
                        m.router.weight.copy_(torch.randn(m.router.weight.shape, generator=g) * 0.02)
                    if ep_group is not None:
                        self.expert_params += [m.w_in, m.w_out]
        self.den.checkpoint_blocks = cfg.act_checkpoint
        self.lm_te = isinstance(te, LMTextEncoder)
        if self.lm_te:
            te.checkpoint_blocks = cfg.act_checkpoint
        self.frozen_lm = build_frozen_lm(te_cfg, self.device, cfg.random_lm) if self.lm_te else None
        mlm = 0.0 if self.lm_te else cfg.mlm_weight
        self.repa_proj = self.repa_target = None
        if cfg.repa_weight > 0:
            from .repa import LatentTarget, REPATarget, make_projector
            self.repa_target = LatentTarget(den_cfg.latent_channels, spatial_norm=cfg.irepa, seed=cfg.seed,
                                            device=self.device) if cfg.repa_target == "latent" else \
                REPATarget(cfg.repa_target, device=self.device, spatial_norm=cfg.irepa)
            self.repa_proj = make_projector(den_cfg.dim, self.repa_target.dim, conv=cfg.irepa).to(self.device)
        self.model = FlowModel(te, den, mlm_weight=mlm, moe_aux_weight=cfg.moe_aux_weight if cfg.moe_experts else 0.0,
                               repa_proj=self.repa_proj, repa_layer=cfg.repa_layer, repa_weight=cfg.repa_weight)
        lr_scale, ema = cfg.derived(self.world)
        self.named = [(pre, n, p) for pre, mod in (("te", te), ("den", den)) for n, p in mod.named_parameters()]
        if self.repa_proj is not None:  # projector: AdamW, outside the EMA and the exported model
            self.named += [("repa_proj", n, p) for n, p in self.repa_proj.named_parameters()]
        self.params = [p for _, _, p in self.named if p.requires_grad]
        self.gns_request, self.last_gns = False, None  # set gns_request before a step to measure the noise scale
        reduce_grads = not cfg.diloco
        eids = {id(p) for p in self.expert_params}
        mdt = torch.bfloat16 if cfg.muon_momentum_dtype == "bf16" else None
        self.opts, self.counts = build_optimizers(
            self.named, optimizer=cfg.optimizer, lr_muon=cfg.lr_muon, lr_emb=cfg.lr_emb, lr_adam=cfg.lr_adam,
            lr_hidden=cfg.lr_hidden, lr_scale=lr_scale, wd=cfg.wd, beta2=cfg.beta2, momentum=cfg.momentum,
            ns_steps=cfg.ns_steps, cmuon=cfg.cmuon, muon_period=cfg.muon_period, muon_gamma=cfg.muon_gamma,
            momentum_dtype=mdt, shard=cfg.shard_muon and not cfg.diloco, group=group)
        self.muon = next((o for o in self.opts if isinstance(o, Muon)), None)
        self.muon_comm = None
        self.buckets = self.muon_buckets = None
        sharded = (cfg.muon_comm == "sharded" and self.muon is not None and reduce_grads and self.world > 1
                   and self.muon.world == self.world)
        if self.device.type == "cuda" or self.world > 1:  # expert-parallel weights are not replicated: never averaged
            dense = [p for p in self.params if id(p) not in eids]
            if sharded:
                from ..parallel.muon_comm import MuonShardedComm
                mids = {id(p) for g in self.muon.param_groups for p in g["params"]}
                transport = "p2p" if cfg.grad_comm == "p2p" else "torch"
                self.muon_comm = MuonShardedComm(self.muon, group=group, device=self.device, transport=transport)
                self.muon_buckets = GradBuckets([p for p in dense if id(p) in mids], group=group,
                                                comm="nccl_bf16", reducer=self.muon_comm.reduce_bucket)
                self.muon_comm.attach_buckets(self.muon_buckets)
                dense = [p for p in dense if id(p) not in mids]
            self.powersgd = None
            if cfg.grad_comm == "powersgd" and reduce_grads:
                from ..parallel.powersgd import PowerSGD
                self.buckets = GradBuckets(dense, group=group, comm="nccl_fp32")
                self.powersgd = PowerSGD(self.buckets, cfg.powersgd_rank, cfg.powersgd_start, group, cfg.seed)
                self.buckets.reducer = self.powersgd
            else:
                self.buckets = GradBuckets(dense, group=group, comm=cfg.grad_comm if reduce_grads else "none")
        self.ema_decay = ema
        self.grad_norm = GradNorm(self.device) if self.device.type == "cuda" else None
        self.timer = None  # utils.profiling.PhaseTimer: per-phase device times of each step when set
        self.global_params = self.outer_opt = None
        if cfg.diloco:
            if self.distributed and self.world > 1:
                for p in self.params:
                    dist.broadcast(p.data, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
            self.global_params = D.make_global(self.params, cfg.offload)
            self.outer_opt = D.make_outer_opt(self.global_params, cfg.outer_lr, cfg.outer_momentum)
        model_params = [p for pre, _, p in self.named if pre in ("te", "den") and p.requires_grad]
        self.ema = EMA(model_params, ema, device="cpu" if cfg.ema_cpu else None) \
            if (self.rank == 0 or cfg.ema_on_all_ranks) else None
        self.step_idx = 0
        self.gen = torch.Generator(device=self.device)
        self.cpu_gen = torch.Generator().manual_seed(cfg.seed * 7 + self.rank)  # host-side shuffles
        self.gen.manual_seed(cfg.seed * 1000 + self.rank)
        self.last_gnorm = None
        self.last = {}
        if not self.lm_te:
            self.null_row = torch.as_tensor(te.null_ids(), device=self.device)

    def _random_rope(self, b, side, mb):
        """RPE-2D positions of micro-batch mb (reference train_pp.py:303-308): drawn from (seed, rank, mb) alone."""
        from ..ops import reference as R
        field = self.den_cfg.rope_ref or side
        g = torch.Generator(device=self.device).manual_seed(self.cfg.seed * 4099 + mb * 131 + self.rank)
        rows, cols = R.random_rope_coords(b, side, field, self.device, g)
        return R.rope_2d_from_coords(rows, cols, self.den_cfg.dim // self.den_cfg.heads)

    def memory_report(self):
        from ..utils.memory import report
        grads = [p.grad for p in self.params if p.grad is not None]
        extra = {}
        if self.muon_comm is not None:
            extra["muon_shards"] = [self.muon_comm.g_owned, self.muon_comm.x_in, self.muon_comm.momentum]
        if self.global_params is not None:
            extra["diloco_global"] = list(self.global_params)
        return report(self.rank, params=self.params, grads=grads, opts=self.opts, ema=self.ema, extra=extra)

    def _fused_tail(self):
        """On-device norm + coefficient: CUDA, gradients in the flat buckets, every optimizer takes a coefficient."""
        return (self.device.type == "cuda" and self.buckets is not None and self.powersgd is None
                and all(isinstance(o, (Muon, FusedAdamW)) for o in self.opts))

    def before_save(self):
        """All ranks: bring sharded optimizer state into the optimizers' state dicts (collective)."""
        if self.muon_comm is not None:
            self.muon_comm.export_momentum()

    def after_load(self):
        """All ranks, after the optimizers' ``load_state_dict``: take this rank's shards."""
        if self.muon_comm is not None:
            self.muon_comm.import_momentum()

    def close(self):
        for b in (self.buckets, self.muon_buckets):
            if b is not None:
                b.close()
        if self.muon_comm is not None:
            self.muon_comm.close()

    def n_params(self):
        return sum(p.numel() for p in self.den.parameters()), sum(p.numel() for p in self.te.parameters())

    def _to_dev(self, t):
        if t is None:
            return None
        return t.to(self.device, non_blocking=True) if t.device != self.device else t

    def _text_inputs(self, batch, sl, b):
        """Text-encoder keyword arguments for micro-batch slice sl, with caption dropout and MLM applied."""
        cfg = self.cfg
        if "ids" in batch and not self.lm_te:
            ids = self._to_dev(batch["ids"][sl])
            drop = torch.rand(b, device=self.device, generator=self.gen) < cfg.cfg_drop
            cond_ids = torch.where(drop[:, None], self.null_row[: ids.shape[1]], ids)
            kw = dict(ids=cond_ids)
            if self.model.mlm_weight > 0 and self.step_idx % cfg.mlm_every == 0:
                kw["mlm_ids"], kw["mlm_labels"] = make_mlm(ids, cfg.mlm_prob, self.gen)
            return kw
        if "ids" in batch:
            ids = batch["ids"][sl]
            if cfg.text_bucket:
                ids = trim_ids(ids, cfg.text_bucket)
            ids = self._to_dev(ids)
            valid = ids.ne(LM_PAD)
            is_null = ids[:, 0].eq(LM_NULL)
            states = self.frozen_lm.states(ids)
        else:
            states = batch["lm_states"][sl]
            valid = batch["valid"][sl] if batch.get("valid") is not None else None
            if cfg.text_bucket and valid is not None:
                n = int(valid.sum(1).max()) if valid.numel() else 1
                w = min(states.shape[1], max(cfg.text_bucket, -(-n // cfg.text_bucket) * cfg.text_bucket))
                states, valid = states[:, :w], valid[:, :w]
            states = self._to_dev(states)
            valid = self._to_dev(valid) if valid is not None else \
                torch.ones(b, states.shape[1], dtype=torch.bool, device=self.device)
            is_null = self._to_dev(batch["is_null"][sl]) if batch.get("is_null") is not None else None
        if cfg.cfg_drop > 0:
            is_null, valid = drop_captions(is_null, valid, cfg.cfg_drop, self.gen)
        return dict(lm_states=states, valid=valid, is_null=is_null)

    def _micro_items(self, batch):
        """(x0 micro-batch, source dict, row slice of the source) for every micro-batch of the step: fixed
        micro-batches of ``batch["x0"]``, or with ``batch["groups"]`` (mixed-resolution training, reference
        train_pp.py:1227-1240, 2239-2255) each group's own resolution and micro-batch size ``mb``."""
        groups = batch.get("groups")
        if not groups:
            x0_all = self._to_dev(batch["x0"])
            if self.cfg.length_sort and batch.get("ids") is not None:
                for idx in length_sorted(batch["ids"], self.accum, self.cpu_gen):
                    yield x0_all[idx.to(x0_all.device)], batch, idx
                return
            for m in range(self.accum):
                sl = slice(m * self.micro, (m + 1) * self.micro)
                yield x0_all[sl], batch, sl
            return
        for g in groups:
            x0 = self._to_dev(g["x0"])
            for i in range(0, x0.shape[0], g["mb"]):
                sl = slice(i, i + g["mb"])
                yield x0[sl], g, sl

    def step(self, batch):
        """One optimizer step over this rank's share of the global batch. Returns the mean flow-matching loss
        (device scalar); ``self.last`` holds the MLM loss and the gradient norm."""
        cfg = self.cfg
        timer = self.timer
        if timer is not None:
            timer.begin()
        items = list(self._micro_items(batch))
        total = sum(x0.shape[0] for x0, _, _ in items)
        if self.muon_buckets is not None:
            self.muon_buckets.zero()
            self.muon_comm.begin_step()
        if self.buckets is not None:
            self.buckets.zero()
        else:
            for p in self.params:
                p.grad = None
        for p in self.expert_params:
            if p.grad is not None:
                p.grad.zero_()
        acc = torch.zeros((), device=self.device)
        acc_mlm = torch.zeros((), device=self.device)
        acc_repa = torch.zeros((), device=self.device)
        for m, (x0, src, sl) in enumerate(items):
            x0 = x0.float()
            b = x0.shape[0]
            w = b / total  # the step's loss is the mean over its images, whatever the micro-batch sizes
            kw = self._text_inputs(src, sl, b)
            t = torch.sigmoid(torch.randn(b, device=self.device, generator=self.gen))
            shift = x0.shape[-1] * 16 / cfg.t_shift_ref if cfg.t_shift_ref else cfg.t_shift
            if shift != 1.0:
                t = shift * t / (1 + (shift - 1) * t)
            if src.get("cond") is not None:  # micro-conditions of crops (original size, crop box, target size)
                kw["cond"] = self._to_dev(src["cond"][sl])
            if cfg.rope_random:
                kw["rope"] = self._random_rope(b, x0.shape[-1], self.step_idx * len(items) + m)
            eps = torch.randn(x0.shape, device=self.device, generator=self.gen)
            if self.buckets is not None and m == len(items) - 1:
                self.buckets.arm()
                if self.muon_buckets is not None:
                    self.muon_buckets.arm()
            if self.repa_target is not None:
                from .repa import repa_active
                if repa_active(self.step_idx, cfg.steps, cfg.repa_until, cfg.repa_every):
                    kw["repa_target"] = self.repa_target(x0[: max(1, round(cfg.repa_frac * b))])
            loss, l_fm, l_mlm, l_repa = self.model(x0, t, eps, **kw)
            if l_repa is not None:
                acc_repa += l_repa * w
            (loss * w).backward()
            acc += l_fm * w
            if l_mlm is not None:
                acc_mlm += l_mlm * w
        if timer is not None:
            timer.mark("forward_backward")
        if self.buckets is not None:
            self.buckets.finish()
            if getattr(self, "powersgd", None) is not None:
                self.powersgd.next_step()
        if self.muon_buckets is not None:
            self.muon_buckets.finish()
        if self.expert_params and self.world > 1:  # their gradients summed every rank's loss: make it the mean
            torch._foreach_mul_([p.grad for p in self.expert_params if p.grad is not None], 1.0 / self.world)
        if self.gns_request and cfg.diloco and self.world > 1:
            # gradient noise scale (McCandlish et al. 2018): this worker's gradient (its share of the batch) against
            # the mean over workers (the global batch), one extra bucketed all-reduce (reference train.py:937-960)
            from .evaluate import grad_sq_norms, noise_scale
            grads = [p.grad for p in self.params if p.grad is not None]
            small, big = grad_sq_norms(grads, self.world, group=self.group)
            g2, sig = noise_scale(small, big, total, total * self.world)
            self.last_gns = dict(b_noise=(sig / g2.clamp_min(1e-30)).item(), g2=g2.item(), trace=sig.item())
            self.gns_request = False
        if timer is not None:
            timer.mark("grad_sync_exposed")  # reductions still running after the last backward kernel
        coef = None
        if self.muon_comm is None:
            if self._fused_tail():  # norm + clip coefficient on the device; the optimizers take the coefficient
                grads = list(self.buckets.flat) + [p.grad for p in self.expert_params if p.grad is not None]
                self.last_gnorm, coef = self.grad_norm(grads, cfg.clip)
            else:
                self.last_gnorm = torch.nn.utils.clip_grad_norm_(self.params, cfg.clip, foreach=True)
        else:  # Muon gradients exist reduced only on their owners: norm = other grads + all-reduced owned squares
            others = [p.grad for p in self.buckets.params if p.grad is not None] + \
                [p.grad for p in self.expert_params if p.grad is not None]
            sq = self.muon_comm.owned_sumsq().reshape(())
            if others:
                sq = sq + torch.stack(torch._foreach_norm(others)).square().sum()
            self.last_gnorm = sq.sqrt()
            coef = (cfg.clip / (self.last_gnorm + 1e-6)).clamp(max=1.0)  # applied by the optimizers
        if timer is not None:
            timer.mark("grad_norm")
        set_lr(self.opts, lr_mult(self.step_idx, cfg.steps, cfg.warmup, cfg.schedule))
        # the per-step EMA is updated inside the fused optimizers' parameter-update launches where they can
        ema = self.ema if (self.ema is not None and not cfg.diloco) else None
        rate = 1.0 - self.ema.decay_at(self.step_idx + 1) if ema is not None else 0.0
        for o in self.opts:
            if o is self.muon and self.muon_comm is not None:
                self.muon_comm.step(coef, ema=ema, ema_rate=rate, timer=timer)
            elif isinstance(o, Muon):
                o.step(coef=coef, ema=ema, ema_rate=rate, timer=timer)
            elif isinstance(o, FusedAdamW):
                o.step(coef=coef, ema=ema, ema_rate=rate)
                if timer is not None:
                    timer.mark("adamw")
            else:
                if coef is not None:
                    grads = [p.grad for g in o.param_groups for p in g["params"] if p.grad is not None]
                    if grads:
                        torch._foreach_mul_(grads, coef)
                o.step()
                if timer is not None:
                    timer.mark(type(o).__name__.lower())
        self.step_idx += 1
        if cfg.diloco:
            if self.step_idx % cfg.diloco == 0 or self.step_idx == cfg.steps:
                D.outer_sync(self.global_params, self.params, self.outer_opt, self.world, cfg.outer_comm,
                             self.group)
                if self.ema is not None:
                    n = self.step_idx // cfg.diloco
                    self.ema.update(self.step_idx, D.ema_decay_at_sync(self.ema_decay, cfg.diloco, n))
        elif self.ema is not None:
            self.ema.update(self.step_idx)  # what the fused launches did not cover
        if timer is not None:
            timer.mark("ema_and_rest")
        self.last = dict(mlm=acc_mlm, gnorm=self.last_gnorm, repa=acc_repa)
        return acc
