"""Flow-matching DiT training (DDP or DiLoCo), the single-model trainer of this framework.

  # 8 GPUs, data prepared in the shard format (data/shards.py), from-scratch text encoder with MLM
  torchrun --nproc_per_node 8 train.py --data data/aurora --out runs/aurora --size 253m --te-size 27m
  # no data at hand: synthetic latents / captions of the same shapes
  python train.py --synthetic 4096 --out runs/smoke --size 50m --te-size 13m --steps 20
  # DiLoCo / MuLoCo: every GPU trains its own copy, outer sync every 16 steps
  torchrun --nproc_per_node 8 train.py --data ... --out ... --diloco 16

Flag names follow the reference's train.py (train.py:42-184); derived defaults (LR batch scaling, steps, EMA
decay, cadences, refiner width, REPA layer) follow its resolve_defaults (train.py:549-586). Checkpoints are
written in the reference's layout (latest.pt, snap_<step>.pt, merge/step_<step>.pt) and resume from either
framework's files.
"""
import argparse
import json
import math
import os
import time
from dataclasses import asdict, replace

import torch
import torch.distributed as dist

from trenowanie_generatora_obrazkow_b200.data.shards import (ShardStore, TrainStream, load_val, select_shards, subsets,
                                                             val_groups)
from trenowanie_generatora_obrazkow_b200.models import (SIZES, TE_SIZES, DenoiserConfig, LMEncoderConfig,
                                                        make_configs, te_config_from_dict)
from trenowanie_generatora_obrazkow_b200.train.evaluate import evaluate, weight_sq, wrms_stats
from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig, Trainer
from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt
from trenowanie_generatora_obrazkow_b200.utils.logging import RunLogger
from trenowanie_generatora_obrazkow_b200.utils.flops import PEAK_TFLOPS, peak_tflops, train_flops_per_sample


def build_parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    a = p.add_argument
    a("--data", default="data/aurora")
    a("--synthetic", type=int, default=0, help="train on N synthetic samples (no data directory needed)")
    a("--out", required=True)
    a("--size", choices=sorted(SIZES), default="253m")
    a("--depth", type=int, default=None)
    a("--res", type=int, default=256, help="image resolution in px (latent side = res / 16)")
    a("--te-size", choices=sorted(TE_SIZES), default="27m")
    a("--te-dim", type=int, default=None)
    a("--te-depth", type=int, default=None)
    a("--te-experts", type=int, default=None)
    a("--te-quant", choices=["", "int8"], default=None)
    a("--random-lm", action="store_true", help="frozen-LM encoders: a fixed random embedding stands in for the LM")
    a("--ema-cpu", action="store_true", help="keep the EMA on the CPU (pinned); needs --diloco, whose EMA is updated "
      "only at the outer syncs")
    a("--pl-prob", type=float, default=0.0, help="share of training captions from the Polish token rows "
      "(<shard>.tok_<enc>_pl.npy, prepare_data.py tokenize --lang pl); validation stays English")
    a("--rope-ref", type=int, default=0,
      help="RoPE position field: 0 = integer positions per grid; N = every resolution spread over an N x N field")
    a("--rope-random", action="store_true",
      help="RPE-2D: random sorted distinct token positions of 0..rope-ref-1 per sample and axis (needs --rope-ref)")
    a("--micro-cond", type=int, default=0,
      help="micro-conditioning on (original size, crop box, target size); the original image size in px, 0 = off")
    a("--crop-res", type=int, nargs="*", default=[],
      help="resize-and-crop: take --res windows from these larger latent grids (<shard>.lat<res>.npy; 256 = .lat.npy)")
    a("--crop-prob", type=float, default=0.5)
    a("--t-shift-ref", type=float, default=0.0, help="resolution-dependent time shift res / REF (overrides --t-shift)")
    a("--text-bucket", type=int, default=0, choices=[0, 8, 16, 32, 64, 128],
      help="trim each micro-batch's captions to its longest one, rounded up to this multiple (0 = off)")
    a("--length-sort", action="store_true", help="micro-batches of similar caption length (with --text-bucket)")
    a("--multi-res", type=int, nargs="*", default=[],
      help="mixed-resolution steps: these resolutions in every step (--res = the largest); latents of each from "
           "<shard>.lat<res>.npy (.lat.npy at 256)")
    a("--multi-res-mbs", type=int, nargs="*", default=[], help="--multi-res: micro-batches per GPU and step at each")
    a("--multi-res-mb", type=int, nargs="*", default=[], help="--multi-res: images per micro-batch at each")
    a("--repa-weight", type=float, default=0.0,
      help="REPA loss weight (0 = off; the reference's 0.5 needs DINOv2 targets, see --repa-target)")
    a("--repa-layer", type=int, default=None)
    a("--repa-frac", type=float, default=0.25)
    a("--repa-until", type=float, default=0.4)
    a("--repa-every", type=int, default=1)
    a("--irepa", action="store_true", help="iREPA: 3x3 conv projector + spatially normalised targets")
    a("--repa-target", default="latent",
      help="a local FLUX.2 VAE directory (decoder + DINOv2 targets) or 'latent' (offline stand-in target)")
    a("--optimizer", choices=["muon", "adamw"], default="muon")
    a("--lr-hidden", type=float, default=None)
    a("--beta2", type=float, default=None)
    a("--steps", type=int, default=None)
    a("--batch", type=int, default=2048)
    a("--fraction", type=float, default=0.1)
    a("--micro-batch", type=int, default=64)
    a("--warmup-frac", type=float, default=0.02)
    a("--lr-muon", type=float, default=1e-2)
    a("--lr-emb", type=float, default=5e-4)
    a("--lr-adam", type=float, default=3e-4)
    a("--no-lr-batch-scaling", action="store_true")
    a("--wd", type=float, default=None)
    a("--schedule", choices=["constant", "cosine"], default="constant")
    a("--momentum", type=float, default=0.95)
    a("--ns-steps", type=int, default=5)
    a("--cmuon", action="store_true")
    a("--muon-period", type=int, default=1)
    a("--muon-gamma", type=float, default=0.15)
    a("--clip", type=float, default=1.0)
    a("--ema", type=float, default=None)
    a("--cfg-drop", type=float, default=0.1)
    a("--t-shift", type=float, default=1.0)
    a("--mlm-weight", type=float, default=0.05)
    a("--mlm-every", type=int, default=4)
    a("--mlm-prob", type=float, default=0.15)
    a("--grad-comm", choices=["fp32", "bf16", "powersgd"], default="bf16",
      help="powersgd: low-rank gradient compression with error feedback (prefer --optimizer adamw)")
    a("--powersgd-rank", type=int, default=8)
    a("--grad-transport", choices=["auto", "nccl", "p2p"], default="auto",
      help="bf16 gradient averaging through NCCL or the peer-memory kernel (auto: p2p on CUDA)")
    a("--muon-comm", choices=["auto", "gather", "sharded"], default="auto",
      help="sharded: Muon gradients reduce-scattered to their owners, updates all-gathered into the parameter "
           "update (auto: sharded with bf16 gradients on CUDA)")
    a("--diloco", type=int, default=0)
    a("--outer-lr", type=float, default=0.7)
    a("--outer-momentum", type=float, default=0.9)
    a("--offload", action="store_true")
    a("--outer-comm", choices=["bf16", "fp32"], default="bf16")
    a("--muon-momentum-dtype", choices=["fp32", "bf16"], default="fp32")
    a("--act-checkpoint", nargs="?", const="full", default=None, choices=["full", "selective"],
      help="activation checkpointing per block: full recompute, or selective (keep GEMM / attention outputs, "
           "recompute the norms, q/k-norm + RoPE and SwiGLU in the backward)")
    a("--workers", type=int, default=4)
    a("--seed", type=int, default=0)
    a("--log-every", type=int, default=None)
    a("--eval-every", type=int, default=None)
    a("--ckpt-every", type=int, default=None)
    a("--merge-every", type=int, default=None)
    a("--merge-start", type=float, default=0.8)
    a("--keep-every", type=int, default=None)
    a("--val-samples", type=int, default=4096)
    a("--peak-tflops", type=float, default=0)
    a("--wandb", default="trenowanie_generatora_obrazkow")
    a("--no-wandb", action="store_true")
    a("--eval-only", action="store_true")
    a("--init", default="", help="start from this checkpoint's EMA weights (ignored on resume)")
    a("--load-hf", default="", help="start from an export directory (export.py layout; its weights, as --init)")
    a("--freeze-den", action="store_true")
    a("--fid-every", type=int, default=0, help="Fréchet distance of EMA samples of held-out prompts every N steps "
      "(features: DINOv2 of decoded images with --vae, else the offline latent stand-in); 0 = off")
    a("--fid-at-start", action="store_true", help="also measure it before the first step")
    a("--fid-samples", type=int, default=4096, help="held-out prompts per measurement (<= --val-samples)")
    a("--fid-steps", type=int, default=50, help="Euler steps of the samples")
    a("--fid-cfg", type=float, default=3.0, help="guidance scale of the samples")
    a("--vae", default="", help="local FLUX.2 VAE directory: decoder of the DINOv2 features (FD) and REPA targets")
    a("--repa-encoder", default="vit_base_patch14_reg4_dinov2.lvd142m", help="timm encoder of the DINOv2 features")
    a("--gns-every", type=int, default=None, help="with --diloco: gradient noise scale (B_noise) from one worker's "
      "vs the all-worker gradient on the first step after an outer sync, every N steps (default 8 x --diloco; "
      "0 = off)")
    a("--per-shard", type=int, default=0, help="--eval-only: also the loss of N samples of every held-out shard and "
      "of the first and a middle training shard of every subset (generalisation vs memorisation)")
    a("--no-compile", action="store_true", help="accepted for command-line compatibility: nothing is compiled here")
    return p


def resolve_defaults(args, world=1):
    ratio = args.batch / 256
    if args.steps is None:
        args.steps = max(1, round(247_805 * args.fraction / ratio))
    lr_ratio = args.batch / world / 256 if args.diloco else ratio
    args.lr_scale = 1.0 if args.no_lr_batch_scaling else math.sqrt(lr_ratio)
    if args.ema is None:
        args.ema = 0.9995 ** ratio
    args.log_every = args.log_every or min(100, max(1, args.steps // 40))
    args.eval_every = max(1, args.steps // 20) if args.eval_every is None else args.eval_every
    args.ckpt_every = max(1, args.steps // 50) if args.ckpt_every is None else args.ckpt_every
    args.merge_every = max(1, args.steps // 25) if args.merge_every is None else args.merge_every
    args.keep_every = max(1, args.steps // 10) if args.keep_every is None else args.keep_every
    if args.wd is None:
        args.wd = 0.1 if args.optimizer == "adamw" else 0.01
    if args.lr_hidden is None:
        args.lr_hidden = 1e-4 * 768 / SIZES[args.size].dim
    lm = isinstance(TE_SIZES[args.te_size], LMEncoderConfig)
    if lm and args.te_dim is None and TE_SIZES[args.te_size].backend != "states":
        args.te_dim = SIZES[args.size].dim // 2
    if lm:
        args.mlm_weight = 0.0
    if args.repa_layer is None:
        args.repa_layer = max(1, round(0.3 * (args.depth or SIZES[args.size].depth)))
    if args.gns_every is None:
        args.gns_every = 8 * args.diloco
    if args.vae and args.repa_target == "latent":
        args.repa_target = args.vae
    if args.diloco:
        up = lambda n: n and -(-n // args.diloco) * args.diloco
        args.eval_every, args.ckpt_every = up(args.eval_every), up(args.ckpt_every)
        args.merge_every, args.keep_every = up(args.merge_every), up(args.keep_every)
        args.fid_every = up(args.fid_every)
    return args


class SyntheticStream:
    """Random latents + caption rows of the configured shapes (no data directory)."""

    def __init__(self, n, side, te_cfg, micro, rank, seed):
        self.n, self.side, self.te_cfg, self.micro = n, side, te_cfg, micro
        self.g = torch.Generator().manual_seed(seed * 1000 + rank)

    def __iter__(self):
        L = self.te_cfg.max_tokens
        lm = isinstance(self.te_cfg, LMEncoderConfig)
        while True:
            lat = torch.randn(self.micro, 128, self.side, self.side, generator=self.g).half()
            if lm and self.te_cfg.backend == "states":
                yield lat, torch.randn(self.micro, L, self.te_cfg.lm_dim, generator=self.g).bfloat16()
                continue
            ids = torch.randint(6, 8000 if not lm else 60000, (self.micro, L), generator=self.g)
            n = torch.randint(3, L, (self.micro,), generator=self.g)
            pad = 65535 if lm else 0
            ids[torch.arange(L)[None] >= n[:, None]] = pad
            yield lat, ids


def main():
    distributed = "RANK" in os.environ
    if distributed:
        backend = os.environ.get("DIST_BACKEND", "nccl")
        local = int(os.environ.get("LOCAL_RANK", 0))
        if torch.cuda.is_available():
            torch.cuda.set_device(local % torch.cuda.device_count())
        dist.init_process_group(backend)
        rank, world = dist.get_rank(), dist.get_world_size()
    else:
        rank, world, local = 0, 1, 0
    args = resolve_defaults(build_parser().parse_args(), world)
    mr_groups = list(zip(args.multi_res, args.multi_res_mbs, args.multi_res_mb))
    if args.multi_res:
        assert len(args.multi_res) == len(args.multi_res_mbs) == len(args.multi_res_mb), \
            "--multi-res, --multi-res-mbs and --multi-res-mb need one value per resolution"
        assert max(args.multi_res) == args.res and all(r % 16 == 0 for r in args.multi_res), \
            "--multi-res: --res must be the largest resolution, all multiples of 16"
        assert not (args.repa_weight or args.crop_res or args.diloco), "--multi-res: no REPA / crops / DiLoCo"
        per = sum(n * b for _, n, b in mr_groups)
        assert args.batch == world * per, f"--multi-res: {per} images per GPU and step, so --batch must be {world * per}"
        args.micro_batch = max(b for _, _, b in mr_groups)
    device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    master = rank == 0
    os.makedirs(args.out, exist_ok=True)
    log = print if master else (lambda *a, **k: None)

    den_cfg, te_cfg = make_configs(args.size, args.te_size, args.te_dim, args.te_depth, args.depth,
                                   args.te_experts, args.te_quant)
    den_cfg = replace(den_cfg, latent_size=args.res // 16, rope_ref=args.rope_ref, micro_cond=args.micro_cond)
    ckpt_path = os.path.join(args.out, "latest.pt")
    if master:  # a save cut short leaves only a temporary: removed, the previous latest.pt is the checkpoint
        ckpt.recover_commit(args.out, log)
    resume = ckpt.load(ckpt_path) if os.path.exists(ckpt_path) else None
    if resume is not None:  # the checkpoint's architecture wins
        den_cfg = DenoiserConfig(**resume["den_config"])
        te_cfg = te_config_from_dict(resume["te_config"])
    assert not args.rope_random or den_cfg.rope_ref, "--rope-random needs --rope-ref (the position field)"
    assert not args.ema_cpu or args.diloco, "--ema-cpu needs --diloco (the host EMA is updated at the outer syncs)"
    assert not args.crop_res or den_cfg.micro_cond, "--crop-res needs --micro-cond"
    cuda = device.type == "cuda"
    transport = args.grad_transport if args.grad_transport != "auto" else ("p2p" if cuda else "nccl")
    grad_comm = "nccl_fp32" if args.grad_comm == "fp32" else "powersgd" if args.grad_comm == "powersgd" else \
        ("p2p" if transport == "p2p" else "nccl_bf16")
    muon_comm = args.muon_comm if args.muon_comm != "auto" else \
        ("sharded" if cuda and args.grad_comm == "bf16" else "gather")
    tc = TrainConfig(global_batch=args.batch, micro_batch=args.micro_batch, steps=args.steps,
                     warmup=int(args.warmup_frac * args.steps), schedule=args.schedule, optimizer=args.optimizer,
                     lr_muon=args.lr_muon, lr_emb=args.lr_emb, lr_adam=args.lr_adam, lr_hidden=args.lr_hidden,
                     no_lr_batch_scaling=args.no_lr_batch_scaling, wd=args.wd, beta2=args.beta2,
                     momentum=args.momentum, ns_steps=args.ns_steps, cmuon=args.cmuon, muon_period=args.muon_period,
                     muon_gamma=args.muon_gamma, muon_momentum_dtype=args.muon_momentum_dtype, clip=args.clip,
                     ema=args.ema, ema_cpu=args.ema_cpu, cfg_drop=args.cfg_drop, t_shift=args.t_shift, mlm_weight=args.mlm_weight,
                     mlm_every=args.mlm_every, mlm_prob=args.mlm_prob,
                     grad_comm=grad_comm, muon_comm=muon_comm, diloco=args.diloco,
                     powersgd_rank=args.powersgd_rank, powersgd_start=max(2, int(args.warmup_frac * args.steps)),
                     rope_random=args.rope_random, t_shift_ref=args.t_shift_ref,
                     repa_weight=args.repa_weight, repa_layer=args.repa_layer, repa_frac=args.repa_frac,
                     repa_until=args.repa_until, repa_every=args.repa_every, repa_target=args.repa_target,
                     irepa=args.irepa, text_bucket=args.text_bucket, length_sort=args.length_sort,
                     outer_lr=args.outer_lr, outer_momentum=args.outer_momentum, outer_comm=args.outer_comm,
                     offload=args.offload, seed=args.seed, act_checkpoint=args.act_checkpoint,
                     random_lm=args.random_lm)
    tr = Trainer(den_cfg, te_cfg, tc, device)
    te, den = tr.te, tr.den
    if args.freeze_den:
        den.requires_grad_(False)
    step, samples = 0, 0
    if resume is not None:
        ckpt.load_weights(resume, te, den)
        if resume.get("opts"):
            for o, s in zip(tr.opts, resume["opts"]):
                ckpt.load_opt_state(o, s)
            tr.after_load()
        if tr.ema is not None and resume.get("ema"):
            for s, e in zip(tr.ema.shadow, resume["ema"]):
                s.copy_(e.to(s.device))
        if tr.repa_proj is not None and resume.get("repa_proj"):
            tr.repa_proj.load_state_dict(resume["repa_proj"])
        if tr.outer_opt is not None and resume.get("outer"):
            ckpt.load_opt_state(tr.outer_opt, resume["outer"])
        step, samples = int(resume["step"]), int(resume.get("samples", 0))
        tr.step_idx = step
        log(f"resumed from {ckpt_path} at step {step}")
    elif args.init:  # EMA weights by name; a larger --depth grows identity blocks, a new text encoder stays fresh
        init = ckpt.load(args.init)
        named = [("te", n, p) for n, p in te.named_parameters()] + [("den", n, p) for n, p in den.named_parameters()]
        ckpt.init_named(init, named, log)
        ckpt.reset_ema(tr.ema)
        log(f"init: weights from {args.init}")
    elif args.load_hf:
        from trenowanie_generatora_obrazkow_b200.utils.export import load_export
        xte, xden, _, _, _ = load_export(args.load_hf)
        te.load_state_dict(xte.state_dict())
        den.load_state_dict(xden.state_dict())
        log(f"init: weights from the export {args.load_hf}")
    del resume
    n_den, n_te = tr.n_params()
    log(f"params: denoiser {n_den / 1e6:.1f}M, text encoder {n_te / 1e6:.1f}M (trainable)")

    # ---- data --------------------------------------------------------------------------------------------
    side = args.res // 16
    val = None
    groups = ()
    group_loaders = []
    if args.synthetic:
        stream = SyntheticStream(args.synthetic, side, te_cfg, tr.micro, rank, args.seed)
        loader = iter(stream)
        group_loaders = [iter(SyntheticStream(args.synthetic, r // 16, te_cfg, b, rank, args.seed + 17 * i))
                         for i, (r, _, b) in enumerate(mr_groups)]
        if master:
            vs = SyntheticStream(args.synthetic, side, te_cfg, min(args.val_samples, 64), 10 ** 6, args.seed + 1)
            val = next(iter(vs))
    else:
        tok_suffix = getattr(te_cfg, "tok_suffix", "")
        null_row = te.null_ids()
        # --pl-prob: that share of the training captions from the Polish token rows (<shard>.tok_<enc>_pl.npy);
        # validation stays English (reference train.py:669-676)
        alt_suffix = f"{tok_suffix}_pl" if args.pl_prob > 0 else ""
        assert not alt_suffix or tok_suffix, "--pl-prob needs a frozen-LM text encoder with its own token rows"
        train_names, val_names = select_shards(args.data, args.fraction, tok_suffix, alt_suffix)
        crops = [("lat" if r == 256 else f"lat{r}", "") for r in args.crop_res]
        store = ShardStore(args.data, train_names, tok_suffix, null_row, alt_suffix=alt_suffix, alt_prob=args.pl_prob,
                           lat_kind="lat" if side == 16 else f"lat{args.res}", crops=crops, crop_prob=args.crop_prob,
                           cond_base=den_cfg.micro_cond)
        if alt_suffix:
            log(f"captions: {100 * args.pl_prob:.0f}% Polish ({alt_suffix}), the rest English")
        stream = TrainStream(store, tr.micro, rank, world, args.seed, start_micro=samples // (tr.micro * world))
        loader = iter(torch.utils.data.DataLoader(stream, batch_size=None, num_workers=args.workers,
                                                  pin_memory=device.type == "cuda",
                                                  persistent_workers=args.workers > 0))
        for i, (r, _, b) in enumerate(mr_groups):  # one stream per resolution, its own micro-batch size
            st = ShardStore(args.data, train_names, tok_suffix, null_row, lat_kind="lat" if r == 256 else f"lat{r}",
                            cond_base=den_cfg.micro_cond)
            ts = TrainStream(st, b, rank, world, args.seed + 17 * i, start_micro=step * mr_groups[i][1])
            group_loaders.append(iter(torch.utils.data.DataLoader(ts, batch_size=None, num_workers=1,
                                                                  pin_memory=device.type == "cuda")))
        if master and val_names:
            val = load_val(args.data, val_names, args.val_samples, tok_suffix, null_row)
            groups = val_groups(args.data, val_names, args.val_samples)
        log(f"train: {len(train_names)} shards / {len(store):,} images, val: {len(val_names)} shards")
    lm_states_key = isinstance(te_cfg, LMEncoderConfig) and te_cfg.backend == "states"

    # ---- Fréchet distance of samples during training (every rank generates a slice of the held-out prompts) ------
    fid = None
    if args.fid_every or args.fid_at_start:
        from trenowanie_generatora_obrazkow_b200.train.fid import (DinoFeatures, LatentFeatures, TrainingFD,
                                                                   my_prompts)
        if args.synthetic:
            held = next(iter(SyntheticStream(args.synthetic, side, te_cfg, min(args.val_samples, 64), 10 ** 6,
                                             args.seed + 1)))
        else:
            held = load_val(args.data, val_names, args.val_samples, tok_suffix, null_row) if val_names else None
        if held is None:
            log("--fid-every: no held-out shards, Fréchet distance off")
        else:
            lat, prompts = held
            n = min(args.fid_samples, len(lat))
            mine = my_prompts(n, rank, world)
            feats = DinoFeatures(args.vae, args.repa_encoder, device) if args.vae else \
                LatentFeatures(den_cfg.latent_channels, seed=args.seed)
            fd_shift = args.res / args.t_shift_ref if args.t_shift_ref else args.t_shift
            fid = TrainingFD(lat[mine].float(), prompts[mine], n, feats, args.fid_steps, args.fid_cfg, fd_shift,
                             args.seed, lm=isinstance(te_cfg, LMEncoderConfig), frozen_lm=tr.frozen_lm)
            log(f"Fréchet distance of {n} held-out prompts every {args.fid_every} steps "
                f"({'DINOv2 ' + args.repa_encoder if args.vae else 'latent stand-in'} features)")

    logger = RunLogger(args.out, vars(args), enabled=master and not args.no_wandb, project=args.wandb)
    peak = args.peak_tflops or (peak_tflops(torch.cuda.get_device_name(device)) if device.type == "cuda" else 0)
    flops_sample = train_flops_per_sample(den_cfg, te_cfg, side * side)

    def save():
        tr.before_save()  # collective: every rank takes part
        if not master:
            return
        ckpt.save_latest(ckpt_path, step, samples, den_cfg, te_cfg, te, den, tr.opts, tr.ema, vars(args),
                         outer=tr.outer_opt.state_dict() if tr.outer_opt is not None else None,
                         repa_proj=tr.repa_proj)
        if args.keep_every and step % args.keep_every == 0:
            ckpt.save_snapshot(args.out, step, den_cfg, te_cfg, te, den, tr.ema)

    def with_ema(fn):
        """fn() with the EMA weights in place of the live ones (restored afterwards)."""
        swap = [p.detach().clone() for p in tr.params] if tr.ema is not None else None
        if swap is not None:
            tr.ema.copy_to()
        try:
            return fn()
        finally:
            if swap is not None:
                with torch.no_grad():
                    for p, s in zip(tr.params, swap):
                        p.copy_(s)

    def run_eval():
        if val is None:
            return {}
        return with_ema(lambda: evaluate(te, den, val, device, groups=groups))

    def run_fid():
        fd = with_ema(lambda: fid(te, den, device))
        log(f"step {step} FD {fd:.3f}")
        logger.log({"val/fd": fd}, step)

    if args.eval_only:
        res = run_eval()
        if val is not None and not torch.is_floating_point(val[1]):
            # the same images with the empty prompt: the gap shows how much the model uses the text
            # (reference train.py:681-687)
            null = torch.as_tensor(te.null_ids(), dtype=val[1].dtype).expand_as(val[1]).clone()
            no_text = with_ema(lambda: evaluate(te, den, (val[0], null), device))
            res.update({k.replace("val/", "val_no_text/"): v for k, v in no_text.items()})
            res["text_gain"] = no_text["val/loss"] - res["val/loss"]
        log(json.dumps(res, indent=1))
        if args.per_shard and master and not args.synthetic:
            # held-out shards, then the first and a middle training shard of every subset: a loss much lower on
            # the training shards than on the held-out ones means memorisation rather than generalisation
            picks = [("val", n) for n in val_names]
            for sub, names in sorted(subsets(train_names).items()):
                for n in dict.fromkeys([names[0], names[len(names) // 2]]):
                    picks.append((f"train {sub}", n))
            for kind, name in picks:
                shard_val = load_val(args.data, [name], args.per_shard, tok_suffix, null_row)
                loss = with_ema(lambda: evaluate(te, den, shard_val, device))["val/loss"]
                log(f"per-shard {kind:>16s} {name}: loss {loss:.4f} ({len(shard_val[0])} samples)")
        if fid is not None:
            run_fid()
        if distributed:
            dist.destroy_process_group()
        return

    if fid is not None and args.fid_at_start:
        run_fid()

    t0, acc, nacc = time.time(), 0.0, 0
    def gather(micros):
        batch = {"x0": torch.cat([m[0] for m in micros]),
                 ("lm_states" if lm_states_key else "ids"): torch.cat([m[1] for m in micros])}
        if den_cfg.micro_cond and len(micros[0]) > 2:
            batch["cond"] = torch.cat([m[-1] for m in micros])
        return batch

    while step < args.steps:
        if mr_groups:
            groups = []
            for (r, n, b), it in zip(mr_groups, group_loaders):
                g = gather([next(it) for _ in range(n)])
                g["mb"] = b
                groups.append(g)
            batch = {"groups": groups}
        else:
            batch = gather([next(loader) for _ in range(tr.accum)])
        if args.diloco and distributed and args.gns_every and step % args.diloco == 0 and step % args.gns_every == 0:
            tr.gns_request = True  # the first step after an outer sync: all workers start from the same weights
        loss = tr.step(batch)
        step += 1
        if tr.last_gns is not None:
            log(f"step {step} gradient noise scale B_noise {tr.last_gns['b_noise']:.1f} (|G|^2 "
                f"{tr.last_gns['g2']:.3e}, tr S {tr.last_gns['trace']:.3e})")
            logger.log({"train/gns_b_noise": tr.last_gns["b_noise"]}, step)
            tr.last_gns = None
        samples += args.batch
        acc += loss.detach()
        nacc += 1
        if step % args.log_every == 0 or step == args.steps:
            l = acc.clone()
            if distributed:
                dist.all_reduce(l)
                l /= world
            torch.cuda.synchronize() if device.type == "cuda" else None
            dt = time.time() - t0
            img_s = nacc * args.batch / dt
            tflops = img_s * flops_sample / world / 1e12
            stats = {"train/loss": (l / nacc).item(), "train/grad_norm": float(tr.last_gnorm), "train/img_s": img_s,
                     "train/tflops_per_gpu": tflops, "train/samples": samples}
            if peak:
                stats["train/mfu"] = tflops / peak
            if float(tr.last.get("mlm", 0)) > 0:
                stats["train/mlm"] = float(tr.last["mlm"])
            stats.update(wrms_stats(weight_sq(tr.named, device)))
            log(f"step {step}/{args.steps} loss {stats['train/loss']:.4f} gnorm {stats['train/grad_norm']:.3f} "
                f"{img_s:.1f} img/s {tflops:.1f} TFLOPS/GPU" + (f" MFU {100 * stats['train/mfu']:.1f}%" if peak else ""))
            logger.log(stats, step)
            t0, acc, nacc = time.time(), 0.0, 0
        if args.eval_every and (step % args.eval_every == 0 or step == args.steps) and master:
            res = run_eval()
            if res:
                log(" ".join(f"{k} {v:.4f}" for k, v in res.items()))
                logger.log(res, step)
        if fid is not None and args.fid_every and (step % args.fid_every == 0 or step == args.steps):
            run_fid()  # collective: every rank samples its slice
        if args.merge_every and step >= args.merge_start * args.steps and step % args.merge_every == 0 and master:
            ckpt.save_merge(args.out, step, args.steps, den_cfg, te_cfg, te, den)
        if (args.ckpt_every and step % args.ckpt_every == 0) or step == args.steps:
            save()
            if distributed:
                dist.barrier()
    logger.close()
    if distributed:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
