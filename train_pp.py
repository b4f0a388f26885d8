"""Pipeline-parallel flow-matching training and on-policy distillation (OPD) with separate actor / teacher GPUs.

  # 1F1B pipeline, 4 stages x 2 replicas, 1024 px, 8 micro-batches of 4 per replica
  torchrun --nproc_per_node 8 train_pp.py --out runs/pp --synthetic 4096 --size 1.24b --te-size states1024 \
      --pp 4 --microbatches 8 --micro-batch 4 --res 1024 --steps 100
  # OPD: 4 learners, 2 rollout actors, 2 teacher GPUs (a frozen DiT teacher), DanceOPD, 8-step rollouts
  torchrun --nproc_per_node 8 train_pp.py --out runs/opd --synthetic 4096 --size 1.24b --te-size states1024 \
      --dance-opd --opd-actor-gpus 2 --teacher-ranks 2 --teacher-size teacher-4b --opd-rollout-steps 8 --opd-cfg 3

Flag names follow the reference's train_pp.py (train_pp.py:79-268). The reference's OPD teacher is FLUX.2-klein
through diffusers; here the teacher interface takes any frozen denoiser (--teacher-size preset, random init, or
--teacher-ckpt), since no pretrained teacher weights are available offline.
"""
import argparse
import os
import time
from dataclasses import replace

import torch
import torch.distributed as dist

from trenowanie_generatora_obrazkow_b200.models import SIZES, TE_SIZES, DenoiserConfig, make_configs
from trenowanie_generatora_obrazkow_b200.models.config import LMEncoderConfig
from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig
from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt


def build_parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    a = p.add_argument
    a("--out", required=True)
    a("--data", default="data/aurora")
    a("--synthetic", type=int, default=0)
    a("--size", default="1.5b", choices=sorted(SIZES))
    a("--depth", type=int, default=None)
    a("--te-size", default="states1024", choices=sorted(TE_SIZES))
    a("--res", type=int, default=256)
    a("--batch", type=int, default=512, help="global batch (flow matching)")
    a("--pp", type=int, default=1)
    a("--microbatches", type=int, default=None, help="micro-batches per step and replica (default 4 x pp)")
    a("--micro-batch", type=int, default=4)
    a("--te-cost", type=float, default=1.0, help="text encoder + stem cost in blocks (stage balancing)")
    a("--act-checkpoint", action="store_true")
    a("--steps", type=int, default=100)
    a("--lr-muon", type=float, default=1e-2)
    a("--lr-adam", type=float, default=3e-4)
    a("--wd", type=float, default=0.01)
    a("--t-shift", type=float, default=1.0)
    a("--t-shift-ref", type=float, default=0.0)
    a("--clip", type=float, default=1.0)
    a("--seed", type=int, default=0)
    a("--log-every", type=int, default=10)
    a("--ckpt-every", type=int, default=0)
    a("--dist-timeout", type=float, default=120.0, help="minutes")
    # OPD
    a("--dance-opd", action="store_true")
    a("--diffusion-opd", action="store_true")
    a("--dance-beta", type=float, nargs=2, default=(5.0, 2.0))
    a("--opd-states", type=int, default=2)
    a("--opd-rollout-steps", type=int, default=8)
    a("--opd-cfg", type=float, default=3.0)
    a("--opd-reuse", type=int, default=1)
    a("--opd-state-weighting", action="store_true")
    a("--opd-resolutions", type=int, nargs="*", default=())
    a("--opd-res-weights", type=float, nargs="*", default=())
    a("--opd-token-batch", action="store_true")
    a("--opd-actor-gpus", type=int, default=0)
    a("--teacher-ranks", type=int, default=0)
    a("--teacher-size", default="teacher-4b", choices=sorted(SIZES))
    a("--teacher-ckpt", default="")
    return p


def main():
    args = build_parser().parse_args()
    from datetime import timedelta
    local = int(os.environ.get("LOCAL_RANK", 0))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    backend = os.environ.get("DIST_BACKEND", "nccl" if torch.cuda.is_available() else "gloo")
    dist.init_process_group(backend, timeout=timedelta(minutes=args.dist_timeout))
    rank, world = dist.get_rank(), dist.get_world_size()
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    den_cfg, te_cfg = make_configs(args.size, args.te_size, depth=args.depth)
    side = args.res // 16
    den_cfg = replace(den_cfg, latent_size=side)
    opd = args.dance_opd or args.diffusion_opd
    if opd:
        run_opd(args, den_cfg, te_cfg, rank, world, device)
    else:
        run_fm(args, den_cfg, te_cfg, rank, world, device)
    dist.destroy_process_group()


def run_fm(args, den_cfg, te_cfg, rank, world, device):
    from trenowanie_generatora_obrazkow_b200.train.pp_trainer import PPTrainer
    M = args.microbatches or 4 * args.pp
    dp = world // args.pp
    cfg = TrainConfig(global_batch=M * args.micro_batch * dp, micro_batch=args.micro_batch, steps=args.steps,
                      lr_muon=args.lr_muon, lr_adam=args.lr_adam, wd=args.wd, clip=args.clip, seed=args.seed,
                      t_shift=args.t_shift, grad_comm="p2p" if device.type == "cuda" else "nccl_fp32")
    tr = PPTrainer(den_cfg, te_cfg, cfg, device, args.pp, M, args.te_cost)
    side, L = den_cfg.latent_size, te_cfg.max_tokens
    n = M * args.micro_batch
    g = torch.Generator().manual_seed(args.seed * 1000 + tr.replica)
    t0 = time.time()
    for step in range(args.steps):
        x0 = torch.randn(n, den_cfg.latent_channels, side, side, generator=g) if tr.first else None
        st = torch.randn(n, L, te_cfg.lm_dim, generator=g) if tr.first else None
        loss = tr.step(dict(x0=x0, lm_states=st, n=n, side=side, text_len=L))
        if tr.last and tr.replica == 0 and ((step + 1) % args.log_every == 0 or step + 1 == args.steps):
            dt = time.time() - t0
            print(f"[stage {tr.stage}] step {step + 1}/{args.steps} loss {loss.item():.4f} "
                  f"{args.log_every * n * dp / dt:.1f} img/s", flush=True)
            t0 = time.time()
        if args.ckpt_every and (step + 1) % args.ckpt_every == 0 and tr.replica == 0:
            os.makedirs(args.out, exist_ok=True)
            ckpt.atomic_save({f"{pre}.{nm}": p.detach().cpu() for pre, nm, p in tr.named},
                             os.path.join(args.out, f"stage{tr.stage}.pt"))


@torch.no_grad()
def randomize_teacher(den, std=0.02):
    """A random-init teacher without a checkpoint: give the zero-initialised output layers (adaLN, cross-attention
    output, patch_out) small random values so its velocity targets are not identically zero."""
    g = torch.Generator(device="cpu").manual_seed(4321)
    for name, p in den.named_parameters():
        if name.startswith(("ada.", "patch_out.")) or name.endswith(("cross.out.weight", "mod_table")):
            p.copy_((torch.randn(p.shape, generator=g) * std).to(p.device, p.dtype))


def run_opd(args, den_cfg, te_cfg, rank, world, device):
    from trenowanie_generatora_obrazkow_b200.models import build_models
    from trenowanie_generatora_obrazkow_b200.optim import build_optimizers, set_lr
    from trenowanie_generatora_obrazkow_b200.parallel.roles import (ActorClient, RoleLayout, RolloutActor,
                                                                    SnapshotSender, TeacherClient, TeacherServer)
    from trenowanie_generatora_obrazkow_b200.train.opd import (DiTTeacher, OPDLearner, batch_resolution,
                                                                resolution_shift, token_batch_multiplier)
    assert args.pp == 1, "OPD runs with --pp 1 (as in the reference)"
    n_learn = world - args.opd_actor_gpus - args.teacher_ranks
    lay = RoleLayout(world, n_learn, args.opd_actor_gpus, args.teacher_ranks)
    role = lay.role(rank)
    ctl = dist.new_group(backend="gloo")
    learner_group = dist.new_group(lay.learners)
    method = "dance" if args.dance_opd else "diffusion"
    kw = dict(K=args.opd_rollout_steps, m=args.opd_states, method=method, beta=tuple(args.dance_beta),
              shift=args.t_shift, mb=args.micro_batch, seed=args.seed,
              dtype=torch.float32)
    if role == "teacher":
        tcfg = replace(SIZES[args.teacher_size], text_dim=den_cfg.text_dim, latent_size=den_cfg.latent_size)
        torch.manual_seed(1234)
        tte, tden = build_models(tcfg, te_cfg, device=device)
        if args.teacher_ckpt:
            ckpt.load_weights(ckpt.load(args.teacher_ckpt), tte, tden, use_ema=True)
        else:
            randomize_teacher(tden)
        served = TeacherServer(DiTTeacher(tte, tden, args.opd_cfg), device, ctl).serve()
        print(f"[teacher {rank}] served {served} requests", flush=True)
        return
    torch.manual_seed(args.seed)
    te, den = build_models(den_cfg, te_cfg, device=device)
    params = list(te.parameters()) + list(den.parameters())
    if role == "actor":
        jobs = RolloutActor(te, den, params, device, ctl, kw).serve()
        print(f"[actor {rank}] {jobs} rollout jobs", flush=True)
        return
    # ---- learner ----
    lrank = lay.learners.index(rank)
    named = [(pre, n, p) for pre, mod in (("te", te), ("den", den)) for n, p in mod.named_parameters()]
    opts, _ = build_optimizers(named, lr_muon=args.lr_muon, lr_adam=args.lr_adam, wd=args.wd, group=learner_group)
    teacher = TeacherClient(lay.teachers, ctl, rank) if lay.teachers else None
    if teacher is None:
        tcfg = replace(SIZES[args.teacher_size], text_dim=den_cfg.text_dim, latent_size=den_cfg.latent_size)
        torch.manual_seed(1234)
        tte, tden = build_models(tcfg, te_cfg, device=device)
        randomize_teacher(tden)
        teacher = DiTTeacher(tte, tden, args.opd_cfg)
    actor = ActorClient(lay.actors[lrank % len(lay.actors)], ctl, args.opd_states) if lay.actors else None
    sender = SnapshotSender(params, lay.actors, ctl) if (lay.actors and lrank == 0) else None
    learner = OPDLearner(te, den, teacher, args.opd_rollout_steps, args.opd_states, method, tuple(args.dance_beta),
                         args.t_shift, args.micro_batch, args.opd_reuse, args.opd_state_weighting, args.seed, lrank)
    per = max(args.micro_batch, args.batch // n_learn)
    L = te_cfg.max_tokens
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    version = 0
    t0 = time.time()
    for step in range(args.steps):
        res = batch_resolution(args.seed, step, args.opd_resolutions, args.opd_res_weights or None, args.res)
        mult = token_batch_multiplier(res, args.res) if args.opd_token_batch else 1
        B, side = per * mult, res // 16
        shift = resolution_shift(res, args.opd_resolutions, (), args.t_shift_ref, args.t_shift, args.res)
        noise = torch.randn(B, den_cfg.latent_channels, side, side, generator=g).to(device)
        st = torch.randn(B, L, te_cfg.lm_dim, generator=g).to(device)
        valid = torch.ones(B, L, dtype=torch.bool, device=device)
        for p in params:
            p.grad = None
        if actor is not None and (learner.cache is None or learner.uses >= learner.reuse):
            if sender is not None:
                version = sender.send()
            states, t = actor.rollouts(noise, st, valid, step, version)
            rep = lambda a: a.repeat_interleave(args.opd_states, dim=0)
            target = teacher.velocity(states, t, dict(lm_states=rep(st), valid=rep(valid)))
            learner.cache = dict(x=states, t=t, target=target, text_kw=dict(lm_states=rep(st), valid=rep(valid)),
                                 errors=None)
            learner.uses = 0
        loss = learner.step_grads(step, st, valid, noise, shift)
        if n_learn > 1:
            for p in params:
                if p.grad is not None:
                    dist.all_reduce(p.grad, group=learner_group)
                    p.grad /= n_learn
        torch.nn.utils.clip_grad_norm_(params, args.clip)
        set_lr(opts, 1.0)
        for o in opts:
            o.step()
        if lrank == 0 and ((step + 1) % args.log_every == 0 or step + 1 == args.steps):
            print(f"[learner] step {step + 1}/{args.steps} opd loss {float(loss):.4f} res {res} "
                  f"{(time.time() - t0) / args.log_every:.2f} s/step", flush=True)
            t0 = time.time()
    if lrank == 0:
        if isinstance(teacher, TeacherClient):
            teacher.stop()
    dist.barrier(group=learner_group)
    if actor is not None and lrank < len(lay.actors):
        actor.stop()


if __name__ == "__main__":
    main()
