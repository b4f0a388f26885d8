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

# GPU numbers as nvidia-smi prints them (--lm-gpu, --vae-gpu, --skip-gpus, ...): before anything initialises CUDA
os.environ.setdefault("CUDA_DEVICE_ORDER", "PCI_BUS_ID")

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
    a("--opd-actor", action="store_true", help="dedicated rollout-actor rank(s) (one per --opd-actor-gpus entry)")
    a("--opd-actor-gpus", type=int, nargs="*", default=[], help="GPUs of the rollout actors (nvidia-smi numbers)")
    a("--opd-text-ahead", type=int, default=0,
      help="OPD: encode this many future caption batches per learner on the LM server (CPU queue, needs --lm-rank)")
    a("--teacher-ranks", type=int, default=0)
    a("--teacher-size", default="teacher-4b", choices=sorted(SIZES))
    a("--teacher-ckpt", default="")
    a("--teacher-gpu", type=int, default=-1)
    # frozen LM / VAE placement
    a("--lm-rank", type=int, default=0, help="dedicated LM server ranks (after the learners, actors and teachers)")
    a("--lm-gpu", type=int, default=-1, help="GPU of the (last) LM server")
    a("--lm-split", action="store_true", help="split the frozen LM's layers over the pipeline stages")
    a("--vae-rank", type=int, default=0, help="dedicated VAE server ranks (last); learners send uint8 images")
    a("--vae-gpu", type=int, default=-1)
    a("--vae-on-lm", action="store_true", help="the LM server also encodes the learners' images")
    a("--vae", default="", help="FLUX.2 VAE directory (default: the PatchEncoder stand-in)")
    a("--skip-gpus", type=int, nargs="*", default=[])
    a("--random-lm", action="store_true",
      help="caption ids through a random-init Slayer-shaped LM of the encoder's width (no pretrained weights)")
    a("--lm-layers", type=int, default=4, help="--random-lm: LM depth")
    return p


def actor_count(args):
    return (len(args.opd_actor_gpus) or 1) if args.opd_actor else 0


def build_lm(args, te_cfg, device):
    """Frozen LM for caption ids: the pretrained one the encoder config names, or the --random-lm stand-in.
    Returns (SlayerFrozenLM-like object with .states / .model, width)."""
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import SlayerFrozenLM, build_frozen_lm
    if args.random_lm or te_cfg.backend == "states":
        from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
        torch.manual_seed(4242)
        d = te_cfg.lm_dim
        gpt = GPT(GPTConfig(vocab=65536, n_layer=args.lm_layers, n_embd=d, n_head=max(1, d // 64), block=1024))
        with torch.no_grad():
            for blk in gpt.blocks[1:]:
                blk.vr_lambda.fill_(0.5)
        dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
        return SlayerFrozenLM(None, skip_last=0, model=gpt, device=device, dtype=dtype), d
    return build_frozen_lm(te_cfg, device), te_cfg.lm_dim


def build_vae(args, device):
    from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentEncoder, PatchEncoder
    return LatentEncoder(args.vae, device) if args.vae else PatchEncoder(device=device)


def synthetic_ids(g, n, L, vocab=60000):
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    ids = torch.randint(6, vocab, (n, L), generator=g)
    lens = torch.randint(3, L + 1, (n,), generator=g)
    ids[torch.arange(L)[None] >= lens[:, None]] = LM_PAD
    return ids


def serve(args, role, lay, te_cfg, device, ctl, text_group, pp):
    """Body of an LM or VAE server rank."""
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import LMService
    rank = dist.get_rank()
    opd = args.dance_opd or args.diffusion_opd
    step_pp = 1 if opd else pp
    if role == "lm":
        lm, width = build_lm(args, te_cfg, device)
        clients = lay.lm_clients(rank, step_pp)
        vae = build_vae(args, device) if args.vae_on_lm else None
        svc = LMService(lm.states, width, device, ctl, clients, vae=vae, text_group=text_group)
    else:
        clients = [r for r in lay.learners if r % step_pp == 0 and
                   lay.vae_servers[(r // step_pp) % len(lay.vae_servers)] == rank]
        svc = LMService(None, 0, device, ctl, clients, vae=build_vae(args, device))
    n = svc.serve()
    print(f"[{role} server {rank}] served {n} captions", flush=True)


def main():
    args = build_parser().parse_args()
    from datetime import timedelta

    from trenowanie_generatora_obrazkow_b200.parallel.placement import RankLayout, local_device
    world_all = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    lay = RankLayout(world_all, actors=actor_count(args), teachers=args.teacher_ranks, lm_servers=args.lm_rank,
                     vae_servers=args.vae_rank)
    cuda = torch.cuda.is_available()
    if cuda:
        local = local_device(local_rank, torch.cuda.device_count(), lay, args.skip_gpus, args.lm_gpu, args.vae_gpu,
                             args.opd_actor_gpus, args.teacher_gpu)
        torch.cuda.set_device(local)
    backend = os.environ.get("DIST_BACKEND", "nccl" if cuda else "gloo")
    dist.init_process_group(backend, timeout=timedelta(minutes=args.dist_timeout))
    rank = dist.get_rank()
    device = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    role = lay.role(rank)
    if cuda and role != "learner":  # say which physical card a service rank got (nvidia-smi shows the bus id)
        bus = torch.cuda.get_device_properties(device).pci_bus_id
        print(f"rank {rank} ({role}): GPU {device.index}, PCI bus {bus:02X}", flush=True)
    den_cfg, te_cfg = make_configs(args.size, args.te_size, depth=args.depth)
    side = args.res // 16
    den_cfg = replace(den_cfg, latent_size=side)
    # control planes (Gloo, any-source headers; CPU text jobs): every rank creates them, in the same order
    ctl = dist.new_group(backend="gloo")
    text_group = dist.new_group(backend="gloo")
    opd = args.dance_opd or args.diffusion_opd
    assert not args.vae_on_lm or args.lm_rank, "--vae-on-lm needs an LM server (--lm-rank)"
    assert opd or not (lay.actors or lay.teachers), "actor / teacher ranks belong to OPD runs"
    assert not (args.lm_split and args.lm_rank), "--lm-split and --lm-rank are alternatives"
    if opd:
        run_opd(args, den_cfg, te_cfg, lay, device, ctl, text_group)
    else:
        run_fm(args, den_cfg, te_cfg, lay, device, ctl, text_group)
    dist.barrier()
    dist.destroy_process_group()


def fm_text(args, tr, lm, lm_client, ids_all, M, mb, width):
    """LM states (M * mb, L, width) for this step's caption ids, on stage 0 (None elsewhere): from the LM server,
    the LM layer split over the stages, or per-stage LM work gathered to stage 0 (micro-batch k on stage k % pp)."""
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import gather_to_stage, lm_split_forward
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    base, s, pp = tr.replica * tr.pp, tr.stage, tr.pp
    if args.lm_rank:  # stage 0 holds the client
        return lm_client.collect(lm_client.request(ids_all)) if tr.first else None
    chunks = list(ids_all.split(mb))
    if args.lm_split:
        nb = len(lm.model.blocks)
        lo, hi = s * nb // pp, (s + 1) * nb // pp
        outs = lm_split_forward(lambda x: lm.model.run_slice(x, lo, hi), chunks, s, pp, base, tr.device, width,
                                carry_width=2 * width)  # stages after the first receive (residual, block-0 values)
    else:
        mine = {k: lm.states(chunks[k].to(tr.device)).to(torch.bfloat16).contiguous()
                for k in range(M) if k % pp == s}
        outs = gather_to_stage(mine, M, s, pp, 0, base)
    return torch.cat(outs) if outs is not None else None


def run_fm(args, den_cfg, te_cfg, lay, device, ctl, text_group):
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import LMClient
    from trenowanie_generatora_obrazkow_b200.train.pp_trainer import PPTrainer, pp_groups
    M = args.microbatches or 4 * args.pp
    world = lay.n_learners
    dp = world // args.pp
    groups = pp_groups(world, args.pp)  # collective: service ranks take part
    role = lay.role(dist.get_rank())
    if role != "learner":
        serve(args, role, lay, te_cfg, device, ctl, text_group, args.pp)
        return
    cfg = TrainConfig(global_batch=M * args.micro_batch * dp, micro_batch=args.micro_batch, steps=args.steps,
                      lr_muon=args.lr_muon, lr_adam=args.lr_adam, wd=args.wd, clip=args.clip, seed=args.seed,
                      t_shift=args.t_shift, grad_comm="p2p" if device.type == "cuda" else "nccl_fp32")
    tr = PPTrainer(den_cfg, te_cfg, cfg, device, args.pp, M, args.te_cost, world=world, groups=groups)
    side, L = den_cfg.latent_size, te_cfg.max_tokens
    n = M * args.micro_batch
    use_ids = args.random_lm or te_cfg.backend != "states" or args.lm_rank > 0 or args.lm_split
    lm = lm_client = None
    width = te_cfg.lm_dim
    if use_ids:
        if args.lm_rank:
            if tr.first:
                lm_client = LMClient(lay.lm_server_of(tr.replica), width, device, ctl)
        else:
            lm, width = build_lm(args, te_cfg, device)
            if args.lm_split:  # keep only this stage's slice of the LM (and the embedding on stage 0)
                nb = len(lm.model.blocks)
                lo, hi = tr.stage * nb // tr.pp, (tr.stage + 1) * nb // tr.pp
                for i in range(nb):
                    if not lo <= i < hi:
                        lm.model.blocks[i] = torch.nn.Identity()
    vae_client = None
    if tr.first and (args.vae_rank or args.vae_on_lm):
        vae_srv = lay.lm_server_of(tr.replica) if args.vae_on_lm else \
            lay.vae_servers[tr.replica % len(lay.vae_servers)]
        vae_client = lm_client if (args.vae_on_lm and lm_client is not None) else LMClient(vae_srv, 0, device, ctl)
    g = torch.Generator().manual_seed(args.seed * 1000 + tr.replica)
    t0 = time.time()
    for step in range(args.steps):
        batch = dict(n=n, side=side, text_len=L)
        x0 = None
        if tr.first:
            if vae_client is not None:  # images -> latents on the VAE / LM server rank
                u8 = torch.randint(0, 256, (n, 3, args.res, args.res), generator=g, dtype=torch.uint8)
                h = vae_client.request_vae(u8, (n, den_cfg.latent_channels, side, side))
                x0 = LMClient.vae_collect(h)
            else:
                x0 = torch.randn(n, den_cfg.latent_channels, side, side, generator=g)
        if use_ids:
            # identical on every stage of the replica: a generator of its own, seeded by (replica, step)
            ids = synthetic_ids(torch.Generator().manual_seed(args.seed * 7919 + 104729 * tr.replica + step), n, L)
            batch["lm_states"] = fm_text(args, tr, lm, lm_client, ids, M, args.micro_batch, width)
            batch["valid"] = ids.ne(LM_PAD)
        else:
            batch["lm_states"] = torch.randn(n, L, te_cfg.lm_dim, generator=g) if tr.first else None
        batch["x0"] = x0
        loss = tr.step(batch)
        if tr.last and tr.replica == 0 and ((step + 1) % args.log_every == 0 or step + 1 == args.steps):
            dt = time.time() - t0
            print(f"[stage {tr.stage}] step {step + 1}/{args.steps} loss {loss.item():.4f} "
                  f"{args.log_every * n * dp / dt:.1f} img/s", flush=True)
            t0 = time.time()
        if args.ckpt_every and (step + 1) % args.ckpt_every == 0 and tr.replica == 0:
            os.makedirs(args.out, exist_ok=True)
            ckpt.atomic_save({f"{pre}.{nm}": p.detach().cpu() for pre, nm, p in tr.named},
                             os.path.join(args.out, f"stage{tr.stage}.pt"))
    for c in {id(c): c for c in (lm_client, vae_client) if c is not None}.values():
        c.stop()


@torch.no_grad()
def randomize_teacher(den, std=0.02):
    """A random-init teacher without a checkpoint: give the zero-initialised output layers (adaLN, cross-attention
    output, patch_out) small random values so its velocity targets are not identically zero."""
    g = torch.Generator(device="cpu").manual_seed(4321)
    for name, p in den.named_parameters():
        if name.startswith(("ada.", "patch_out.")) or name.endswith(("cross.out.weight", "mod_table")):
            p.copy_((torch.randn(p.shape, generator=g) * std).to(p.device, p.dtype))


def run_opd(args, den_cfg, te_cfg, lay, device, ctl, text_group):
    from trenowanie_generatora_obrazkow_b200.models import build_models
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    from trenowanie_generatora_obrazkow_b200.optim import build_optimizers, set_lr
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import LMClient, TextLookahead, encode_remote
    from trenowanie_generatora_obrazkow_b200.parallel.roles import (ActorClient, RolloutActor, SnapshotSender,
                                                                    TeacherClient, TeacherServer)
    from trenowanie_generatora_obrazkow_b200.train.opd import (DiTTeacher, OPDLearner, batch_resolution,
                                                                resolution_shift, token_batch_multiplier)
    assert args.pp == 1, "OPD runs with --pp 1 (as in the reference)"
    assert not args.opd_text_ahead or args.lm_rank, "--opd-text-ahead needs an LM server (--lm-rank)"
    rank = dist.get_rank()
    n_learn = lay.n_learners
    role = lay.role(rank)
    learner_group = dist.new_group(lay.learners)
    if role in ("lm", "vae"):
        serve(args, role, lay, te_cfg, device, ctl, text_group, 1)
        return
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
    lm_client = LMClient(lay.lm_server_of(lrank), te_cfg.lm_dim, device, ctl) if args.lm_rank else None

    def batch_shape(step):
        res = batch_resolution(args.seed, step, args.opd_resolutions, args.opd_res_weights or None, args.res)
        mult = token_batch_multiplier(res, args.res) if args.opd_token_batch else 1
        return res, per * mult

    def caption_ids(step):  # the captions of a step (synthetic, seeded by step so the lookahead can prepare them)
        return synthetic_ids(torch.Generator().manual_seed(args.seed * 7919 + 104729 * rank + step),
                             batch_shape(step)[1], L)

    lookahead = None
    if args.opd_text_ahead:
        lookahead = TextLookahead(lambda at: dict(ids=caption_ids(at), texts=[], step=at),
                                  lambda job: encode_remote(job, lay.lm_server_of(lrank), ctl, text_group),
                                  0, args.steps, 1, args.opd_text_ahead)
    version = 0
    t0 = time.time()
    for step in range(args.steps):
        res, B = batch_shape(step)
        side = res // 16
        shift = resolution_shift(res, args.opd_resolutions, (), args.t_shift_ref, args.t_shift, args.res)
        noise = torch.randn(B, den_cfg.latent_channels, side, side, generator=g).to(device)
        if lookahead is not None:
            job = lookahead.take(step)
            st, valid = job["lm"].to(device), job["ids"].ne(LM_PAD).to(device)
        elif lm_client is not None:
            ids = caption_ids(step)
            st, valid = lm_client.collect(lm_client.request(ids)), ids.ne(LM_PAD).to(device)
        else:
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
    if lookahead is not None:
        lookahead.close()
    if lm_client is not None:
        lm_client.stop()
    if lrank == 0:
        if isinstance(teacher, TeacherClient):
            teacher.stop()
    dist.barrier(group=learner_group)
    if actor is not None and lrank < len(lay.actors):
        actor.stop()


if __name__ == "__main__":
    main()
