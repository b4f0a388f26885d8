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
    """train.py's flags (the reference's train_pp.py takes train.py's parser and adds its own, train_pp.py:79-268),
    then the pipeline / OPD / service-rank flags; where both define a flag, this file's definition wins."""
    import train as train_cli
    p = train_cli.build_parser()
    p.description = __doc__
    for container in [p] + list(p._action_groups):  # a definition below replaces train.py's of the same flag
        container.conflict_handler = "resolve"
    a = p.add_argument
    a("--out", required=True)
    a("--data", default="data/aurora", help="shard directory (latents + LM caption rows); --synthetic N skips it")
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
    a("--act-checkpoint", nargs="?", const="full", default=None, choices=["full", "selective"],
      help="activation checkpointing per block: full recompute, or selective (keep GEMM / attention outputs, "
           "recompute the norms, q/k-norm + RoPE and SwiGLU in the backward)")
    a("--te-checkpoint", action="store_true", help="recompute the text encoder in the backward (with --act-checkpoint "
      "the whole first stage is recomputed already)")
    a("--steps", type=int, default=100)
    a("--lr-muon", type=float, default=1e-2)
    a("--lr-adam", type=float, default=3e-4)
    a("--wd", type=float, default=0.01)
    a("--t-shift", type=float, default=1.0)
    a("--t-shift-ref", type=float, default=0.0)
    a("--clip", type=float, default=1.0)
    a("--seed", type=int, default=0)
    a("--log-every", type=int, default=10)
    a("--ckpt-every", type=int, default=0, help="write latest.pt (+ per-rank optimizer files) every N steps")
    a("--keep-ckpt-steps", type=int, nargs="*", default=[], help="keep latest.pt of these steps as step_<n>.pt")
    a("--resume-opt-mismatch", action="store_true",
      help="resume weights / EMA from latest.pt with fresh optimizer state when the pipeline layout changed")
    a("--lat-dir", default="", help="latents from this directory (shard names as in --data)")
    a("--val-per-shard", action="store_true", help="(train.py's per-shard validation; not run by the pipeline trainer)")
    a("--lm-stage0", action="store_true", help="the frozen LM runs on stage 0 only (default: micro-batch k on stage "
      "k %% pp, gathered to stage 0)")
    a("--masked-attention-backend", default="tcgen05", choices=["tcgen05", "sdpa", "flex", "cudnn"],
      help="accepted for the reference's launch lines; the masked (caption) attention is always this framework's "
           "tcgen05 kernel")
    a("--bench", action="store_true", help="print per-step wall time and latent tokens / s")
    a("--dist-timeout", type=float, default=120.0, help="minutes")
    a("--mem-debug", action="store_true", help="print the memory breakdown after the first step")
    a("--mem-snapshot", default="", help="on an out-of-memory error, dump the CUDA allocator snapshot here")
    a("--profile-dir", default="", help="torch.profiler traces and kernel tables of --profile-steps steps")
    a("--profile-start", type=int, default=2)
    a("--profile-steps", type=int, default=2)
    a("--profile-ranks", type=int, nargs="*", default=[0])
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
    a("--opd-res-shifts", type=float, nargs="*", default=(), help="time shift per --opd-resolutions entry")
    a("--opd-res-batches", type=int, nargs="*", default=(), help="images per learner per --opd-resolutions entry")
    a("--opd-res-mb", type=int, nargs="*", default=(), help="micro-batch per --opd-resolutions entry")
    a("--opd-token-batch", action="store_true")
    a("--opd-actor", action="store_true", help="dedicated rollout-actor rank(s) (one per --opd-actor-gpus entry)")
    a("--opd-actor-gpus", type=int, nargs="*", default=[], help="GPUs of the rollout actors (nvidia-smi numbers)")
    a("--opd-actor-gpu", type=int, default=-1, help="a single rollout actor's GPU (same as --opd-actor-gpus N)")
    a("--opd-text-ahead", type=int, default=0,
      help="OPD: encode this many future caption batches per learner on the LM server (CPU queue, needs --lm-rank)")
    a("--opd-learner-profile", action="store_true", help="print the learner's per-phase times every log step")
    a("--opd-actor-profile", action="store_true", help="print the actor's per-job times")
    a("--opd-captions-only", action="store_true", help="OPD reads only captions from the shards (no latents)")
    a("--opd-balance-rollouts", action="store_true", help="round-robin the learners' rollout jobs over the actors")
    a("--opd-sort-rollouts", action="store_true", help="caption-length-sorted rollout batches")
    a("--opd-prefetch", action="store_true", help="after a cache's first update, roll out the next cycle's batch and "
      "leave its teacher request in flight during the replay updates; needs --opd-reuse > 1, local rollouts; the "
      "rollouts are stale by reuse - 1 updates")
    a("--opd-parts", type=int, default=1, help="split each rollout batch into this many teacher requests")
    a("--teacher-ranks", type=int, default=0)
    a("--teacher-size", default="teacher-4b", choices=sorted(SIZES))
    a("--teacher-ckpt", default="")
    a("--teacher-gpu", type=int, default=-1)
    a("--klein", action="store_true", help="FLUX.2-klein teacher (diffusers + weights; unavailable offline)")
    a("--klein-quant", default="", help="klein teacher weight quantization (with --klein)")
    a("--teacher-on-lm", action="store_true", help="the klein teacher shares the LM server's GPU (with --klein)")
    # frozen LM / VAE placement
    a("--lm-rank", type=int, default=0, help="dedicated LM server ranks (after the learners, actors and teachers)")
    a("--lm-gpu", type=int, default=-1, help="GPU of the (last) LM server")
    a("--lm-split", action="store_true", help="split the frozen LM's layers over the pipeline stages")
    a("--vae-rank", type=int, default=0, help="dedicated VAE server ranks (last); learners send uint8 images")
    a("--vae-gpu", type=int, default=-1)
    a("--vae-on-lm", action="store_true", help="the LM server also encodes the learners' images")
    a("--vae", default="", help="FLUX.2 VAE directory (default: the PatchEncoder stand-in)")
    a("--enc-vae", default="", help="encode --img-dir images with this VAE directory (same as --vae)")
    a("--enc-chunk", type=int, default=64, help="images per VAE encode call")
    a("--img-dir", default="", help="train on packed images (<shard>.img.bin) from this directory, VAE-encoded "
      "in the loop (on the VAE / LM server with --vae-rank / --vae-on-lm, else locally)")
    a("--img-extra", default="", help="(a second image directory; not run by the pipeline trainer)")
    a("--img-extra-val", action="store_true", help="(validation on --img-extra; not run by the pipeline trainer)")
    a("--vae-remote-frac", type=float, default=1.0,
      help="fraction of the images encoded on the VAE server (the rest locally on stage 0)")
    a("--skip-gpus", type=int, nargs="*", default=[])
    a("--random-lm", action="store_true",
      help="caption ids through a random-init Slayer-shaped LM of the encoder's width (no pretrained weights)")
    a("--lm-layers", type=int, default=4, help="--random-lm: LM depth")
    return p


# train.py flags the pipeline trainer does not run; they stop the run when set away from their defaults
UNSUPPORTED = dict(diloco=(0, "DiLoCo / MuLoCo outer steps"), repa_weight=(0.0, "REPA"), offload=(False, "offload"),
                   multi_res=([], "mixed-resolution steps (the reference needs --pp 1 for them too)"),
                   eval_only=(False, "--eval-only"), freeze_den=(False, "--freeze-den"),
                   te_experts=(None, "MoE text encoder"), te_quant=(None, "quantized text encoder"),
                   ema_cpu=(False, "--ema-cpu (a host EMA updated at DiLoCo syncs)"),
                   rope_random=(False, "RPE-2D random positions"), length_sort=(False, "--length-sort"),
                   val_per_shard=(False, "validation per shard group (train.py --eval-every)"),
                   img_extra=("", "a second image directory"), img_extra_val=(False, "validation on --img-extra"))


def check_flags(args):
    for dest, (default, what) in UNSUPPORTED.items():
        if hasattr(args, dest) and getattr(args, dest) != default:
            raise SystemExit(f"train_pp.py: {what} is not run by the pipeline trainer here; use train.py")
    if args.grad_comm == "powersgd":
        raise SystemExit("train_pp.py: PowerSGD gradient compression is not run by the pipeline trainer; use train.py")
    if args.klein or args.klein_quant or args.teacher_on_lm:
        raise SystemExit("train_pp.py: the FLUX.2-klein teacher is unavailable on this box (no diffusers, no "
                         "weights); use a DiT teacher (--teacher-size / --teacher-ckpt)")
    if args.opd_actor_gpu >= 0:
        args.opd_actor = True
        args.opd_actor_gpus = list(args.opd_actor_gpus) or [args.opd_actor_gpu]
    if args.enc_vae and not args.vae:
        args.vae = args.enc_vae
    assert not args.crop_res or args.micro_cond, "--crop-res needs --micro-cond"
    assert not args.opd_prefetch or ((args.dance_opd or args.diffusion_opd) and args.opd_reuse > 1
                                     and not args.opd_actor), \
        "--opd-prefetch needs OPD with --opd-reuse > 1 and local rollouts (no --opd-actor)"
    return args


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
    args = check_flags(build_parser().parse_args())
    from datetime import timedelta

    from trenowanie_generatora_obrazkow_b200.parallel.placement import RankLayout, local_device
    world_all = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    lay = RankLayout(world_all, actors=actor_count(args), teachers=args.teacher_ranks, lm_servers=args.lm_rank,
                     vae_servers=args.vae_rank)
    cuda = torch.cuda.is_available() and not os.environ.get("PP_CPU")  # PP_CPU=1: a CPU (Gloo) run on a GPU box
    if cuda:
        local = local_device(local_rank, torch.cuda.device_count(), lay, args.skip_gpus, args.lm_gpu, args.vae_gpu,
                             args.opd_actor_gpus, args.teacher_gpu)
        torch.cuda.set_device(local)
    backend = os.environ.get("DIST_BACKEND", "nccl" if cuda else "gloo")
    from trenowanie_generatora_obrazkow_b200.utils.profiling import arm_stack_dump
    arm_stack_dump()
    dist.init_process_group(backend, timeout=timedelta(minutes=args.dist_timeout))
    rank = dist.get_rank()
    device = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    role = lay.role(rank)
    if cuda and role != "learner":  # say which physical card a service rank got (nvidia-smi shows the bus id)
        bus = torch.cuda.get_device_properties(device).pci_bus_id
        print(f"rank {rank} ({role}): GPU {device.index}, PCI bus {bus:02X}", flush=True)
    den_cfg, te_cfg = make_configs(args.size, args.te_size, depth=args.depth)
    side = args.res // 16
    den_cfg = replace(den_cfg, latent_size=side, rope_ref=args.rope_ref, micro_cond=args.micro_cond)
    latest = os.path.join(args.out, "latest.pt")
    if os.path.exists(latest):  # the checkpoint's architecture wins (reference train_pp.py:1453-1460)
        from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig as _DC
        from trenowanie_generatora_obrazkow_b200.models.config import te_config_from_dict
        ck = ckpt.load(latest)
        den_cfg = replace(_DC(**ck["den_config"]), latent_size=side)
        te_cfg = te_config_from_dict(ck["te_config"])
        del ck
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
    if args.lm_stage0:  # the whole LM on stage 0
        if not tr.first:
            return None
        return torch.cat([lm.states(c.to(tr.device)).to(torch.bfloat16) for c in ids_all.split(mb)]).contiguous()
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


def shard_loader(args, te_cfg, den_cfg, mb, replica, dp, start_micro, with_data):
    """Micro-batches of --data (or --img-dir) for one replica: every stage of the replica walks the same sample and
    caption choices (TrainStream seeded by (seed, replica)); stage 0 also reads latents (or images) and
    micro-conditions, the others only caption rows."""
    from trenowanie_generatora_obrazkow_b200.data.shards import ShardStore, TrainStream, select_shards
    from trenowanie_generatora_obrazkow_b200.models.text import build_text_encoder
    root = args.img_dir or args.data
    tok_suffix = getattr(te_cfg, "tok_suffix", "")
    with torch.device("meta"):
        null_row = build_text_encoder(te_cfg).null_ids()
    alt_suffix = f"{tok_suffix}_pl" if args.pl_prob > 0 else ""  # --pl-prob: Polish token rows for that share
    assert not alt_suffix or tok_suffix, "--pl-prob needs a frozen-LM text encoder with its own token rows"
    names, _ = select_shards(root, args.fraction, tok_suffix, alt_suffix)
    side = args.res // 16
    kw = dict(lat_kind="lat" if side == 16 else f"lat{args.res}", lat_root=args.lat_dir)
    if with_data:
        kw.update(crops=[("lat" if r == 256 else f"lat{r}", "") for r in args.crop_res], crop_prob=args.crop_prob,
                  cond_base=den_cfg.micro_cond, img_res=args.res if args.img_dir else 0)
        if args.img_dir:
            kw.pop("crops"), kw.pop("crop_prob")
    store = ShardStore(root, names, tok_suffix, null_row, alt_suffix, args.pl_prob, **kw)
    stream = TrainStream(store, mb, replica, dp, args.seed, start_micro=start_micro, captions_only=not with_data)
    return iter(torch.utils.data.DataLoader(stream, batch_size=None, num_workers=min(args.workers, 2) if with_data
                                            else 0, persistent_workers=False))


def pp_val_data(args, te_cfg, den_cfg, tr, lm, lm_client, real, use_ids, device):
    """Validation set of the EMA evaluation, on global rank 0 (stage 0 of replica 0): --val-samples held-out images
    with their first captions as LM states (shards), or synthetic latents and states. None (with a note) when the
    LM runs split over the stages, where rank 0 cannot compute whole states."""
    from trenowanie_generatora_obrazkow_b200.data.shards import load_val, select_shards
    from trenowanie_generatora_obrazkow_b200.models.text import build_text_encoder
    if args.lm_split:
        print("[eval] skipped: with --lm-split no rank holds the whole LM for the validation captions", flush=True)
        return None
    side = den_cfg.latent_size
    g = torch.Generator().manual_seed(args.seed + 1)
    if real and not args.img_dir:
        tok_suffix = getattr(te_cfg, "tok_suffix", "")
        _, val_names = select_shards(args.data, args.fraction, tok_suffix)
        if not val_names:
            print("[eval] skipped: no held-out shard", flush=True)
            return None
        with torch.device("meta"):
            null_row = build_text_encoder(te_cfg).null_ids()
        lat, ids = load_val(args.data, val_names, args.val_samples, tok_suffix, null_row,
                            lat_kind="lat" if side == 16 else f"lat{args.res}", lat_root=args.lat_dir)
    elif real:  # packed images: the held-out images VAE-encoded once per configuration, then read from the cache
        from trenowanie_generatora_obrazkow_b200.data.shards import load_val_cached
        tok_suffix = getattr(te_cfg, "tok_suffix", "")
        _, val_names = select_shards(args.img_dir, args.fraction, tok_suffix)  # captions beside the images
        if not val_names:
            print("[eval] skipped: no held-out shard", flush=True)
            return None
        with torch.device("meta"):
            null_row = build_text_encoder(te_cfg).null_ids()
        enc = build_vae(args, device)
        encode = (lambda u8: enc(u8.to(device)).float().cpu())
        lat, ids = load_val_cached(
            os.path.join(args.out, "val_cache"),
            dict(names=val_names, n=args.val_samples, res=args.res, vae=args.vae or "patch-encoder", tok=tok_suffix),
            lambda: load_val(args.img_dir, val_names, args.val_samples, tok_suffix, null_row, img_res=args.res,
                             encode=encode))
    else:
        n = min(args.val_samples, 64)
        lat = torch.randn(n, den_cfg.latent_channels, side, side, generator=g)
        if not use_ids:
            return lat, torch.randn(n, te_cfg.max_tokens, te_cfg.lm_dim, generator=g)
        ids = synthetic_ids(g, n, te_cfg.max_tokens)
    if lm is not None:
        states = torch.cat([lm.states(c.to(device)).float().cpu() for c in ids.split(args.micro_batch)])
    elif lm_client is not None:
        states = lm_client.collect(lm_client.request(ids)).float().cpu()
    else:
        return lat, ids
    return lat, states


def fit_ids(ids, L):
    """Caption rows trimmed / padded (LM PAD) to the text encoder's max_tokens."""
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    if ids.shape[1] >= L:
        return ids[:, :L]
    return torch.cat([ids, torch.full((ids.shape[0], L - ids.shape[1]), LM_PAD, dtype=ids.dtype)], 1)


def run_fm(args, den_cfg, te_cfg, lay, device, ctl, text_group):
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import LMClient
    from trenowanie_generatora_obrazkow_b200.train import pp_checkpoint
    from trenowanie_generatora_obrazkow_b200.train.pp_trainer import PPTrainer, pp_groups
    from trenowanie_generatora_obrazkow_b200.utils import memory
    from trenowanie_generatora_obrazkow_b200.utils.profiling import TrainingProfile
    M = args.microbatches or 4 * args.pp
    world = lay.n_learners
    dp = world // args.pp
    groups = pp_groups(world, args.pp)  # collective: service ranks take part
    # Gloo groups for checkpoints (replica 0's stages; all learners), created by every rank in the same order
    save_group = dist.new_group(list(range(args.pp)), backend="gloo")
    learner_group = dist.new_group(list(range(world)), backend="gloo")
    role = lay.role(dist.get_rank())
    if role != "learner":
        serve(args, role, lay, te_cfg, device, ctl, text_group, args.pp)
        return
    cuda = device.type == "cuda"
    transport = args.grad_transport if args.grad_transport != "auto" else ("p2p" if cuda else "nccl")
    grad_comm = "nccl_fp32" if (args.grad_comm == "fp32" or not cuda) else ("p2p" if transport == "p2p" else
                                                                           "nccl_bf16")
    cfg = TrainConfig(global_batch=M * args.micro_batch * dp, micro_batch=args.micro_batch, steps=args.steps,
                      warmup=int(args.warmup_frac * args.steps), schedule=args.schedule, optimizer=args.optimizer,
                      lr_muon=args.lr_muon, lr_emb=args.lr_emb, lr_adam=args.lr_adam, lr_hidden=args.lr_hidden,
                      no_lr_batch_scaling=args.no_lr_batch_scaling, wd=args.wd, beta2=args.beta2,
                      momentum=args.momentum, ns_steps=args.ns_steps, cmuon=args.cmuon, muon_period=args.muon_period,
                      muon_gamma=args.muon_gamma, clip=args.clip, ema=args.ema, cfg_drop=args.cfg_drop,
                      seed=args.seed, t_shift=args.t_shift, grad_comm=grad_comm)
    tr = PPTrainer(den_cfg, te_cfg, cfg, device, args.pp, M, args.te_cost, world=world, groups=groups)
    tr.model.act_checkpoint = args.act_checkpoint or False  # per block: "full" or "selective"
    if tr.first and args.te_checkpoint:
        tr.model.te_checkpoint = True
    step, samples = pp_checkpoint.resume(tr, args.out, args.resume_opt_mismatch, group=learner_group)
    if step and tr.first and tr.replica == 0:
        print(f"[stage 0] resumed from {os.path.join(args.out, 'latest.pt')} at step {step}", flush=True)
    elif not step and args.init:  # this stage's tensors by name; a larger --depth grows identity blocks
        quiet = tr.replica != 0
        ckpt.init_named(ckpt.load(args.init), tr.named,
                        log=(lambda *a: None) if quiet else (lambda m: print(f"[stage {tr.stage}] {m}", flush=True)))
        ckpt.reset_ema(tr.ema)
    side, L = den_cfg.latent_size, te_cfg.max_tokens
    n = M * args.micro_batch
    root = args.img_dir or args.data
    real = not args.synthetic and os.path.isdir(root)
    if not args.synthetic and tr.first and tr.replica == 0:
        print(f"[stage 0] data: {'images' if args.img_dir else 'latents'} from {root}" if real else
              f"[stage 0] no data directory {root}: synthetic latents and captions", flush=True)
    use_ids = real or args.random_lm or te_cfg.backend != "states" or args.lm_rank > 0 or args.lm_split
    if real:
        assert te_cfg.backend != "states" or args.random_lm or args.lm_rank, \
            "shard data holds caption ids: use an LM text encoder (--te-size), --random-lm or an LM server"
        assert not (args.crop_res and args.lm_split), "--crop-res: the LM runs on stage 0 or an LM server"
        if args.crop_res and not args.lm_rank:
            args.lm_stage0 = True  # crop draws advance stage 0's generator: only stage 0's caption choice counts
    lm = lm_client = None
    width = te_cfg.lm_dim
    if use_ids:
        if args.lm_rank:
            if tr.first:
                lm_client = LMClient(lay.lm_server_of(tr.replica), width, device, ctl)
        elif tr.first or not args.lm_stage0:
            lm, width = build_lm(args, te_cfg, device)
            if args.lm_split:  # keep only this stage's slice of the LM (and the embedding on stage 0)
                nb = len(lm.model.blocks)
                lo, hi = tr.stage * nb // tr.pp, (tr.stage + 1) * nb // tr.pp
                for i in range(nb):
                    if not lo <= i < hi:
                        lm.model.blocks[i] = torch.nn.Identity()
    vae_client = vae_local = None
    images = bool(args.img_dir) or (not real and (args.vae_rank or args.vae_on_lm))
    if tr.first and images:
        if args.vae_rank or args.vae_on_lm:
            vae_srv = lay.lm_server_of(tr.replica) if args.vae_on_lm else \
                lay.vae_servers[tr.replica % len(lay.vae_servers)]
            vae_client = lm_client if (args.vae_on_lm and lm_client is not None) else LMClient(vae_srv, 0, device,
                                                                                             ctl)
        if vae_client is None or args.vae_remote_frac < 1.0:
            vae_local = build_vae(args, device)
    # caption ids are needed on every stage that runs LM work (all of them, unless the LM is on stage 0 / a server)
    reads_ids = real and (tr.first or (not args.lm_rank and not args.lm_stage0))
    loader = shard_loader(args, te_cfg, den_cfg, args.micro_batch, tr.replica, dp, step * M, tr.first) \
        if reads_ids else None
    g = torch.Generator().manual_seed(args.seed * 1000 + tr.replica)

    def encode(u8):
        """uint8 images -> latents: the first --vae-remote-frac on the VAE / LM server, the rest locally."""
        k = len(u8) if vae_local is None else int(round(args.vae_remote_frac * len(u8))) if vae_client else 0
        shape = lambda m: (m, den_cfg.latent_channels, side, side)
        h = vae_client.request_vae(u8[:k], shape(k)) if k else None
        parts = []
        for i in range(k, len(u8), args.enc_chunk):
            parts.append(vae_local(u8[i:i + args.enc_chunk].to(device)).float().cpu())
        remote = [LMClient.vae_collect(h).float().cpu()] if k else []
        return torch.cat(remote + parts)

    prof = TrainingProfile(args.profile_dir, args.profile_start, args.profile_steps, args.profile_ranks,
                           dist.get_rank()) if args.profile_dir else None
    eval_every = args.eval_every or 0
    val = pp_val_data(args, te_cfg, den_cfg, tr, lm, lm_client, real, use_ids, device) \
        if eval_every and dist.get_rank() == 0 else None
    from trenowanie_generatora_obrazkow_b200.utils.logging import RunLogger
    logger = RunLogger(args.out, vars(args), enabled=tr.last and tr.replica == 0 and not args.no_wandb,
                       project=args.wandb)  # log.jsonl (+ wandb when logged in) on the rank that holds the loss
    t0 = time.time()
    while step < args.steps:
        ts = time.time()
        if prof is not None:
            prof.step_begin(step)
        batch = dict(n=n, side=side, text_len=L)
        x0 = ids = cond = None
        if loader is not None:
            micros = [next(loader) for _ in range(M)]
            ids = fit_ids(torch.cat([m[1] for m in micros]), L)
            if tr.first:
                data = torch.cat([m[0] for m in micros])
                x0 = encode(data) if args.img_dir else data.float()
                if den_cfg.micro_cond and len(micros[0]) > 2:
                    cond = torch.cat([m[-1] for m in micros])
        elif tr.first:
            if images:  # synthetic images -> latents on the VAE / LM server rank
                x0 = encode(torch.randint(0, 256, (n, 3, args.res, args.res), generator=g, dtype=torch.uint8))
            else:
                x0 = torch.randn(n, den_cfg.latent_channels, side, side, generator=g)
        if use_ids:
            if ids is None:  # synthetic captions, identical on every stage of the replica
                ids = synthetic_ids(torch.Generator().manual_seed(args.seed * 7919 + 104729 * tr.replica + step),
                                    n, L)
            batch["lm_states"] = fm_text(args, tr, lm, lm_client, ids, M, args.micro_batch, width)
            batch["valid"] = ids.ne(LM_PAD)
        else:
            batch["lm_states"] = torch.randn(n, L, te_cfg.lm_dim, generator=g) if tr.first else None
        batch["x0"] = x0
        batch["cond"] = cond
        with memory.oom_guard(lambda: memory.report(dist.get_rank(), params=tr.params, opts=tr.opts),
                              args.mem_snapshot or None):
            loss = tr.step(batch)
        step += 1
        samples += n * dp
        if prof is not None:
            prof.step_end(step - 1)
        if args.mem_debug and step == 1:
            print(memory.report(dist.get_rank(), params=tr.params, opts=tr.opts,
                                ema=tr.ema.shadow if tr.ema is not None else None), flush=True)
        if args.bench and tr.last and tr.replica == 0:
            if cuda:
                torch.cuda.synchronize()
            dt = time.time() - ts
            print(f"[bench] step {step} {dt * 1e3:.1f} ms {n * dp * side * side / dt:.0f} latent-tokens/s",
                  flush=True)
        if tr.last and tr.replica == 0 and (step % args.log_every == 0 or step == args.steps):
            dt = time.time() - t0
            print(f"[stage {tr.stage}] step {step}/{args.steps} loss {loss.item():.4f} "
                  f"{args.log_every * n * dp / dt:.1f} img/s", flush=True)
            logger.log({"train/loss": loss.item(), "train/img_per_s": args.log_every * n * dp / dt,
                        "train/samples": samples}, step)
            t0 = time.time()
        if args.ckpt_every and (step % args.ckpt_every == 0 or step == args.steps):
            pp_checkpoint.save(tr, args.out, step, samples, vars(args), save_group, learner_group,
                               keep=step in args.keep_ckpt_steps)
        if eval_every and (step % eval_every == 0 or step == args.steps):  # EMA weights on the unsplit model
            res = pp_checkpoint.ema_eval(tr, save_group, val, device)
            if res is not None:
                print(f"[eval] step {step} | EMA " + " ".join(f"{k}={v:.4f}" for k, v in res.items()), flush=True)
                logger.log(res, step)  # enabled only where rank 0 is also the last stage (pp 1)
            dist.barrier(group=learner_group)
        if args.merge_every and step >= args.merge_start * args.steps and (
                step % args.merge_every == 0 or step == args.steps):  # raw weights for merge.py (WSM)
            pp_checkpoint.merge_save(tr, args.out, step, args.steps, save_group)
            dist.barrier(group=learner_group)
    logger.close()
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
    # checkpoint groups (Gloo): learner 0 alone gathers the weights; all learners agree on the commit
    save_group = dist.new_group(lay.learners[:1], backend="gloo")
    ckpt_group = dist.new_group(lay.learners, backend="gloo")
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
    from types import SimpleNamespace

    from trenowanie_generatora_obrazkow_b200.optim import EMA, lr_mult
    from trenowanie_generatora_obrazkow_b200.train import pp_checkpoint
    lrank = lay.learners.index(rank)
    named = [(pre, n, p) for pre, mod in (("te", te), ("den", den)) for n, p in mod.named_parameters()]
    # the same optimizer settings as the flow-matching trainers (TrainConfig.derived: LR scaled by the square root
    # of the global batch / 256 unless --no-lr-batch-scaling; EMA decay 0.9995 ** (batch / 256) unless --ema)
    ocfg = TrainConfig(global_batch=args.batch, ema=args.ema, no_lr_batch_scaling=args.no_lr_batch_scaling)
    lr_scale, ema_decay = ocfg.derived(n_learn)
    opts, _ = build_optimizers(named, optimizer=args.optimizer, lr_muon=args.lr_muon, lr_emb=args.lr_emb,
                               lr_adam=args.lr_adam, lr_hidden=args.lr_hidden, lr_scale=lr_scale, wd=args.wd,
                               beta2=args.beta2, momentum=args.momentum, ns_steps=args.ns_steps, cmuon=args.cmuon,
                               muon_period=args.muon_period, muon_gamma=args.muon_gamma, group=learner_group)
    ema = EMA([p for p in params if p.requires_grad], ema_decay) if lrank == 0 else None
    # what the pipeline checkpoint code reads: one stage (pp 1), one replica per learner (its optimizer file)
    state = SimpleNamespace(pp=1, dp=n_learn, stage=0, replica=lrank, named=named, ema=ema, opts=opts,
                            den_cfg=den_cfg, te_cfg=te_cfg, te_cost=0.0, step_idx=0)
    step0, samples = pp_checkpoint.resume(state, args.out, args.resume_opt_mismatch, group=ckpt_group)
    extra = getattr(state, "ckpt_extra", {})
    if step0 and lrank == 0:
        print(f"[learner] resumed from {os.path.join(args.out, 'latest.pt')} at step {step0} (the replay cache is "
              "not checkpointed: the first step rolls out a fresh batch)", flush=True)
    elif not step0 and args.init:  # the student from a trained checkpoint (EMA weights by name; growth as train.py)
        ckpt.init_named(ckpt.load(args.init), named, log=(lambda m: print(f"[learner] {m}", flush=True))
                        if lrank == 0 else (lambda *a: None))
        ckpt.reset_ema(ema)
    warmup = int(args.warmup_frac * args.steps)
    teacher = TeacherClient(lay.teachers, ctl, rank) if lay.teachers else None
    if teacher is None:
        tcfg = replace(SIZES[args.teacher_size], text_dim=den_cfg.text_dim, latent_size=den_cfg.latent_size)
        torch.manual_seed(1234)
        tte, tden = build_models(tcfg, te_cfg, device=device)
        if args.teacher_ckpt:
            ckpt.load_weights(ckpt.load(args.teacher_ckpt), tte, tden, use_ema=True)
        else:
            randomize_teacher(tden)
        teacher = DiTTeacher(tte, tden, args.opd_cfg)
    actors = [ActorClient(a, ctl, args.opd_states) for a in lay.actors]
    actor = actors[lrank % len(actors)] if actors else None
    sender = SnapshotSender(params, lay.actors, ctl) if (lay.actors and lrank == 0) else None
    learner = OPDLearner(te, den, teacher, args.opd_rollout_steps, args.opd_states, method, tuple(args.dance_beta),
                         args.t_shift, args.micro_batch, args.opd_reuse, args.opd_state_weighting, args.seed, lrank)
    per = max(args.micro_batch, args.batch // n_learn)
    L = te_cfg.max_tokens
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    lm_client = LMClient(lay.lm_server_of(lrank), te_cfg.lm_dim, device, ctl) if args.lm_rank else None

    def batch_shape(step):
        res = batch_resolution(args.seed, step, args.opd_resolutions, args.opd_res_weights or None, args.res)
        k = list(args.opd_resolutions).index(res) if args.opd_resolutions else 0
        if args.opd_res_batches:  # images per learner at this resolution
            return res, args.opd_res_batches[k]
        mult = token_batch_multiplier(res, args.res) if args.opd_token_batch else 1
        return res, per * mult

    cap_loader = local_lm = None
    if not args.synthetic and os.path.isdir(args.data):  # shard captions (OPD needs no latents); LM server or here
        cap_loader = shard_loader(args, te_cfg, den_cfg, args.micro_batch, lrank, n_learn,
                                  int(extra.get("opd_caption_micro", 0)), False)
        if not args.lm_rank:
            local_lm, _ = build_lm(args, te_cfg, device)
    cap_cache = {}
    # caption micro-batches read so far (from the resumed position) and where each fresh batch's captions began: a
    # checkpoint records where the next untrained batch starts, so batches drawn ahead are read again on resume
    cap_read = [int(extra.get("opd_caption_micro", 0))]
    cap_start = {}

    def caption_ids(step):  # the captions of a step (seeded by step so the lookahead can prepare them)
        B = batch_shape(step)[1]
        if cap_loader is None:
            return synthetic_ids(torch.Generator().manual_seed(args.seed * 7919 + 104729 * rank + step), B, L)
        if step not in cap_cache:  # shard captions in step order (the lookahead asks ahead, the loop later)
            cap_start[step] = cap_read[0]
            rows = []
            while sum(len(r) for r in rows) < B:
                rows.append(fit_ids(next(cap_loader)[1], L))
                cap_read[0] += 1
            cap_cache[step] = torch.cat(rows)[:B]
        return cap_cache[step]

    lookahead = None
    if args.opd_text_ahead:  # fresh batches only: one every --opd-reuse steps
        lookahead = TextLookahead(lambda at: dict(ids=caption_ids(at), texts=[], step=at),
                                  lambda job: encode_remote(job, lay.lm_server_of(lrank), ctl, text_group),
                                  step0, args.steps, args.opd_reuse, args.opd_text_ahead)

    def fresh_data(step):
        """(noise, LM states, valid) of the fresh batch that starts at ``step`` (replay steps draw nothing); seeded
        by the step, so a prefetch draws the same batch the loop would."""
        res, B = batch_shape(step)
        side = res // 16
        gs = torch.Generator().manual_seed(args.seed * 1_000_003 + 7919 * rank + step)
        noise = torch.randn(B, den_cfg.latent_channels, side, side, generator=gs).to(device)
        if lookahead is not None:
            job = lookahead.take(step)
            st, valid = job["lm"].to(device), job["ids"].ne(LM_PAD).to(device)
        elif lm_client is not None:
            ids = caption_ids(step)
            st, valid = lm_client.collect(lm_client.request(ids)), ids.ne(LM_PAD).to(device)
        elif local_lm is not None:
            ids = caption_ids(step)
            st = torch.cat([local_lm.states(c.to(device)).to(torch.bfloat16) for c in ids.split(args.micro_batch)])
            valid = ids.ne(LM_PAD).to(device)
        else:
            st = torch.randn(B, L, te_cfg.lm_dim, generator=gs).to(device)
            valid = torch.ones(B, L, dtype=torch.bool, device=device)
        cap_cache.pop(step, None)
        if args.opd_sort_rollouts:  # caption-length-sorted batch (similar lengths share rollout micro-batches)
            order = valid.sum(1).argsort(stable=True)
            st, valid, noise = st[order], valid[order], noise[order]
        return noise, st, valid

    def step_shift(step):
        res = batch_shape(step)[0]
        return resolution_shift(res, args.opd_resolutions, args.opd_res_shifts, args.t_shift_ref, args.t_shift,
                                args.res)

    def teacher_targets(states, t, kw):
        """Synchronous teacher targets of a fresh batch, in --opd-parts pieces."""
        bounds = [(i * len(states) // args.opd_parts, (i + 1) * len(states) // args.opd_parts)
                  for i in range(args.opd_parts)]
        return torch.cat([teacher.velocity(states[a:b], t[a:b], {k: v[a:b] for k, v in kw.items()})
                          for a, b in bounds if b > a])

    from trenowanie_generatora_obrazkow_b200.train.evaluate import evaluate
    eval_every = args.eval_every or 0
    use_ids = local_lm is not None or lm_client is not None  # else the loop's own random states (synthetic runs)
    val = pp_val_data(args, te_cfg, den_cfg, None, local_lm, lm_client, cap_loader is not None, use_ids, device) \
        if eval_every and lrank == 0 else None

    @torch.no_grad()
    def ema_eval():
        """Flow-matching validation loss of the student's EMA (swapped in, the live weights restored after)."""
        live = [p.detach().clone() for p in ema.params]
        ema.copy_to()
        try:
            return evaluate(te, den, val, device)
        finally:
            for p, w in zip(ema.params, live):
                p.copy_(w)

    from trenowanie_generatora_obrazkow_b200.utils.logging import RunLogger
    logger = RunLogger(args.out, vars(args), enabled=lrank == 0 and not args.no_wandb, project=args.wandb)
    version = 0
    # the next cycle's batch in preparation: {"step", "kw"} plus either "actor": (client, job) while the actor rolls
    # it out, or "x", "t", "teacher" (a deferred teacher request) once the states are here
    pending = None
    rep = lambda a: a.repeat_interleave(args.opd_states, dim=0)

    def actor_for(step):
        return actors[(lrank + step) % len(actors)] if args.opd_balance_rollouts else actor

    def states_to_teacher(p):
        """Actor job collected; the teacher's deferred request starts on its states."""
        client, job = p.pop("actor")
        p["x"], p["t"] = client.collect(job)
        p["teacher"] = teacher.request(p["x"], p["t"], p["kw"], chunks=args.opd_parts, deferred=True)

    t0 = time.time()
    for step in range(step0, args.steps):
        res, B = batch_shape(step)
        side = res // 16
        shift = step_shift(step)
        if args.opd_res_mb and args.opd_resolutions:
            learner.mb = args.opd_res_mb[list(args.opd_resolutions).index(res)]
        tp = time.time()
        fresh = learner.needs_fresh
        t_data = t_roll = t_teach = 0.0
        for p in params:
            p.grad = None
        sent = False
        if fresh and pending is not None:  # prepared during the last cycle (actor job or --opd-prefetch)
            assert pending["step"] == step, "a prepared OPD batch must start the next cycle"
            tt0 = time.time()
            if "actor" in pending:
                states_to_teacher(pending)
            learner.install(pending["x"], pending["t"], teacher.collect(pending["teacher"]), pending["kw"])
            t_teach = time.time() - tt0
            pending = None
        elif fresh:
            noise, st, valid = fresh_data(step)
            t_data = time.time() - tp
            tr0 = time.time()
            if actor is not None:
                if sender is not None:
                    version, sent = sender.send(), True
                states, t = actor_for(step).rollouts(noise, st, valid, step, version, shift=shift)
                kw_all = dict(lm_states=rep(st), valid=rep(valid))
            else:
                states, t, kw_all = learner.rollout_states(step, st, valid, noise, shift)
            t_roll = time.time() - tr0
            tt0 = time.time()
            learner.install(states, t, teacher_targets(states, t, kw_all), kw_all)
            t_teach = time.time() - tt0
        if fresh and actor is not None and step + learner.reuse < args.steps:
            # the actor rolls out the next cycle's batch with the weights of now while this cycle trains (states
            # reuse .. 2 reuse - 1 updates old when trained on, as the reference's actor cache)
            if sender is not None and not sent:
                version = sender.send()
            nxt = step + learner.reuse
            noise_n, st_n, valid_n = fresh_data(nxt)
            client = actor_for(nxt)
            pending = dict(step=nxt, kw=dict(lm_states=rep(st_n), valid=rep(valid_n)),
                           actor=(client, client.request(noise_n, st_n, valid_n, nxt, version, deferred=True,
                                                         shift=step_shift(nxt))))
        elif pending is not None and "actor" in pending and step == pending["step"] - 1:
            states_to_teacher(pending)  # last replay update of the cycle: the teacher scores meanwhile
        if fresh:
            samples += B * n_learn
        tl0 = time.time()
        loss = learner.step_grads(step)
        t_learn = time.time() - tl0
        if n_learn > 1:
            for p in params:
                if p.grad is not None:
                    dist.all_reduce(p.grad, group=learner_group)
                    p.grad /= n_learn
        torch.nn.utils.clip_grad_norm_(params, args.clip)
        set_lr(opts, lr_mult(step, args.steps, warmup, args.schedule))
        for o in opts:
            o.step()
        if ema is not None:
            ema.update(step + 1)
        t_pref = 0.0
        if args.opd_prefetch and pending is None and learner.uses == 1 and step + learner.reuse < args.steps:
            # after the first update of a cache: the next cycle's rollouts with the weights of now (stale by
            # reuse - 1 updates when trained on), its teacher request left in flight through the replay updates
            tf0, nxt = time.time(), step + learner.reuse
            mb_now = learner.mb
            if args.opd_res_mb and args.opd_resolutions:
                learner.mb = args.opd_res_mb[list(args.opd_resolutions).index(batch_shape(nxt)[0])]
            noise_n, st_n, valid_n = fresh_data(nxt)
            states_n, t_n, kw_n = learner.rollout_states(nxt, st_n, valid_n, noise_n, step_shift(nxt))
            learner.mb = mb_now
            pending = dict(step=nxt, x=states_n, t=t_n, kw=kw_n,
                           teacher=teacher.request(states_n, t_n, kw_n, chunks=args.opd_parts, deferred=True))
            t_pref = time.time() - tf0
        if args.bench and lrank == 0:  # learner throughput: student latent tokens trained per second
            torch.cuda.synchronize(device) if device.type == "cuda" else None
            dt = time.time() - tp
            toks = n_learn * B * args.opd_states * side * side
            line = (f"[bench] step {step} {dt * 1e3:.1f} ms {toks / dt:.0f} learner-latent-tokens/s res {res} "
                    f"(rollouts {t_roll * 1e3:.0f} ms, teacher {t_teach * 1e3:.0f} ms, student {t_learn * 1e3:.0f} ms)")
            if sender is not None and sender.last_copy is not None and t_roll:
                nb, ms = sender.last_copy
                line += f"; snapshot {nb / 1e9:.2f} GB in {ms:.2f} ms = {nb / ms / 1e6:.0f} GB/s"
            print(line, flush=True)
        if lrank == 0 and ((step + 1) % args.log_every == 0 or step + 1 == args.steps):
            print(f"[learner] step {step + 1}/{args.steps} opd loss {float(loss):.4f} res {res} "
                  f"{(time.time() - t0) / args.log_every:.2f} s/step", flush=True)
            logger.log({"opd/loss": float(loss), "opd/resolution": res, "opd/s_per_step":
                        (time.time() - t0) / args.log_every, "opd/reuse_pass": learner.uses,
                        "opd/fresh_trajectories": samples}, step + 1)
            if args.opd_learner_profile:
                print(f"[learner profile] captions {t_data * 1e3:.0f} ms, rollouts {t_roll * 1e3:.0f} ms, teacher "
                      f"{t_teach * 1e3:.0f} ms ({args.opd_parts} parts), student {t_learn * 1e3:.0f} ms, prefetch "
                      f"{t_pref * 1e3:.0f} ms", flush=True)
            t0 = time.time()
        if args.opd_actor_profile and actor is not None and t_roll:
            print(f"[actor profile] learner {lrank} step {step + 1}: {len(noise)} rollouts of "
                  f"{args.opd_rollout_steps} steps in {t_roll * 1e3:.0f} ms (request to reply)", flush=True)
        if eval_every and ((step + 1) % eval_every == 0 or step + 1 == args.steps):
            if ema is not None and val is not None:
                res = ema_eval()
                print(f"[eval] step {step + 1} | EMA " + " ".join(f"{k}={v:.4f}" for k, v in res.items()), flush=True)
                logger.log(res, step + 1)
            dist.barrier(group=ckpt_group)
        if args.ckpt_every and ((step + 1) % args.ckpt_every == 0 or step + 1 == args.steps):
            # the caption position saved is where the next untrained fresh batch starts (batches drawn ahead for
            # the actor, a prefetch or the lookahead are read again after a resume)
            nxt = pending["step"] if pending is not None else step + 1 + max(0, learner.reuse - learner.uses)
            pp_checkpoint.save(state, args.out, step + 1, samples, vars(args), save_group, ckpt_group,
                               keep=(step + 1) in args.keep_ckpt_steps,
                               extra=dict(opd_caption_micro=cap_start.get(nxt, cap_read[0])))
            for k in [k for k in cap_start if k < nxt]:
                del cap_start[k]
    logger.close()
    if lookahead is not None:
        lookahead.close()
    if lm_client is not None:
        lm_client.stop()
    if lrank == 0:
        if isinstance(teacher, TeacherClient):
            teacher.stop()
    dist.barrier(group=learner_group)
    if actors and lrank < len(actors):
        actors[lrank].stop()


if __name__ == "__main__":
    main()
