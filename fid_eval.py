"""Fréchet distance of saved checkpoints against held-out latents: latest.pt / snap_*.pt (EMA weights) and
merge/*.pt / merged.pt (raw weights), with the prompts, noise seeds and per-rank split of the in-training
evaluation (reference fid_eval.py:21-97).

  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 fid_eval.py --data data/x runs/r/latest.pt runs/r/snap_*.pt
  python fid_eval.py --data data/x runs/r/latest.pt --samples 256 --features latent

--features dino decodes with the FLUX.2 VAE (--vae) and uses DINOv2 features (needs timm, diffusers and local
weights); --features latent is the offline stand-in of train/fid.py (numbers not comparable to FD-DINOv2).
"""
import argparse
import json
import os
import time

import torch
import torch.distributed as dist

from trenowanie_generatora_obrazkow_b200.data.shards import load_val, select_shards
from trenowanie_generatora_obrazkow_b200.models import LMEncoderConfig, build_models, configs_from_ckpt
from trenowanie_generatora_obrazkow_b200.sampling.euler import sample
from trenowanie_generatora_obrazkow_b200.train.fid import DinoFeatures, LatentFeatures, fd_of_samples, my_prompts
from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("ckpts", nargs="+")
    p.add_argument("--data", required=True)
    p.add_argument("--features", choices=["dino", "latent"], default="dino")
    p.add_argument("--vae", default="", help="local FLUX.2 VAE directory (--features dino)")
    p.add_argument("--ref-vae", default="", help="decoder of the held-out (real) latents (default: --vae); fixing it "
                   "while --vae changes compares decoders against one reference")
    p.add_argument("--encoder", default="vit_base_patch14_reg4_dinov2.lvd142m", help="timm encoder (--features dino)")
    p.add_argument("--lang", default="", help="caption language of the held-out prompts ('' = the original; pl = "
                   "<shard>.tok_<enc>_pl.npy, frozen-LM text encoders only); images, noise and reference stay")
    p.add_argument("--random-lm", action="store_true", help="frozen-LM encoders: random stand-in LM (smoke runs)")
    p.add_argument("--samples", type=int, default=4096)
    p.add_argument("--val-samples", type=int, default=4096)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--cfg", type=float, default=3.0)
    p.add_argument("--shift", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--raw", action="store_true", help="raw weights even where the checkpoint has EMA weights")
    p.add_argument("--out", default=None, help="append one JSON line per checkpoint to this file")
    a = p.parse_args(argv)
    distributed = "RANK" in os.environ
    if distributed:
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
        rank, world, local = dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", 0))
    else:
        rank, world, local = 0, 1, 0
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    cache = {}
    for path in a.ckpts:
        t0 = time.time()
        ck = ckpt.load(path)
        den_cfg, te_cfg = configs_from_ckpt(ck)
        te, den = build_models(den_cfg, te_cfg)
        ckpt.load_weights(ck, te, den)
        ema = not a.raw and bool(ck.get("ema"))
        if ema:
            ckpt.load_weights(ck, te, den, use_ema=True)
        step = ck.get("step")
        del ck
        te.to(device).eval(), den.to(device).eval()
        lm = isinstance(te_cfg, LMEncoderConfig)
        if a.lang and not lm:
            raise SystemExit("fid_eval.py: --lang needs a frozen-LM text encoder (translated token rows)")
        base = getattr(te_cfg, "tok_suffix", "")
        key = base + (f"_{a.lang}" if a.lang else "")
        if key not in cache:
            # the held-out shards and images are chosen with the original rows; only the prompt rows change
            _, val_names = select_shards(a.data, 1.0, base)
            lat, ids = load_val(a.data, val_names, a.val_samples, key, te.null_ids())
            n = min(a.samples, len(ids))
            mine = my_prompts(n, rank, world)
            cache[key] = (lat[mine], ids[mine], n)
        real, ids, n = cache[key]
        if a.features == "latent":
            feats = ref_feats = LatentFeatures(den_cfg.latent_channels, seed=a.seed)
        else:
            feats = DinoFeatures(a.vae, a.encoder, device=device)
            ref_feats = DinoFeatures(a.ref_vae, a.encoder, device=device) if a.ref_vae else feats
        kw = dict(ids=ids.to(device))
        if lm:  # frozen-LM refiner: the LM's states of the prompt rows
            from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD, build_frozen_lm
            flm = build_frozen_lm(te_cfg, device, allow_random=a.random_lm)
            rows = ids.to(device)
            kw = dict(lm_states=flm.states(rows), valid=rows.ne(LM_PAD))
        with torch.no_grad():  # noise fixed by (seed, batch of this rank's prompts), as the reference
            z = sample(te, den, a.steps, a.cfg, a.seed, a.shift, batch=a.batch, **kw)
        fd = fd_of_samples(z.cpu() if a.features == "latent" else z, real, n, feats, real_features=ref_feats)
        if rank == 0:
            res = dict(ckpt=path, step=step, weights="ema" if ema else "raw", fd=round(fd, 3), features=a.features,
                       samples=n, steps=a.steps, cfg=a.cfg)
            print(f"{path}  step {step}  {res['weights']}  FD-{a.features} {fd:.3f}  ({time.time() - t0:.0f} s)",
                  flush=True)
            if a.out:
                with open(a.out, "a") as f:
                    f.write(json.dumps(res) + "\n")
    if distributed:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
