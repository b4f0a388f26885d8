"""Images (or latents) from a training checkpoint or an export, with the Euler / CFG sampler.

  python sample_ckpt.py runs/x/latest.pt --out-dir out --prompt "a red cat" "rudy kot" --steps 50 --cfg 3
  python sample_ckpt.py runs/x/latest.pt --out-dir exports/x --export

EMA weights by default (--raw for the trained weights); --res / --rope-ref / --attn-scale / --t-shift / --batch as
in the reference's sample_ckpt.py (sample_ckpt.py:119-146). Decoding needs the FLUX.2 VAE decoder (--vae, a local
diffusers AutoencoderKLFlux2 directory); without it the normalised latents are saved (latents.pt) together with a
small false-colour preview of latent channels per prompt. --export writes text_encoder/ and transformer/
safetensors + config.json (the reference's legacy export layout).
"""
import argparse
import json
import os
from dataclasses import asdict, replace

import numpy as np
import torch

from trenowanie_generatora_obrazkow_b200.models import LMEncoderConfig, build_models, configs_from_ckpt
from trenowanie_generatora_obrazkow_b200.models.frozen_lm import build_frozen_lm
from trenowanie_generatora_obrazkow_b200.models.text import LM_PAD
from trenowanie_generatora_obrazkow_b200.sampling.euler import sample
from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt
from trenowanie_generatora_obrazkow_b200.utils.tokenize import load_tokenizer, tokenize

PROMPTS = ["a red fox sitting in the snow", "a lighthouse on a cliff at sunset", "a bowl of ramen, studio photo",
           "an old wooden boat on a calm lake", "a cat wearing a tiny crown", "a futuristic city at night",
           "a watercolor painting of mountains", "a vintage car on a desert road"]


def load(src, raw=False, res=None, rope_ref=None):
    """(te, den, info) from a .pt checkpoint or an export directory (text_encoder/, transformer/)."""
    if src.endswith(".pt"):
        ck = ckpt.load(src)
        den_cfg, te_cfg = configs_from_ckpt(ck)
    else:
        from safetensors.torch import load_file
        from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, te_config_from_dict
        with open(os.path.join(src, "transformer", "config.json")) as f:
            den_cfg = DenoiserConfig(**{k: v for k, v in json.load(f).items()
                                        if k in DenoiserConfig.__dataclass_fields__})
        with open(os.path.join(src, "text_encoder", "config.json")) as f:
            te_cfg = te_config_from_dict({k: v for k, v in json.load(f).items() if not k.startswith("_")})
        ck = dict(te=load_file(os.path.join(src, "text_encoder", "diffusion_pytorch_model.safetensors")),
                  den=load_file(os.path.join(src, "transformer", "diffusion_pytorch_model.safetensors")))
    if res:
        den_cfg = replace(den_cfg, latent_size=res // 16)
    if rope_ref is not None:
        den_cfg = replace(den_cfg, rope_ref=rope_ref)
    te, den = build_models(den_cfg, te_cfg)
    ckpt.load_weights(ck, te, den, strict=False)
    use_ema = bool(ck.get("ema")) and not raw
    if use_ema:
        ckpt.load_weights(ck, te, den, use_ema=True)
    return te, den, dict(step=ck.get("step"), weights="EMA" if use_ema else "raw")


def latent_preview(z):
    """(B, 128, h, w) latents -> (B, h, w, 3) uint8 false colour of three channel groups (not a decoded image)."""
    k = z.shape[1] // 3
    g = z.float()[:, :3 * k].reshape(z.shape[0], 3, k, *z.shape[2:]).mean(2)
    g = (g - g.amin(dim=(2, 3), keepdim=True)) / (g.amax(dim=(2, 3), keepdim=True) - g.amin(dim=(2, 3), keepdim=True)
                                                  + 1e-6)
    return (g.permute(0, 2, 3, 1).cpu().numpy() * 255).round().astype(np.uint8)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("ckpt")
    p.add_argument("--out-dir", required=True)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--cfg", type=float, default=3.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--raw", action="store_true")
    p.add_argument("--vae", default=None, help="local FLUX.2 VAE (diffusers) directory for decoding")
    p.add_argument("--prompt", nargs="+", default=None)
    p.add_argument("--tokenizer", default=None, help="tokenizer.json of the text encoder (default: byte stand-in)")
    p.add_argument("--random-lm", action="store_true", help="frozen-LM encoders: random stand-in LM")
    p.add_argument("--res", type=int, default=None)
    p.add_argument("--rope-ref", type=int, default=None)
    p.add_argument("--attn-scale", type=float, default=1.0)
    p.add_argument("--t-shift", type=float, default=1.0)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--export", action="store_true")
    a = p.parse_args()
    device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    os.makedirs(a.out_dir, exist_ok=True)
    te, den, info = load(a.ckpt, a.raw, a.res, a.rope_ref)
    te_cfg, den_cfg = te.config, den.config
    print(f"{a.ckpt}: step {info['step']}, {info['weights']} weights")
    te.to(device).eval(), den.to(device).eval()
    for m in den.modules():
        if hasattr(m, "logit_mult"):
            m.logit_mult = a.attn_scale
    # the showcase prompts in English and in Polish (the same noise for prompt k in both grids, as the reference's
    # sampler does), or the user's own prompts
    if a.prompt:
        sets = [("", a.prompt)]
    else:
        import sample as showcase
        sets = [("en_", showcase.PROMPTS), ("pl_", showcase.PROMPTS_PL)]
    lm = isinstance(te_cfg, LMEncoderConfig)
    frozen = build_frozen_lm(te_cfg, device, allow_random=a.random_lm) if lm else None
    tok = load_tokenizer(a.tokenizer, getattr(te_cfg, "vocab_size", 8192))
    from PIL import Image
    decoder = None
    if a.vae:
        from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentDecoder
        decoder = LatentDecoder(a.vae, device)
    for prefix, prompts in sets:
        ids = tokenize(prompts, te_cfg.max_tokens, tok, lm=lm).to(device)
        with torch.no_grad():
            if lm:
                z = sample(te, den, a.steps, a.cfg, a.seed, a.t_shift, batch=a.batch, lm_states=frozen.states(ids),
                           valid=ids.ne(LM_PAD))
            else:
                z = sample(te, den, a.steps, a.cfg, a.seed, a.t_shift, batch=a.batch, ids=ids)
        torch.save(dict(latents=z.cpu(), prompts=prompts, steps=a.steps, cfg=a.cfg, seed=a.seed),
                   os.path.join(a.out_dir, f"{prefix}latents.pt"))
        imgs, kind = (decoder.decode(z), "") if decoder is not None else (latent_preview(z), "_latent_preview")
        for i, im in enumerate(imgs):
            Image.fromarray(im).save(os.path.join(a.out_dir, f"{prefix}{i:02d}{kind}.png"))
        if prefix and len(imgs) == 8:  # the 4 x 2 grid of a showcase set
            h, w = imgs[0].shape[:2]
            grid = Image.new("RGB", (4 * w, 2 * h))
            for i, im in enumerate(imgs):
                grid.paste(Image.fromarray(im), ((i % 4) * w, (i // 4) * h))
            grid.save(os.path.join(a.out_dir, f"grid_{prefix[:-1]}{kind}.png"))
        print(f"saved {len(imgs)} images{' and a grid' if prefix and len(imgs) == 8 else ''} to {a.out_dir} "
              f"({prefix[:-1] or 'your prompts'})", flush=True)
    if a.export:
        export_weights(te, den, a.out_dir, dict(steps=a.steps, cfg=a.cfg, seed=a.seed, step=info["step"],
                                                weights=info["weights"]))


def export_weights(te, den, out_dir, meta=None):
    from safetensors.torch import save_file
    for sub, mod in (("text_encoder", te), ("transformer", den)):
        os.makedirs(os.path.join(out_dir, sub), exist_ok=True)
        sd = {k: v.detach().cpu().contiguous() for k, v in mod.state_dict().items()}
        save_file(sd, os.path.join(out_dir, sub, "diffusion_pytorch_model.safetensors"))
        with open(os.path.join(out_dir, sub, "config.json"), "w") as f:
            json.dump(asdict(mod.config), f, indent=1)
    if meta:
        with open(os.path.join(out_dir, "prompts.json"), "w") as f:
            json.dump(meta, f, indent=1)
    print(f"exported weights to {out_dir}/text_encoder, {out_dir}/transformer")


if __name__ == "__main__":
    main()
