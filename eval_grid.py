"""Evaluation grids of a checkpoint (reference tests/homeimg22.py, homeimg22_grid.py, flux36_grid.py,
guidance_grid.py): a prompt list x seeds x guidance methods, sampled with the Euler flow-matching sampler at the
given resolution; per cell the latents are saved, and a grid PNG is assembled (rows = method x seed, columns =
prompts). With --vae (a local FLUX.2 VAE directory; diffusers needed) the cells are decoded images, otherwise
false-colour latent previews.

  python eval_grid.py runs/x/latest.pt --prompts prompts.json --seeds 0 1 2 3 --res 1024 --out-dir grids/x \\
      --methods cfg:3 "cfg:3|shift=6" cfgzero:3 ag:runs/small/latest.pt:2

prompts.json: a JSON list of strings, or of {"prompt": ...} objects.
"""
import argparse
import json
import os

import numpy as np
import torch


def load_prompts(path):
    items = json.load(open(path))
    return [p["prompt"] if isinstance(p, dict) else p for p in items]


def grid_image(cells, cols):
    """cells: list of (H, W, 3) uint8 in row-major order -> one (rows H, cols W, 3) array."""
    h, w = cells[0].shape[:2]
    rows = -(-len(cells) // cols)
    out = np.zeros((rows * h, cols * w, 3), dtype=np.uint8)
    for i, c in enumerate(cells):
        r, k = divmod(i, cols)
        out[r * h:(r + 1) * h, k * w:(k + 1) * w] = c
    return out


def main(argv=None):
    import sample_ckpt as S
    from trenowanie_generatora_obrazkow_b200.models import LMEncoderConfig
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD, build_frozen_lm
    from trenowanie_generatora_obrazkow_b200.sampling.euler import encode_prompts, prompt_noise
    from trenowanie_generatora_obrazkow_b200.sampling.guidance import guided_latents, parse_method
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("ckpt")
    p.add_argument("--prompts", required=True)
    p.add_argument("--seeds", type=int, nargs="+", default=[0])
    p.add_argument("--methods", nargs="+", default=["cfg:3"])
    p.add_argument("--res", type=int, default=None)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--random-lm", action="store_true")
    p.add_argument("--vae", default=None)
    p.add_argument("--out-dir", required=True)
    a = p.parse_args(argv)
    device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    os.makedirs(a.out_dir, exist_ok=True)
    prompts = load_prompts(a.prompts)
    models = {}

    def model(path):
        if path not in models:
            te, den, _ = S.load(path, res=a.res)
            te.to(device).eval(), den.to(device).eval()
            lm = isinstance(te.config, LMEncoderConfig)
            ids = S.tokenize(prompts, te.config.max_tokens,
                             S.load_tokenizer(a.tokenizer, getattr(te.config, "vocab_size", 8192)), lm=lm).to(device)
            with torch.no_grad():
                if lm:
                    states = build_frozen_lm(te.config, device, allow_random=a.random_lm).states(ids)
                    enc = encode_prompts(te, lm_states=states, valid=ids.ne(LM_PAD))
                else:
                    enc = encode_prompts(te, ids=ids)
            models[path] = (den, enc)
        return models[path]

    den, (text, lens, null, nlen) = model(a.ckpt)
    c = den.config
    decoder = None
    if a.vae:
        from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentDecoder
        decoder = LatentDecoder(a.vae, device)
    cells, record = [], []
    for spec in a.methods:
        m = parse_method(spec)
        guide = None
        if m["method"] == "ag":
            bden, (btext, blens, _, _) = model(m["guide"])
            guide = (bden, btext, blens)
        for seed in a.seeds:
            noise = prompt_noise(len(prompts), c.latent_channels, c.latent_size, seed, 0, device)
            z = guided_latents(den, text, lens, null, nlen, noise, a.steps, m["w"], m["method"], m["shift"],
                               m["off"], guide)
            imgs = decoder.decode(z) if decoder is not None else S.latent_preview(z)
            cells += list(imgs)
            record.append(dict(method=spec, seed=seed, latents=z.cpu()))
    torch.save(dict(prompts=prompts, cells=record, steps=a.steps), os.path.join(a.out_dir, "latents.pt"))
    from PIL import Image
    kind = "" if decoder is not None else "_latent_preview"
    path = os.path.join(a.out_dir, f"grid{kind}.png")
    Image.fromarray(grid_image(cells, len(prompts))).save(path)
    print(f"{len(a.methods)} methods x {len(a.seeds)} seeds x {len(prompts)} prompts -> {path}")
    return record


if __name__ == "__main__":
    main()
