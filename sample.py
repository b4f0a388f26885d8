"""An 8-image showcase grid (4 x 2) from an export directory (reference sample.py:1-60): every prompt is sampled
alone with the same seed, so each cell is what a user gets for that prompt at that seed.

  python sample.py exports/x-step1000 --out grid.png
  python sample.py exports/x-pl --lang pl --out grid_pl.png --cfg 1        # a guidance-distilled (OPD) student
  python sample.py exports/x --prompts my_prompts.json --res 512 --steps 30

The export is loaded through its own pipeline.py (homeimg_loader.py). Cells are images when the export carries a
VAE and diffusers is importable, else false-colour previews of the latents. --prompts replaces the built-in list
(a JSON list of strings or of {"prompt": ...}; the grid has 4 columns).
"""
import argparse
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))

# eight showcase prompts of this project's own choosing (photo, night scene, still life, painting, character,
# fantasy, lettering, people), in English and in Polish for bilingual text encoders
PROMPTS = [
    "a grey heron standing in shallow water at dawn, mist over the lake, photograph",
    "a narrow old-town street at night after rain, warm lamps reflected on cobblestones",
    "a glass jar of honey and a slice of bread on a linen cloth, morning light",
    "an oil painting of sailing boats in a harbour, thick brush strokes",
    "a knitted toy bear sitting on a windowsill next to a potted cactus",
    "a dragon made of autumn leaves flying over a mountain valley, digital art",
    "a wooden sign that says BAKERY above a shop door",
    "an old man playing chess in a park, shallow depth of field",
]
PROMPTS_PL = [
    "czapla siwa stojąca w płytkiej wodzie o świcie, mgła nad jeziorem, fotografia",
    "wąska uliczka starego miasta nocą po deszczu, ciepłe latarnie odbite w kocich łbach",
    "szklany słoik miodu i kromka chleba na lnianej ściereczce, poranne światło",
    "obraz olejny przedstawiający żaglówki w porcie, grube pociągnięcia pędzla",
    "miś zrobiony na drutach siedzący na parapecie obok kaktusa w doniczce",
    "smok z jesiennych liści lecący nad górską doliną, grafika cyfrowa",
    "drewniany szyld z napisem BAKERY nad drzwiami sklepu",
    "starszy mężczyzna grający w szachy w parku, mała głębia ostrości",
]


def sample_grid(pipe, prompts, seed=0, steps=50, cfg=3.0, res=1024, shift=None, cols=4):
    """(grid image, decoded?) with one pipeline call per prompt, each with ``seed``."""
    sys.path.insert(0, ROOT)
    import eval_suite
    settings = dict(resolution=res, guidance_scale=cfg, time_shift=shift, num_inference_steps=steps)
    cells, decoded = [], True
    for prompt in prompts:
        imgs, _, dec = eval_suite.render(pipe, [prompt], seed, settings)
        cells.append(np.asarray(imgs[0]))
        decoded &= dec
    side = cells[0].shape[0] if decoded else res
    return eval_suite.grid(cells, min(cols, len(cells)), cell=(side, side)), decoded


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("model", help="export directory")
    p.add_argument("--out", default="grid.png")
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--cfg", type=float, default=3.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--lang", choices=["en", "pl"], default="en")
    p.add_argument("--res", type=int, default=1024)
    p.add_argument("--shift", type=float, default=None, help="time shift (default: the export's)")
    p.add_argument("--prompts", default="", help="JSON prompt list replacing the built-in eight")
    p.add_argument("--device", default=None)
    a = p.parse_args(argv)
    import torch
    device = a.device or ("cuda" if torch.cuda.is_available() else "cpu")
    sys.path.insert(0, ROOT)
    from eval_suite import load_prompts, open_pipeline
    prompts = load_prompts(a.prompts) if a.prompts else (PROMPTS_PL if a.lang == "pl" else PROMPTS)
    pipe = open_pipeline(a.model, device)
    g, decoded = sample_grid(pipe, prompts, a.seed, a.steps, a.cfg, a.res, a.shift)
    os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
    g.save(a.out)
    print(f"saved {a.out}{'' if decoded else ' (latent previews: no VAE in the export)'}")
    return a.out


if __name__ == "__main__":
    main()
