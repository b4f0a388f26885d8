"""Fixed evaluation suites over export directories (reference tests/homeimg22.py, face_sweep.py, decoder_grid.py).

  suite     a fixed prompt list x seeds at fixed settings, one image per (prompt, seed), each generated alone with
            its own seed, split into --parts for several processes, with a manifest per part; --resume finishes an
            identical manifest, --dry-run prints it. A directory never mixes models or settings.
  faces     several models side by side: rows = models, columns = prompts, one grid per seed; every model gets the
            same prompts and the same noise (each model loads, samples and is released in turn).
  decoders  the same latents decoded by two VAE directories (top row the export's own, bottom row another one).

  python eval_suite.py suite exports/x --prompts prompts_pl.json --settings settings.json --out-dir suite/x
  python eval_suite.py faces exports/a:3 exports/b:1 --prompts faces.json --seeds 0 1 --out-dir faces
  python eval_suite.py decoders exports/x --full-vae /models/flux2-vae --prompts p.json --out-dir dec

prompts.json: a JSON list of strings (or of {"prompt": ...}). settings.json: {"resolution", "guidance_scale",
"time_shift", "num_inference_steps", "seeds"} (the reference's settings file has this shape). Images are decoded by
the export's VAE when it carries one and diffusers is importable; otherwise each PNG is a false-colour preview of
the latents (the manifest records which) and the latents are saved beside it.
"""
import argparse
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
SETTING_KEYS = ("resolution", "guidance_scale", "time_shift", "num_inference_steps")


def load_prompts(path):
    items = json.load(open(path, encoding="utf-8"))
    return [p["prompt"] if isinstance(p, dict) else p for p in items]


def open_pipeline(root, device):
    sys.path.insert(0, ROOT)
    from homeimg_loader import load_homeimg_pipeline
    return load_homeimg_pipeline(root, device=device)


def render(pipe, prompts, seed, settings, latents_only=False):
    """(images (B, H, W, 3) uint8, latents, decoded?) for one batch with one seed."""
    import sample_ckpt as S
    out = pipe(prompts, height=settings["resolution"], num_inference_steps=settings["num_inference_steps"],
               guidance_scale=settings["guidance_scale"], shift=settings.get("time_shift"), seed=seed,
               output_type="latent" if latents_only else "np")
    if out.images is not None:
        return np.asarray(out.images), out.latents, True
    return S.latent_preview(out.latents), out.latents, False


def grid(cells, cols, cell=None, label_w=0, labels=None):
    """Row-major cells (H, W, 3) -> one image; optional per-row text labels in a left column."""
    from PIL import Image, ImageDraw
    imgs = [Image.fromarray(c) for c in cells]
    w, h = cell or imgs[0].size
    rows = -(-len(imgs) // cols)
    out = Image.new("RGB", (label_w + cols * w, rows * h), "white")
    for i, im in enumerate(imgs):
        r, c = divmod(i, cols)
        out.paste(im.resize((w, h)), (label_w + c * w, r * h))
    if labels:
        draw = ImageDraw.Draw(out)
        for r, text in enumerate(labels):
            draw.multiline_text((8, r * h + h // 2 - 10), text, fill="black")
    return out


# ---------------------------------------------------------------------------------------------------------- suite
def suite_jobs(prompts, seeds):
    return [dict(prompt_id=i + 1, prompt=p, seed=s, file=f"prompt_{i + 1:02d}_seed_{s}.png")
            for i, p in enumerate(prompts) for s in seeds]


def suite_manifest(model, settings, seeds, part, parts, jobs):
    return dict(model=model, settings=settings, seeds=seeds, part=part, parts=parts, images=jobs[part::parts])


def check_existing(out_dir, manifest, resume):
    """The jobs still to run; raises ValueError when the directory holds another model / settings / split, or (no
    --resume) anything of this part already."""
    path = os.path.join(out_dir, f"manifest_part_{manifest['part']:03d}.json")
    mine = manifest["images"]
    if not resume:
        if os.path.exists(path) or any(os.path.exists(os.path.join(out_dir, j["file"])) for j in mine):
            raise ValueError("output already exists; choose a new output directory (or --resume)")
    else:
        if not os.path.exists(path) or json.load(open(path, encoding="utf-8")) != manifest:
            raise ValueError("--resume needs the identical manifest of an earlier run in this directory")
    for name in sorted(os.listdir(out_dir)) if os.path.isdir(out_dir) else []:
        if name.startswith("manifest_part_") and name.endswith(".json"):
            other = json.load(open(os.path.join(out_dir, name), encoding="utf-8"))
            for key in ("model", "settings", "seeds", "parts"):
                if other[key] != manifest[key]:
                    raise ValueError(f"output directory holds a run with a different {key}")
    if not resume:
        return list(mine)
    from PIL import Image
    side = manifest["settings"]["resolution"]
    pending = []
    for j in mine:
        f = os.path.join(out_dir, j["file"])
        if not os.path.exists(f):
            pending.append(j)
            continue
        try:
            with Image.open(f) as im:
                if im.size != (side, side):
                    raise ValueError("wrong image size")
                im.verify()
        except (OSError, ValueError) as e:
            raise ValueError(f"invalid existing image {f}: {e}")
    return pending


def run_suite(a):
    prompts = load_prompts(a.prompts)
    settings = json.load(open(a.settings, encoding="utf-8"))
    seeds = settings.pop("seeds", [0])
    settings = {k: settings[k] for k in SETTING_KEYS}
    if a.parts < 1 or not 0 <= a.part < a.parts:
        raise ValueError("need --parts >= 1 and 0 <= --part < --parts")
    manifest = suite_manifest(a.model, settings, seeds, a.part, a.parts, suite_jobs(prompts, seeds))
    if a.dry_run:
        print(json.dumps(manifest, ensure_ascii=False, indent=2))
        return manifest
    os.makedirs(a.out_dir, exist_ok=True)
    todo = check_existing(a.out_dir, manifest, a.resume)
    if not a.resume:
        with open(os.path.join(a.out_dir, f"manifest_part_{a.part:03d}.json"), "x", encoding="utf-8") as f:
            json.dump(manifest, f, ensure_ascii=False, indent=2)
    if not todo:
        print("all images already exist")
        return manifest
    import torch
    from PIL import Image
    pipe = open_pipeline(a.model, a.device)
    for n, job in enumerate(todo, 1):
        imgs, z, decoded = render(pipe, [job["prompt"]], job["seed"], settings)
        img = imgs[0]
        if not decoded:  # a latent preview: scaled to the image size so the manifest's size check still applies
            img = np.asarray(Image.fromarray(img).resize((settings["resolution"],) * 2, Image.NEAREST))
            torch.save(z.cpu(), os.path.join(a.out_dir, job["file"][:-4] + ".latents.pt"))
        Image.fromarray(img).save(os.path.join(a.out_dir, job["file"]))
        print(f"{n}/{len(todo)} saved {job['file']}{'' if decoded else ' (latent preview)'}", flush=True)
    return manifest


# ---------------------------------------------------------------------------------------------------------- faces
def run_faces(a):
    """rows = models (spec "export_dir:cfg"), columns = prompts; one grid per seed, the same noise for every model."""
    import gc

    import torch
    prompts = load_prompts(a.prompts)
    os.makedirs(a.out_dir, exist_ok=True)
    rows = {}
    for spec in a.models:
        root, _, cfg = spec.rpartition(":")
        if not root:
            root, cfg = cfg, "3"
        pipe = open_pipeline(root, a.device)
        settings = dict(resolution=a.res, guidance_scale=float(cfg), time_shift=a.shift, num_inference_steps=a.steps)
        for seed in a.seeds:  # one batch per seed: the same noise rows for every model
            rows[seed, spec] = render(pipe, prompts, seed, settings)[0]
        print(f"done {spec}", flush=True)
        del pipe
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
    paths = []
    for seed in a.seeds:
        cells = [im for spec in a.models for im in rows[seed, spec]]
        labels = [spec.replace(":", "\ncfg ") for spec in a.models]
        g = grid(cells, len(prompts), cell=(a.cell, a.cell), label_w=220, labels=labels)
        path = os.path.join(a.out_dir, f"faces_seed{seed}.png")
        g.save(path)
        paths.append(path)
        print(f"saved {path}", flush=True)
    return paths


# ------------------------------------------------------------------------------------------------------- decoders
def run_decoders(a):
    """The same latents through the export's own VAE (top row) and another VAE directory (bottom row); both must
    share the latent normalisation. Saved 1:1 and 2x (nearest)."""
    from PIL import Image

    from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentDecoder
    prompts = load_prompts(a.prompts)
    os.makedirs(a.out_dir, exist_ok=True)
    pipe = open_pipeline(a.model, a.device)
    if pipe.vae_dir is None:
        raise ValueError("the export carries no VAE (vae/): nothing to compare against")
    settings = dict(resolution=a.res, guidance_scale=a.cfg, time_shift=a.shift, num_inference_steps=a.steps)
    _, z, _ = render(pipe, prompts, a.seed, settings, latents_only=True)
    rows = [LatentDecoder(d, pipe.device).decode(z) for d in (pipe.vae_dir, a.full_vae)]
    g = grid([np.asarray(im) for r in rows for im in r], len(prompts), cell=(a.cell, a.cell))
    path = os.path.join(a.out_dir, "decoders.png")
    g.save(path)
    g.resize((g.width * 2, g.height * 2), Image.NEAREST).save(os.path.join(a.out_dir, "decoders_2x.png"))
    print(f"saved {path}: top the export's decoder, bottom {a.full_vae}", flush=True)
    return path


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("suite")
    s.add_argument("model", help="export directory")
    s.add_argument("--prompts", required=True)
    s.add_argument("--settings", required=True)
    s.add_argument("--out-dir", required=True)
    s.add_argument("--part", type=int, default=0)
    s.add_argument("--parts", type=int, default=1)
    s.add_argument("--dry-run", action="store_true")
    s.add_argument("--resume", action="store_true")
    f = sub.add_parser("faces")
    f.add_argument("models", nargs="+", help="export_dir:cfg")
    f.add_argument("--prompts", required=True)
    f.add_argument("--seeds", type=int, nargs="+", default=[0, 1])
    d = sub.add_parser("decoders")
    d.add_argument("model")
    d.add_argument("--full-vae", required=True)
    d.add_argument("--prompts", required=True)
    d.add_argument("--seed", type=int, default=7)
    d.add_argument("--cfg", type=float, default=3.0)
    for q in (f, d):
        q.add_argument("--out-dir", required=True)
        q.add_argument("--res", type=int, default=1024)
        q.add_argument("--steps", type=int, default=50)
        q.add_argument("--shift", type=float, default=None, help="time shift (default: the export's)")
        q.add_argument("--cell", type=int, default=256, help="grid cell size in pixels")
    for q in (s, f, d):
        q.add_argument("--device", default=None)
    a = p.parse_args(argv)
    if a.device is None:
        import torch
        a.device = "cuda" if torch.cuda.is_available() else "cpu"
    try:
        return {"suite": run_suite, "faces": run_faces, "decoders": run_decoders}[a.cmd](a)
    except ValueError as e:
        p.error(str(e))


if __name__ == "__main__":
    main()
