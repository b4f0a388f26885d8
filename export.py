"""Export a training checkpoint (EMA weights by default) into a self-contained diffusers-layout directory.

  python export.py runs/x/latest.pt exports/x-step1000
  python export.py runs/x/latest.pt exports/raw --no-ema --time-shift 6 --vae-dir /models/flux2-vae

Same command line as the reference's export.py (export.py:104-115): --no-ema, --time-shift, --time-shift-ref, --ref.
--ref is a local export directory (a released model, or an earlier export) whose vae/ and tokenizer/tokenizer.json
are copied when --vae-dir / --tokenizer-json are not given; the explicit paths win.

  python export.py runs/x/latest.pt exports/x-step2000 --ref exports/x-step1000
"""
import argparse
import os

from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt
from trenowanie_generatora_obrazkow_b200.utils.export import export_checkpoint


def ref_assets(ref, vae_dir=None, tokenizer_json=None):
    """(vae directory, tokenizer.json) to copy: the explicit paths, else the ones a --ref export carries."""
    if ref is None:
        return vae_dir, tokenizer_json
    if not os.path.isdir(ref):
        raise SystemExit(f"--ref {ref}: not a directory")
    if vae_dir is None and os.path.isdir(os.path.join(ref, "vae")):
        vae_dir = os.path.join(ref, "vae")
    tj = os.path.join(ref, "tokenizer", "tokenizer.json")
    if tokenizer_json is None and os.path.exists(tj):
        tokenizer_json = tj
    return vae_dir, tokenizer_json


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("ckpt")
    p.add_argument("out")
    p.add_argument("--no-ema", action="store_true")
    p.add_argument("--time-shift", type=float, default=None)
    p.add_argument("--time-shift-ref", type=float, default=None)
    p.add_argument("--vae-dir", default=None, help="local diffusers AutoencoderKLFlux2 directory to copy into vae/")
    p.add_argument("--tokenizer-json", default=None)
    p.add_argument("--ref", default=None, help="local export directory to take vae/ and tokenizer/ from")
    p.add_argument("--lm-dir", default=None, help="local Slayer LM directory (config.json + model.safetensors): "
                   "its blocks the refiner reads are packed into text_encoder/, with its tokenizer.json")
    a = p.parse_args(argv)
    vae_dir, tok = ref_assets(a.ref, a.vae_dir, a.tokenizer_json)
    ck = ckpt.load(a.ckpt)
    index = export_checkpoint(ck, a.out, use_ema=not a.no_ema, time_shift=a.time_shift,
                              time_shift_ref=a.time_shift_ref, vae_dir=vae_dir, tokenizer_json=tok,
                              lm_dir=a.lm_dir)
    print(f"exported step {index['step']} ({index['weights']} weights) to {a.out}")


if __name__ == "__main__":
    main()
