"""Export a training checkpoint (EMA weights by default) into a self-contained diffusers-layout directory.

  python export.py runs/x/latest.pt exports/x-step1000
  python export.py runs/x/latest.pt exports/raw --no-ema --time-shift 6 --vae-dir /models/flux2-vae

Same command line as the reference's export.py (export.py:104-115): --no-ema, --time-shift, --time-shift-ref; the
VAE and tokenizer are copied from local paths (--vae-dir, --tokenizer-json) instead of a reference repository.
"""
import argparse

from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt
from trenowanie_generatora_obrazkow_b200.utils.export import export_checkpoint


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("ckpt")
    p.add_argument("out")
    p.add_argument("--no-ema", action="store_true")
    p.add_argument("--time-shift", type=float, default=None)
    p.add_argument("--time-shift-ref", type=float, default=None)
    p.add_argument("--vae-dir", default=None, help="local diffusers AutoencoderKLFlux2 directory to copy into vae/")
    p.add_argument("--tokenizer-json", default=None)
    p.add_argument("--lm-dir", default=None, help="local Slayer LM directory (config.json + model.safetensors): "
                   "its blocks the refiner reads are packed into text_encoder/, with its tokenizer.json")
    a = p.parse_args(argv)
    ck = ckpt.load(a.ckpt)
    index = export_checkpoint(ck, a.out, use_ema=not a.no_ema, time_shift=a.time_shift,
                              time_shift_ref=a.time_shift_ref, vae_dir=a.vae_dir, tokenizer_json=a.tokenizer_json,
                              lm_dir=a.lm_dir)
    print(f"exported step {index['step']} ({index['weights']} weights) to {a.out}")


if __name__ == "__main__":
    main()
