"""An export directory (export.py / the released layout) -> a fresh checkpoint for ``train.py --init``.

  python import_homeimg.py exports/x runs/new/init.pt

The weights are validated against freshly built modules (strict load) and stored as both the live weights and the
EMA list, with no optimizer state (reference import_homeimg.py:18-67).
"""
import argparse

from trenowanie_generatora_obrazkow_b200.utils.export import export_to_init


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("src")
    p.add_argument("out")
    a = p.parse_args(argv)
    ck = export_to_init(a.src, a.out)
    n = sum(v.numel() for v in ck["den"].values()) + sum(v.numel() for v in ck["te"].values())
    print(f"wrote {a.out}: {n / 1e6:.1f}M parameters")


if __name__ == "__main__":
    main()
