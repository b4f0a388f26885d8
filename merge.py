"""WSM / QAM checkpoint merging: sweep (method, scheme, window) over the raw-weight checkpoints train.py writes to
<run>/merge/step_*.pt, score each merge on the held-out set, write the best as <run>/merged.pt (training-checkpoint
layout; "ema" also holds the merged weights so samplers / exporters pick them by default).

  python merge.py runs/p10
  python merge.py runs/p10 --schemes 1-sqrt --windows 0.2 --methods wsm
"""
import argparse
import glob
import os

import torch

from trenowanie_generatora_obrazkow_b200.data.shards import full_shard_list, load_val, split_shards
from trenowanie_generatora_obrazkow_b200.models import build_models, configs_from_ckpt
from trenowanie_generatora_obrazkow_b200.optim.merge import merge_coefficients
from trenowanie_generatora_obrazkow_b200.train.evaluate import evaluate


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("run")
    p.add_argument("--schemes", default="1-sqrt,mean,cosine")
    p.add_argument("--methods", default="wsm,qam")
    p.add_argument("--windows", default="0.04,0.08,0.12,0.2")
    p.add_argument("--data", default="data/aurora")
    p.add_argument("--synthetic-val", type=int, default=0, help="score on N synthetic samples (no data dir)")
    p.add_argument("--val-samples", type=int, default=4096)
    p.add_argument("--out", default=None)
    args = p.parse_args()
    files = sorted(glob.glob(os.path.join(args.run, "merge", "step_*.pt")))
    assert files, f"no merge checkpoints in {args.run}/merge"
    meta = [torch.load(f, map_location="cpu", weights_only=False, mmap=True) for f in files]
    steps = [m["step"] for m in meta]
    total, last = meta[-1]["total_steps"], steps[-1]
    print(f"{len(files)} merge checkpoints, steps {steps[0]}..{last} (run of {total} steps)")
    combos = []
    for window in (float(x) for x in args.windows.split(",")):
        idx = [i for i, s in enumerate(steps) if s >= last - window * total]
        for scheme in args.schemes.split(","):
            for method in args.methods.split(","):
                combos.append(dict(method=method, scheme=scheme, window=window, idx=idx,
                                   c=merge_coefficients(scheme, len(idx), method)))
    keys = [("te", k) for k in meta[0]["te"]] + [("den", k) for k in meta[0]["den"]]
    used = sorted({i for cb in combos for i in cb["idx"]})
    cks = {i: [meta[i][part][k].float().clone() for part, k in keys] for i in used}
    buf = [torch.empty_like(t) for t in cks[used[0]]]

    def build(cb):
        torch._foreach_zero_(buf)
        for cj, i in zip(cb["c"], cb["idx"]):
            torch._foreach_add_(buf, cks[i], alpha=cj)
        return ({k: t for (part, k), t in zip(keys, buf) if part == "te"},
                {k: t for (part, k), t in zip(keys, buf) if part == "den"})

    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    den_cfg, te_cfg = configs_from_ckpt(meta[0])
    te, den = build_models(den_cfg, te_cfg, device=dev)
    if args.synthetic_val:
        g = torch.Generator().manual_seed(0)
        lat = torch.randn(args.synthetic_val, den_cfg.latent_channels, den_cfg.latent_size, den_cfg.latent_size,
                          generator=g)
        ids = torch.randint(6, 8000, (args.synthetic_val, te_cfg.max_tokens), generator=g)
        val = (lat, ids)
    else:
        val = load_val(args.data, split_shards(full_shard_list(args.data))[1], args.val_samples,
                       getattr(te_cfg, "tok_suffix", ""), te.null_ids())

    def score(te_sd, den_sd):
        te.load_state_dict(te_sd), den.load_state_dict(den_sd)
        return evaluate(te, den, val, dev)["val/loss"]

    print(f"{'raw weights @ last step':34s} val/loss {score(dict(meta[-1]['te']), dict(meta[-1]['den'])):.5f}")
    best = None
    for cb in combos:
        te_sd, den_sd = build(cb)
        loss = score(te_sd, den_sd)
        if best is None or loss < best[0]:
            best = (loss, cb, {k: v.clone() for k, v in te_sd.items()}, {k: v.clone() for k, v in den_sd.items()})
        print(f"{cb['method'].upper()} {cb['scheme']:7s} window {cb['window']:.0%} ({len(cb['idx'])} ckpt)"
              f"{'':4s} val/loss {loss:.5f}")
    loss, cb, te_sd, den_sd = best
    out = args.out or os.path.join(args.run, "merged.pt")
    torch.save(dict(step=last, den_config=meta[0]["den_config"], te_config=meta[0].get("te_config", {}), te=te_sd,
                    den=den_sd, ema=list(te_sd.values()) + list(den_sd.values()),
                    wsm=dict(method=cb["method"], scheme=cb["scheme"], window=cb["window"],
                             steps=[steps[i] for i in cb["idx"]], weights=cb["c"], val_loss=loss)), out)
    print(f"best: {cb['method'].upper()} {cb['scheme']} window {cb['window']:.0%} val/loss {loss:.5f} -> {out}")


if __name__ == "__main__":
    main()
