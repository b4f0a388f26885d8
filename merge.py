"""WSM / QAM checkpoint merging (reference tool: merge.py): choose, on the held-out set, which decay-emulating average
of the raw-weight checkpoints that train.py writes to <run>/merge/step_*.pt gives the best model, and write it as
<run>/merged.pt in the training-checkpoint layout ("ema" holds the merged weights too, so samplers and exporters use
them by default).

  python merge.py runs/p10
  python merge.py runs/p10 --schemes 1-sqrt --windows 0.2 --methods wsm

How it works here: every candidate (method x decay scheme x window) is a row of a coefficient table over the
checkpoints (zero outside its window; weights from optim/merge.py). A candidate is built directly in the parameters
of the one model used for scoring, on the scoring device, by streaming the checkpoints it uses one at a time from
their memory maps (fp32 accumulation; each checkpoint is read, cast and added, then dropped). Host memory therefore
holds no fp32 copy of any checkpoint and device memory holds one model, whatever the number of checkpoints.
"""
import argparse
import glob
import os
from dataclasses import dataclass, field

import torch

from trenowanie_generatora_obrazkow_b200.data.shards import full_shard_list, load_val, split_shards
from trenowanie_generatora_obrazkow_b200.models import build_models, configs_from_ckpt
from trenowanie_generatora_obrazkow_b200.optim.merge import merge_coefficients
from trenowanie_generatora_obrazkow_b200.train.evaluate import evaluate

PARTS = ("te", "den")


@dataclass
class Candidate:
    method: str
    scheme: str
    window: float
    weights: dict = field(default_factory=dict)  # checkpoint position -> coefficient
    loss: float = float("inf")

    def label(self):
        return f"{self.method.upper()} {self.scheme:7s} window {self.window:.0%} ({len(self.weights)} ckpt)"


def candidate_table(steps, total, windows, schemes, methods):
    """One Candidate per (window, scheme, method); a window of fraction f holds the checkpoints of the last f of the
    run (counted back from the newest checkpoint)."""
    last = steps[-1]
    table = []
    for window in windows:
        members = [i for i, s in enumerate(steps) if s >= last - window * total]
        for scheme in schemes:
            for method in methods:
                coef = merge_coefficients(scheme, len(members), method)
                table.append(Candidate(method, scheme, window, dict(zip(members, coef))))
    return table


class CheckpointStream:
    """The merge checkpoints of a run, opened as memory maps on demand."""

    def __init__(self, files):
        self.files = list(files)
        self.head = torch.load(self.files[-1], map_location="cpu", weights_only=False, mmap=True)
        self.steps = [self._open(i)["step"] for i in range(len(self.files) - 1)] + [self.head["step"]]

    def _open(self, i):
        if i == len(self.files) - 1:
            return self.head
        return torch.load(self.files[i], map_location="cpu", weights_only=False, mmap=True)

    def state(self, i):
        ck = self._open(i)
        return {part: ck[part] for part in PARTS}


def assemble(targets, stream, weights):
    """targets: {part: {name: tensor}} views of the scoring model's floating state; overwritten with
    sum_i weights[i] * checkpoint_i. fp32 targets accumulate in place; others through an fp32 temporary."""
    acc = {part: {k: (t if t.dtype == torch.float32 else torch.empty(t.shape, dtype=torch.float32, device=t.device))
                  for k, t in sd.items()} for part, sd in targets.items()}
    with torch.no_grad():
        for sd in acc.values():
            torch._foreach_zero_(list(sd.values()))
        for i, c in sorted(weights.items()):
            src = stream.state(i)
            for part, sd in acc.items():
                for k, a in sd.items():
                    a.add_(src[part][k].to(a.device, torch.float32, non_blocking=True), alpha=float(c))
            del src
        for part, sd in targets.items():
            for k, t in sd.items():
                if acc[part][k] is not t:
                    t.copy_(acc[part][k])


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("run", help="training output directory (holds merge/ and latest.pt)")
    p.add_argument("--schemes", default="1-sqrt,mean,cosine")
    p.add_argument("--methods", default="wsm,qam", help="wsm (first order) and / or qam (second order)")
    p.add_argument("--windows", default="0.04,0.08,0.12,0.2",
                   help="merge windows as fractions of the whole run, counted back from the last checkpoint")
    p.add_argument("--data", default="data/aurora")
    p.add_argument("--synthetic-val", type=int, default=0, help="score on N synthetic samples (no data dir)")
    p.add_argument("--val-samples", type=int, default=4096)
    p.add_argument("--out", default=None, help="default: <run>/merged.pt")
    args = p.parse_args(argv)

    files = sorted(glob.glob(os.path.join(args.run, "merge", "step_*.pt")))
    if not files:
        raise SystemExit(f"no merge checkpoints in {args.run}/merge (train with --merge-every > 0)")
    stream = CheckpointStream(files)
    head = stream.head
    print(f"{len(files)} merge checkpoints, steps {stream.steps[0]}..{stream.steps[-1]} "
          f"(run of {head['total_steps']} steps)")
    table = candidate_table(stream.steps, head["total_steps"], [float(w) for w in args.windows.split(",")],
                            args.schemes.split(","), args.methods.split(","))

    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    den_cfg, te_cfg = configs_from_ckpt(head)
    te, den = build_models(den_cfg, te_cfg, device=dev)
    modules = {"te": te, "den": den}
    targets = {part: {k: t for k, t in m.state_dict().items() if t.is_floating_point()}
               for part, m in modules.items()}
    if args.synthetic_val:
        g = torch.Generator().manual_seed(0)
        val = (torch.randn(args.synthetic_val, den_cfg.latent_channels, den_cfg.latent_size, den_cfg.latent_size,
                           generator=g),
               torch.randint(6, 8000, (args.synthetic_val, te_cfg.max_tokens), generator=g))
    else:
        val = load_val(args.data, split_shards(full_shard_list(args.data))[1], args.val_samples,
                       getattr(te_cfg, "tok_suffix", ""), te.null_ids())

    def score(weights):
        assemble(targets, stream, weights)
        return evaluate(te, den, val, dev)["val/loss"]

    print(f"{'raw weights @ last step':34s} val/loss {score({len(files) - 1: 1.0}):.5f}")
    latest = os.path.join(args.run, "latest.pt")
    if os.path.exists(latest):  # the EMA of the training checkpoint, for comparison
        ck = torch.load(latest, map_location="cpu", weights_only=False, mmap=True)
        ema = iter(ck["ema"])  # one tensor per parameter: the text encoder's, then the denoiser's
        with torch.no_grad():
            for part in PARTS:
                for t in modules[part].parameters():
                    t.copy_(next(ema).to(t.device, t.dtype))
        print(f"{'EMA @ step ' + str(ck['step']):34s} val/loss {evaluate(te, den, val, dev)['val/loss']:.5f}")
    for cand in table:
        cand.loss = score(cand.weights)
        print(f"{cand.label():34s} val/loss {cand.loss:.5f}")
    best = min(table, key=lambda c: c.loss)

    assemble(targets, stream, best.weights)  # rebuild the winner and save it in the checkpoint layout
    sds = {part: {k: v.detach().to("cpu").clone() for k, v in modules[part].state_dict().items()} for part in PARTS}
    order = sorted(best.weights)
    out = args.out or os.path.join(args.run, "merged.pt")
    torch.save({"step": stream.steps[-1], "den_config": head["den_config"], "te_config": head.get("te_config", {}),
                "te": sds["te"], "den": sds["den"], "ema": list(sds["te"].values()) + list(sds["den"].values()),
                "wsm": {"method": best.method, "scheme": best.scheme, "window": best.window,
                        "steps": [stream.steps[i] for i in order], "weights": [best.weights[i] for i in order],
                        "val_loss": best.loss}}, out)
    print(f"best: {best.method.upper()} {best.scheme} window {best.window:.0%} val/loss {best.loss:.5f} -> {out}")


if __name__ == "__main__":
    main()
