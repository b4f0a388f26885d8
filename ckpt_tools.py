"""Checkpoint inspection helpers (reference tests/block_norms.py, tests/resume_cmd.py), reading train.py /
train_pp.py checkpoints lazily (memory-mapped).

  python ckpt_tools.py info runs/x/latest.pt
  python ckpt_tools.py block-norms runs/grow12/latest.pt --old 6
  python ckpt_tools.py resume-cmd runs/253m/latest.pt --out runs/gns_253m --extra-steps 200 -- --gns-every 32

info         step, samples, model configs, parameter counts, EMA / optimizer state present, pipeline layout.
block-norms  how far blocks grown by --init (zero-initialised output projections) have moved: per denoiser block the
             RMS of attn.out, cross.out and mlp.out_proj, raw and EMA weights, and each relative to the mean of the
             first --old blocks.
resume-cmd   a torchrun command that continues the checkpoint with its stored settings in another output directory
             (the original run stays untouched; copy latest.pt there first), e.g. to measure the gradient noise scale
             late in training. Flags after `--` are appended and replace the stored value of the same flag; the
             step count becomes step + --extra-steps with evaluation and checkpointing at that step only.
"""
import argparse
import os
import shlex
import sys

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
OUTS = ("attn.out.weight", "cross.out.weight", "mlp.out_proj.weight")
# settings of the original run that make no sense for a continuation (or are set by the command itself)
RESUME_SKIP = {"out", "steps", "eval_every", "ckpt_every", "merge_every", "keep_every", "log_every", "load_hf", "init",
               "help"}


def _load(path):
    return torch.load(path, map_location="cpu", weights_only=False, mmap=True)


def info(ck):
    den, te = ck.get("den") or {}, ck.get("te") or {}
    n = lambda sd: sum(v.numel() for v in sd.values())
    out = dict(step=ck.get("step"), samples=ck.get("samples"), den_params=n(den), te_params=n(te),
               ema=ck.get("ema") is not None and len(ck["ema"]) > 0, opts=ck.get("opts") is not None,
               den_config=ck.get("den_config"), te_config=ck.get("te_config"), pp_layout=ck.get("pp_layout"),
               outer=ck.get("outer") is not None, repa_proj=ck.get("repa_proj") is not None,
               extra=ck.get("extra") or {})  # e.g. the OPD caption-stream position
    return out


def block_norms(ck, old):
    """{"raw"|"EMA": [(block, {proj: (rms, rms / mean of the old blocks)})]}."""
    den = ck["den"]
    sources = {"raw": den}
    if ck.get("ema"):  # the flat EMA list: text-encoder parameters, then denoiser parameters
        sources["EMA"] = dict(zip(den.keys(), ck["ema"][len(ck["te"]):]))
    depth = 1 + max(int(k.split(".")[1]) for k in den if k.startswith("blocks."))
    if not 1 <= old <= depth:
        raise ValueError(f"--old {old}: the checkpoint has {depth} blocks")
    res = {}
    for name, sd in sources.items():
        rms = {(i, o): sd[f"blocks.{i}.{o}"].float().pow(2).mean().sqrt().item() for i in range(depth) for o in OUTS}
        base = {o: sum(rms[i, o] for i in range(old)) / old for o in OUTS}
        res[name] = [(i, {o: (rms[i, o], rms[i, o] / base[o] if base[o] else float("nan")) for o in OUTS})
                     for i in range(depth)]
    return res, depth


def resume_command(ck, out, extra_steps, extra=(), nproc=8):
    """The command line (a string) continuing ``ck`` in ``out``."""
    stored, step = ck.get("args") or {}, int(ck["step"])
    if not stored:
        raise ValueError("the checkpoint has no stored arguments")
    sys.path.insert(0, ROOT)
    pipeline = ck.get("pp_layout") is not None or "pp" in stored
    script = "train_pp.py" if pipeline else "train.py"
    if pipeline:
        import train_pp as mod
    else:
        import train as mod
    parser = mod.build_parser()
    override = {a.split("=", 1)[0][2:].replace("-", "_") for a in extra if a.startswith("--")}
    flags = []
    for action in parser._actions:
        k = action.dest
        if k in RESUME_SKIP or k in override or k not in stored or not action.option_strings:
            continue
        v, opt = stored[k], action.option_strings[-1]
        if v is None or v == action.default:
            continue
        if action.nargs == 0:  # store_true / store_false: the flag itself
            flags.append(opt)
        elif isinstance(v, (list, tuple)):
            flags += [opt] + [str(x) for x in v]
        else:
            flags += [opt, str(v)]
    end = step + extra_steps
    tail = ["--steps", str(end), "--eval-every", str(end), "--ckpt-every", str(end), "--merge-every", "0",
            "--keep-every", "0", "--out", out]
    cmd = (["torchrun", "--nproc-per-node", str(nproc), "--master-addr", "127.0.0.1", script] + flags + tail
           + list(extra))
    return " ".join(shlex.quote(c) for c in cmd), step, stored


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("info")
    s.add_argument("ckpt")
    s = sub.add_parser("block-norms")
    s.add_argument("ckpt")
    s.add_argument("--old", type=int, default=6, help="blocks that came from the --init checkpoint")
    s = sub.add_parser("resume-cmd")
    s.add_argument("ckpt")
    s.add_argument("--out", required=True)
    s.add_argument("--extra-steps", type=int, default=200)
    s.add_argument("--nproc", type=int, default=8)
    argv = list(sys.argv[1:] if argv is None else argv)
    extra = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    a = p.parse_args(argv)
    ck = _load(a.ckpt)
    if a.cmd == "info":
        res = info(ck)
        for k, v in res.items():
            print(f"{k:12s} {v}")
        return res
    if a.cmd == "block-norms":
        res, depth = block_norms(ck, a.old)
        print(f"{a.ckpt}: step {ck.get('step')}, {depth} blocks (0-{a.old - 1} old, {a.old}-{depth - 1} grown)")
        for name, rows in res.items():
            print(f"\n{name} weights: RMS of the output projections (x 1e-3), relative to the old blocks' mean")
            print("block      " + "  ".join(f"{o[:-len('.weight')]:>22s}" for o in OUTS))
            for i, cells in rows:
                tag = "old" if i < a.old else "new"
                print(f"{i:3d} {tag}    " + "  ".join(f"{cells[o][0] * 1e3:10.3f} ({cells[o][1]:7.1%})" for o in OUTS))
        return res
    cmd, step, stored = resume_command(ck, a.out, a.extra_steps, extra, a.nproc)
    print(f"# checkpoint at step {step} (of {stored.get('steps')}), batch {stored.get('batch')}, size "
          f"{stored.get('size')}, text encoder {stored.get('te_size')}")
    print(f"# mkdir -p {shlex.quote(a.out)} && cp {shlex.quote(a.ckpt)} {shlex.quote(os.path.join(a.out, 'latest.pt'))}")
    print(cmd)
    return cmd


if __name__ == "__main__":
    main()
