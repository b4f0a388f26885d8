"""Component costs inside training (reference tests/bench_ckpt.py, tests/bench_te.py).

  python -m trenowanie_generatora_obrazkow_b200.ops.component_bench ckpt --size 2b --blocks 4 --mb 16 --inflight 8
  python -m trenowanie_generatora_obrazkow_b200.ops.component_bench te --layers 4 8 12 --batch 32 --tokens 96

ckpt  speed and peak memory of activation checkpointing (none / full / selective) for one pipeline stage's worth of
      denoiser blocks in a 1F1B-like pattern: ``inflight`` micro-batches are run forward and kept, then run backward
      in order (the activations a stage holds at once). Reported per mode: device ms per micro-batch forward +
      backward and the peak memory above the weights.
te    cost of the frozen LM text encoder inside training: forward time of one micro-batch of captions (random
      lengths, packed without padding on CUDA) and resident weight memory, per number of kept layers of a
      Slayer-shaped GPT (random init: the weights do not change the cost).

Device times use CUDA events after warm-up with a synchronize on both sides; on a CPU the numbers are wall clock (a
harness check, not a measurement). Prints one JSON line per configuration.
"""
import argparse
import json
import time
from dataclasses import replace

import torch


def _timer(device):
    cuda = torch.device(device).type == "cuda"

    def run(fn, iters, warmup):
        for _ in range(warmup):
            fn()
        if cuda:
            torch.cuda.synchronize(device)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(iters):
                fn()
            b.record()
            torch.cuda.synchronize(device)
            return a.elapsed_time(b) / iters
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        return (time.perf_counter() - t0) * 1e3 / iters
    return run


def _peak_mb(device, fn):
    if torch.device(device).type != "cuda":
        fn()
        return None
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    base = torch.cuda.memory_allocated(device)
    fn()
    torch.cuda.synchronize(device)
    return (torch.cuda.max_memory_allocated(device) - base) / 2 ** 20


def ckpt_bench(size="2b", blocks=4, mb=16, inflight=8, res=256, text_len=96, modes=("none", "full", "selective"),
               iters=3, warmup=1, device=None, log=print):
    """[{mode, ms_per_microbatch, peak_mb}] for ``blocks`` denoiser blocks of preset ``size``."""
    from ..models.config import SIZES
    from ..models.dit import Denoiser
    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    cfg = replace(SIZES[size], depth=blocks, latent_size=res // 16)
    torch.manual_seed(0)
    den = Denoiser(cfg).to(device)
    side = res // 16
    g = torch.Generator(device="cpu").manual_seed(1)
    mk = lambda *s: torch.randn(*s, generator=g).to(device)
    z = mk(mb, cfg.latent_channels, side, side)
    t = torch.rand(mb, generator=g).to(device)
    text = mk(mb, text_len, cfg.text_dim)
    valid = torch.ones(mb, text_len, dtype=torch.bool, device=device)
    valid[:, text_len // 2:] = False
    run = _timer(device)
    rows = []
    for mode in modes:
        den.checkpoint_blocks = False if mode == "none" else mode

        def pattern():
            outs = [den(z, t, text, valid).float().square().mean() for _ in range(inflight)]
            for o in outs:
                o.backward()
            den.zero_grad(set_to_none=True)

        peak = _peak_mb(device, pattern)
        ms = run(pattern, iters, warmup) / inflight
        row = dict(bench="ckpt", mode=mode, size=size, blocks=blocks, mb=mb, inflight=inflight, res=res,
                   ms_per_microbatch=ms, peak_mb=peak, device=str(device))
        rows.append(row)
        log(json.dumps(row))
    den.checkpoint_blocks = False
    return rows


def te_bench(layers=(4, 8, 12), batch=32, tokens=96, n_embd=768, n_head=12, iters=5, warmup=2, device=None,
             log=print):
    """[{layers, ms, weights_mb}] of a Slayer-shaped frozen LM (random init) over ``batch`` caption rows."""
    from ..models.frozen_lm import LM_PAD, SlayerFrozenLM
    from ..models.slayer import GPT, GPTConfig
    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    g = torch.Generator().manual_seed(0)
    ids = torch.full((batch, tokens), LM_PAD, dtype=torch.int64)
    for r in range(batch):
        n = int(torch.randint(4, tokens + 1, (1,), generator=g))
        ids[r, :n] = torch.randint(0, 50000, (n,), generator=g)
    ids = ids.to(device)
    run = _timer(device)
    rows = []
    for n_layer in layers:
        torch.manual_seed(0)
        lm = SlayerFrozenLM("", model=GPT(GPTConfig(n_layer=n_layer, n_embd=n_embd, n_head=n_head)), device=device)
        weights = sum(p.numel() * p.element_size() for p in lm.model.parameters()) / 2 ** 20
        ms = run(lambda: lm.states(ids), iters, warmup)
        row = dict(bench="te", layers=n_layer, batch=batch, tokens=tokens, ms=ms, weights_mb=weights,
                   real_tokens=int(ids.ne(LM_PAD).sum()), device=str(device))
        rows.append(row)
        log(json.dumps(row))
        del lm
    return rows


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("ckpt")
    c.add_argument("--size", default="2b")
    c.add_argument("--blocks", type=int, default=4)
    c.add_argument("--mb", type=int, default=16)
    c.add_argument("--inflight", type=int, default=8)
    c.add_argument("--res", type=int, default=256)
    c.add_argument("--text-len", type=int, default=96)
    c.add_argument("--modes", nargs="+", default=["none", "full", "selective"], choices=["none", "full", "selective"])
    c.add_argument("--iters", type=int, default=3)
    c.add_argument("--warmup", type=int, default=1)
    t = sub.add_parser("te")
    t.add_argument("--layers", type=int, nargs="+", default=[4, 8, 12])
    t.add_argument("--batch", type=int, default=32)
    t.add_argument("--tokens", type=int, default=96)
    t.add_argument("--n-embd", type=int, default=768)
    t.add_argument("--n-head", type=int, default=12)
    t.add_argument("--iters", type=int, default=5)
    t.add_argument("--warmup", type=int, default=2)
    for q in (c, t):
        q.add_argument("--device", default=None)
    a = p.parse_args(argv)
    if a.cmd == "ckpt":
        return ckpt_bench(a.size, a.blocks, a.mb, a.inflight, a.res, a.text_len, a.modes, a.iters, a.warmup, a.device)
    return te_bench(a.layers, a.batch, a.tokens, a.n_embd, a.n_head, a.iters, a.warmup, a.device)


if __name__ == "__main__":
    main()
