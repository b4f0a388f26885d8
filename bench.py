"""Headline benchmark: 1.24B-DiT flow-matching training throughput in latent tokens per second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
      bench.py --gpus N --steps K --warmup W

Config (the headline "1.24B DiT" training config): DiT hidden 2048, 24 blocks, 16 heads of 128, SwiGLU 5504 ("MLP 4x" param-matched),
2-block text refiner (1024 wide) on synthetic frozen-LM states [B, 128, 1024] ~ N(0, 1); 512 px synthetic FLUX.2
latents (128 channels at 32 x 32 = 1024 tokens / image) ~ N(0, 1); global batch 256 (micro-batch 32, gradient
accumulation 256 / (32 N)); bf16 compute; Muon (5 Newton-Schulz steps, sharded over ranks) + AdamW; EMA; random
init. One step = the whole optimizer step over the global batch. Global batch fixed across N: strong scaling.
Timing: W untimed warm-up steps, then K steps bracketed by barrier + synchronize, CUDA events on the launching
stream, max over ranks. Every step touches far more than L2 (126 MB) of activations and weights.
``e2e`` repeats the K steps through ``Trainer.step`` with the step's inputs in pinned host memory (copied to the
device inside the step) and the loss read back to the host every step.
``--impl reference`` runs the unmodified reference (installed in baseline/_ref) through its own modules on the
same config: aurora.model.Denoiser, aurora.slayer.LMTextEncoder (refiner on the same synthetic states),
train.param_groups (sharded Muon + fused AdamW), DDP with the bf16 compress hook, torch.compile, bf16 autocast.
"""
import argparse
import contextlib
import json
import os
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "baseline", "_ref")
BASELINE_VALUE = None  # the reference publishes no number for this metric
METRIC = "1.24B DiT train latent-tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="1.24b")
    p.add_argument("--global-batch", type=int, default=256)
    p.add_argument("--micro-batch", type=int, default=32)
    p.add_argument("--res", type=int, default=512)
    p.add_argument("--text-len", type=int, default=128)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--moe", action="store_true", help="MoE config: every other MLP -> 8 experts, top-2, "
                   "expert hidden 4096, expert-parallel over the GPUs")
    p.add_argument("--moe-transport", default="p2p", choices=["p2p", "nccl"],
                   help="--moe expert exchange: peer memory fused with the expert GEMMs (p2p) or NCCL all_to_all")
    p.add_argument("--pp", type=int, default=1, help="pipeline stages (pipeline config: --pp 4 on 8 GPUs, "
                   "--res 1024 --microbatches 8 --pp-micro 4)")
    p.add_argument("--microbatches", type=int, default=8)
    p.add_argument("--pp-micro", type=int, default=4)
    p.add_argument("--muon-comm", default="sharded", choices=["sharded", "gather"],
                   help="sharded: Muon gradients reduce-scattered to their owners and updates all-gathered into the "
                        "parameter update over peer memory; gather: all-reduce every gradient, all-gather updates")
    p.add_argument("--grad-comm", default="p2p", choices=["p2p", "nccl_bf16", "nccl_fp32"],
                   help="gradient reduction: the fused peer-memory kernel (p2p) or NCCL")
    p.add_argument("--sample-batch", type=int, default=8, help="prompts per GPU for the sampling measurement "
                   "(1024 px, 50 Euler steps, CFG 3, shift 6); 0 = skip it")
    p.add_argument("--sample-res", type=int, default=1024)
    p.add_argument("--sample-steps", type=int, default=50)
    p.add_argument("--sample-only", action="store_true", help="skip the training measurement: sampling img/s only")
    p.add_argument("--profile-dir", default="", help="profile one step after warm-up (torch.profiler), print the "
                   "kernel table and write traces there; the timed numbers are taken without the profiler")
    return p.parse_args()


# ------------------------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------------------------
# common harness
# ------------------------------------------------------------------------------------------------------------------
def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    from trenowanie_generatora_obrazkow_b200.utils.profiling import arm_stack_dump
    arm_stack_dump()
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def timed(step_fn, steps, world, local):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local)
    clk.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step_fn()
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    ms = torch.tensor([s.elapsed_time(e) / steps], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return ms.item(), clocks


def synthetic_batch(per_rank, res, text_len, lm_dim, device, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    side = res // 16
    x0 = torch.randn(per_rank, 128, side, side, generator=g)
    states = torch.randn(per_rank, text_len, lm_dim, generator=g).to(torch.bfloat16)
    host = {"x0": x0.pin_memory(), "lm_states": states.pin_memory()}
    dev = {k: v.to(device) for k, v in host.items()}
    return host, dev


def measure_sampling(run_batch, args, world, local):
    """Second headline metric: img/s of 1024 px, 50-step CFG sampling (one prompt batch per rank, whole-job
    images / max-over-ranks device time). run_batch(steps) samples one batch of args.sample_batch prompts."""
    run_batch(1)  # warm-up at the sampling shapes
    torch.cuda.synchronize()
    ms, clocks = timed(lambda: run_batch(args.sample_steps), 1, world, local)
    images = args.sample_batch * world
    return {"metric": "1024px 50-step CFG img/s", "value": round(images / (ms / 1e3), 3), "unit": "img/s",
            "ms_per_batch": round(ms, 1), "images_per_rank": args.sample_batch, "res": args.sample_res,
            "steps": args.sample_steps, "cfg": 3.0, "shift": 6.0, "clocks": clocks,
            "timed": "denoising loop on device (VAE decode not included: no FLUX.2 VAE weights offline)"}


def profile_sampling(run_batch, args, rank, steps=2):
    """With --profile-dir: torch.profiler table of `steps` sampling steps (after the warm-up; not a timed number)."""
    if not args.profile_dir:
        return
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        run_batch(steps)
        torch.cuda.synchronize()
    if rank == 0:
        os.makedirs(args.profile_dir, exist_ok=True)
        prof.export_chrome_trace(os.path.join(args.profile_dir, f"sampling_{args.impl}.json"))
        print(f"sampling profile ({steps} denoiser steps, batch {2 * args.sample_batch} with CFG):", flush=True)
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=45, max_name_column_width=90),
              flush=True)


def phase_breakdown(tr, batch, world, device, steps=2):
    """Per-phase device time of a step (ms, mean of `steps` extra steps after the timed region, max over ranks):
    forward_backward, grad_sync_exposed (gradient reductions still running after the last backward kernel),
    grad_norm, muon_momentum, muon_newton_schulz, muon_apply / muon_allgather_apply, adamw, ema_and_rest."""
    from trenowanie_generatora_obrazkow_b200.utils.profiling import PhaseTimer
    tr.timer = PhaseTimer(device)
    for _ in range(steps):
        tr.step(batch)
    got = tr.timer.collect()
    tr.timer = None
    names = list(got)
    vals = torch.tensor([got[k] / steps for k in names], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    return {k: round(v, 2) for k, v in zip(names, vals.tolist())}


def emit(rank, out):
    if rank == 0:
        print(json.dumps(out), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# our implementation
# ------------------------------------------------------------------------------------------------------------------
def run_ours(args):
    sys.path.insert(0, HERE)
    from trenowanie_generatora_obrazkow_b200.models.config import benchmark_configs
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, ext
    from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig, Trainer
    rank, world, local = setup_dist(args)
    device = torch.device("cuda", local)
    den_cfg, te_cfg = benchmark_configs(args.config)
    from dataclasses import replace
    den_cfg = replace(den_cfg, latent_size=args.res // 16)
    cfg = TrainConfig(global_batch=args.global_batch, micro_batch=args.micro_batch, steps=10 ** 6,
                      grad_comm=args.grad_comm, moe_experts=8 if args.moe else 0, muon_comm=args.muon_comm,
                      moe_transport=args.moe_transport)
    tr = Trainer(den_cfg, te_cfg, cfg, device)
    per_rank = args.global_batch // world
    if args.sample_only:
        return sample_ours(args, tr, den_cfg, te_cfg, rank, world, local, device, {"impl": "ours"})
    host, devb = synthetic_batch(per_rank, args.res, args.text_len, te_cfg.lm_dim, device, 1234 + rank)
    for _ in range(args.warmup):
        tr.step(devb)
    torch.cuda.synchronize()
    check_errors(device)
    if args.profile_dir:
        from trenowanie_generatora_obrazkow_b200.utils.profiling import TrainingProfile, export_profile, \
            summarize_kernels
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU,
                                                torch.profiler.ProfilerActivity.CUDA]) as prof:
            tr.step(devb)
            torch.cuda.synchronize()
        table, total = export_profile(prof, args.profile_dir, rank)
        if rank == 0:
            print(summarize_kernels(table[:40], total), flush=True)
    n0 = ext().launch_count()
    ms, clocks = timed(lambda: tr.step(devb), args.steps, world, local)
    launches = (ext().launch_count() - n0) // args.steps * args.steps
    check_errors(device)
    tokens = args.global_batch * (args.res // 16) ** 2
    value = tokens / (ms / 1e3)
    out = {"metric": METRIC, "value": round(value, 1), "unit": "latent-tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
           "dtype": "bf16", "data": "synthetic (N(0,1) FLUX.2-shaped latents and frozen-LM states), random init",
           "config": {"model": f"DiT {args.config}: hidden {den_cfg.dim}, {den_cfg.depth} blocks, {den_cfg.heads} "
                               f"heads, SwiGLU {den_cfg.mlp_hidden}, refiner {te_cfg.dim}x{te_cfg.depth}",
                      "params_denoiser": tr.n_params()[0], "params_text": tr.n_params()[1],
                      "global_batch": args.global_batch, "micro_batch": tr.micro, "seq_len": (args.res // 16) ** 2,
                      "text_len": args.text_len, "res": args.res, "parallelism": f"dp{world}",
                      "optimizer": "muon(sharded)+adamw", "grad_comm": args.grad_comm, "muon_comm": args.muon_comm,
                      "moe": (f"8 experts top-2 hidden 4096 every other block, expert-parallel, {args.moe_transport} "
                              "exchange") if args.moe else None,
                      "l2": "inputs larger than L2 (no flush needed)"},
           "clocks": clocks, "gpu_launches": int(launches), "impl": "ours"}
    out["phases_ms"] = phase_breakdown(tr, devb, world, device)
    if not args.no_e2e:
        loss_host = []

        def e2e_step():
            loss = tr.step(host)
            loss_host.append(loss.item())

        ms_e2e, _ = timed(e2e_step, args.steps, world, local)
        x_bytes = host["x0"].numel() * host["x0"].element_size()
        s_bytes = host["lm_states"].numel() * host["lm_states"].element_size()
        out["e2e"] = {"value": round(tokens / (ms_e2e / 1e3), 1), "unit": "latent-tokens/s",
                      "ms_per_step": round(ms_e2e, 2), "h2d_bytes_per_step": (x_bytes + s_bytes) * world,
                      "d2h_bytes_per_step": 4 * world,
                      "api": "Trainer.step(batch in pinned host memory) + loss.item()"}
    sample_ours(args, tr, den_cfg, te_cfg, rank, world, local, device, out)


def sample_ours(args, tr, den_cfg, te_cfg, rank, world, local, device, out):
    """Sampling img/s through sampling.euler.sample_latents (fused CFG + Euler update), then emit the line."""
    if args.sample_batch > 0:
        from trenowanie_generatora_obrazkow_b200.sampling.euler import encode_prompts, prompt_noise, sample_latents
        side = args.sample_res // 16
        g = torch.Generator(device="cpu").manual_seed(99 + rank)
        sst = torch.randn(args.sample_batch, args.text_len, te_cfg.lm_dim, generator=g).to(device, torch.bfloat16)
        tr.te.eval(), tr.den.eval()
        text, lens, null, nlen = encode_prompts(tr.te, lm_states=sst)
        noise = prompt_noise(args.sample_batch, den_cfg.latent_channels, side, 0, rank * args.sample_batch, device)

        def run_batch(steps):
            return sample_latents(tr.den, text, lens, null, nlen, steps=steps, cfg=3.0, shift=6.0,
                                  latent_size=side, noise=noise)

        out["sampling"] = measure_sampling(run_batch, args, world, local)
        profile_sampling(run_batch, args, rank)
    emit(rank, out)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------------------------------------
# the reference, unmodified, through its own modules
# ------------------------------------------------------------------------------------------------------------------
def run_reference(args):
    if not os.path.isdir(os.path.join(REF, "aurora")):
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
        return
    sys.path.insert(0, REF)
    import torch.nn as nn
    import torch.nn.functional as F
    from torch.nn.parallel import DistributedDataParallel as DDP

    import train as ref_train
    from aurora.model import Denoiser, DenoiserConfig, LMEncoderConfig
    from aurora.slayer import LM_NULL, LMTextEncoder

    rank, world, local = setup_dist(args)
    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    side = args.res // 16
    den_cfg = DenoiserConfig(dim=2048, depth=24, heads=16, mlp_hidden=5504, text_dim=1024, latent_size=side)
    te_cfg = LMEncoderConfig(repo="", tok_suffix="", lm_dim=1024, skip_last=0, dim=1024, depth=2, heads=16,
                             kv_heads=4, head_dim=64, mlp_hidden=2816, max_tokens=args.text_len, backend="states")
    torch.manual_seed(0)
    te = LMTextEncoder(te_cfg, with_lm=False)
    den = Denoiser(den_cfg)
    te.init_weights()
    den.init_weights()
    te.to(device), den.to(device)
    ref_args = ref_train.resolve_defaults(ref_train.get_args(
        ["--out", "/tmp/ref_bench", "--batch", str(args.global_batch), "--micro-batch", str(args.micro_batch),
         "--steps", "1000000", "--te-size", "slayer149", "--te-dim", "1024", "--repa-weight", "0",
         "--mlm-weight", "0", "--no-wandb"]))
    opts, _ = ref_train.param_groups(te, den, ref_args)
    te.compile()
    den.compile()

    class Step(nn.Module):  # train.FlowModel's flow-matching math, with the LM states passed to the refiner
        def __init__(self):
            super().__init__()
            self.te, self.den = te, den

        def forward(self, x0, ids, states, t, eps):
            text, valid = self.te(ids, lm_states=states)
            tt = t.view(-1, 1, 1, 1)
            v = self.den((1 - tt) * x0 + tt * eps, t, text, valid)
            return F.mse_loss(v.float(), eps - x0)

    model = Step()
    if world > 1:
        model = DDP(model, device_ids=[local], bucket_cap_mb=64, gradient_as_bucket_view=True)
        from torch.distributed.algorithms.ddp_comm_hooks import default_hooks
        model.register_comm_hook(None, default_hooks.bf16_compress_hook)
    params = [p for p in model.parameters() if p.requires_grad]
    ema_params = list(te.parameters()) + list(den.parameters())
    ema = [p.detach().clone().float() for p in ema_params] if rank == 0 else None
    per_rank = args.global_batch // world
    mb = min(args.micro_batch, per_rank)
    accum = per_rank // mb
    host, devb = synthetic_batch(per_rank, args.res, args.text_len, 1024, device, 1234 + rank)
    ids = torch.randint(0, 60000, (per_rank, args.text_len), device=device)
    null_row = torch.from_numpy(te.null_ids()).to(device)
    state = {"step": 0}

    out = {"impl": "reference"}
    if not args.sample_only:  # training measurement
        def step(batch):
            x0_all = batch["x0"].to(device, non_blocking=True)
            st_all = batch["lm_states"].to(device, non_blocking=True)
            for m in range(accum):
                sl = slice(m * mb, (m + 1) * mb)
                x0 = x0_all[sl].float()
                b = x0.shape[0]
                t = torch.sigmoid(torch.randn(b, device=device))
                eps = torch.randn_like(x0)
                drop = torch.rand(b, device=device) < ref_args.cfg_drop
                cond_ids = torch.where(drop[:, None], null_row[: ids.shape[1]], ids[sl])
                sync = model.no_sync() if (world > 1 and m < accum - 1) else contextlib.nullcontext()
                with sync:
                    with torch.autocast("cuda", dtype=torch.bfloat16):
                        loss = model(x0, cond_ids, st_all[sl], t, eps)
                    (loss / accum).backward()
            torch.nn.utils.clip_grad_norm_(params, ref_args.clip)
            mult = ref_train.lr_mult(state["step"], ref_args.steps, 0, ref_args.schedule)
            for o in opts:
                for g in o.param_groups:
                    g["lr"] = g["base_lr"] * mult
                o.step()
                o.zero_grad(set_to_none=True)
            state["step"] += 1
            if ema is not None:
                d = min(ref_args.ema, state["step"] / (9 + state["step"]))
                torch._foreach_lerp_(ema, [p.detach() for p in ema_params], 1 - d)
            return loss

        for _ in range(args.warmup):
            step(devb)
        torch.cuda.synchronize()
        ms, clocks = timed(lambda: step(devb), args.steps, world, local)
        tokens = args.global_batch * side * side
        value = tokens / (ms / 1e3)
        out = {"metric": METRIC, "value": round(value, 1), "unit": "latent-tokens/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (N(0,1) FLUX.2-shaped latents and frozen-LM states), random init",
               "config": {"model": "reference aurora.model.Denoiser 2048x24, 16 heads, SwiGLU 5504, refiner 1024x2",
                          "global_batch": args.global_batch, "micro_batch": mb, "seq_len": side * side,
                          "parallelism": f"dp{world}", "compile": True},
               "clocks": clocks, "impl": "reference"}
        if not args.no_e2e:
            def e2e_step():
                step(host).item()

            ms_e2e, _ = timed(e2e_step, args.steps, world, local)
            out["e2e"] = {"value": round(tokens / (ms_e2e / 1e3), 1), "unit": "latent-tokens/s",
                          "ms_per_step": round(ms_e2e, 2)}
    if args.sample_batch > 0:
        # the denoising loop of aurora/fid.py:sample with the reference's modules (its sample() derives text from
        # token ids through the frozen LM, which is replaced by synthetic states here)
        ss = args.sample_res // 16
        g = torch.Generator(device="cpu").manual_seed(99 + rank)
        nb = args.sample_batch
        sst = torch.randn(nb, args.text_len, 1024, generator=g).to(device, torch.bfloat16)
        s_ids = torch.randint(0, 60000, (nb, args.text_len), device=device)
        te.eval()
        # the reference's RoPE tables are (non-persistent) buffers sized by latent_size: a denoiser built for the
        # sampling resolution takes the trained weights (the same state dict at any resolution)
        from dataclasses import replace as _replace
        den_s = Denoiser(_replace(den_cfg, latent_size=ss))
        den_s.load_state_dict(den.state_dict())
        den_s.to(device).eval()
        den_s.compile()
        u = torch.linspace(1.0, 0.0, args.sample_steps + 1, device=device)
        shift = 6.0
        ts_all = shift * u / (1 + (shift - 1) * u)
        gz = torch.Generator(device=device).manual_seed(rank * nb)
        z0 = torch.randn(nb, 128, ss, ss, device=device, generator=gz)

        @torch.no_grad()
        def ref_sample(steps):
            z = z0.clone()
            ts = ts_all if steps == args.sample_steps else torch.linspace(1.0, 0.0, steps + 1, device=device)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                text, valid = te(torch.cat([null_row[: s_ids.shape[1]].expand(nb, -1), s_ids]),
                                 lm_states=torch.cat([sst, sst]))
                for k in range(steps):
                    t0, t1 = ts[k], ts[k + 1]
                    v = den_s(torch.cat([z, z]), t0.expand(2 * nb), text, valid).float()
                    v_u, v_c = v.chunk(2)
                    z = z + (t1 - t0) * (v_u + 3.0 * (v_c - v_u))
            return z

        out["sampling"] = measure_sampling(ref_sample, args, world, local)
        profile_sampling(ref_sample, args, rank)
    emit(rank, out)
    if world > 1:
        dist.destroy_process_group()


def run_pp(args):
    """1F1B pipeline x data parallel (the pipeline config): latent tokens / s of the whole job."""
    sys.path.insert(0, HERE)
    from dataclasses import replace
    from trenowanie_generatora_obrazkow_b200.models.config import benchmark_configs
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, ext
    from trenowanie_generatora_obrazkow_b200.train.pp_trainer import PPTrainer
    from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig
    rank, world, local = setup_dist(args)
    device = torch.device("cuda", local)
    den_cfg, te_cfg = benchmark_configs(args.config)
    side = args.res // 16
    den_cfg = replace(den_cfg, latent_size=side)
    dp = world // args.pp
    n = args.microbatches * args.pp_micro
    cfg = TrainConfig(global_batch=n * dp, micro_batch=args.pp_micro, steps=10 ** 6, grad_comm=args.grad_comm)
    tr = PPTrainer(den_cfg, te_cfg, cfg, device, args.pp, args.microbatches)
    host, devb = synthetic_batch(n if tr.first else 1, args.res, args.text_len, te_cfg.lm_dim, device, 1234 + rank)
    batch = dict(devb, n=n, side=side, text_len=args.text_len)
    for _ in range(args.warmup):
        tr.step(batch)
    torch.cuda.synchronize()
    check_errors(device)
    n0 = ext().launch_count()
    ms, clocks = timed(lambda: tr.step(batch), args.steps, world, local)
    launches = (ext().launch_count() - n0)
    check_errors(device)
    tokens = n * dp * side * side
    value = tokens / (ms / 1e3)
    out = {"metric": METRIC, "value": round(value, 1), "unit": "latent-tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (N(0,1) FLUX.2-shaped latents and frozen-LM states), random init",
           "config": {"model": f"DiT {args.config}", "global_batch": n * dp, "microbatches": args.microbatches,
                      "micro_batch": args.pp_micro, "seq_len": side * side, "res": args.res,
                      "parallelism": f"pp{args.pp}xdp{dp}", "schedule": "1F1B", "grad_comm": args.grad_comm,
                      "l2": "inputs larger than L2 (no flush needed)"},
           "clocks": clocks, "gpu_launches_rank0": int(launches), "impl": "ours"}
    emit(rank, out)
    dist.destroy_process_group()


def launch_ranks(args, argv=None):
    """``--gpus N`` without a launcher: re-run this command under torch.distributed.run with N ranks (one per GPU,
    rendezvous on 127.0.0.1). Under a launcher the world size must equal --gpus."""
    world = os.environ.get("WORLD_SIZE")
    if world is not None:
        if int(world) != args.gpus and args.gpus != 1:
            raise SystemExit(f"bench.py --gpus {args.gpus} under a launcher with WORLD_SIZE={world}")
        return None
    if args.gpus <= 1:
        return None
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(args.gpus),
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.abspath(__file__)]
    return cmd + list(sys.argv[1:] if argv is None else argv)


def main():
    args = parse()
    cmd = launch_ranks(args)
    if cmd is not None:
        os.execv(sys.executable, cmd)
    if args.pp > 1:
        run_pp(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
