"""1F1B pipeline (parallel/pipeline.py) against the unsplit model: a 2-stage pipe (one-direction NCCL / Gloo links,
receives posted ahead, sends completed at the end of the step) gives the loss and every parameter gradient of the
same model run as one stage, over several micro-batches. CPU: two Gloo ranks; GPU: two NCCL ranks on two GPUs."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

M = 3  # micro-batches


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfgs():
    from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig
    den = DenoiserConfig(dim=256, depth=4, heads=2, mlp_hidden=512, text_dim=256, latent_size=8)
    te = LMEncoderConfig(repo="", tok_suffix="", lm_dim=128, skip_last=0, dim=256, depth=1, heads=4, kv_heads=2,
                         head_dim=64, mlp_hidden=512, max_tokens=16, backend="states")
    return den, te


def _run(stage_ranks, pp, device, out_dir, tag):
    """Run one 1F1B step of the pipe `stage_ranks` (this rank's stage = its index) and save loss and grads."""
    from trenowanie_generatora_obrazkow_b200.models import build_models
    from trenowanie_generatora_obrazkow_b200.ops import fused as Fz
    from trenowanie_generatora_obrazkow_b200.parallel.pipeline import (OneFOneB, StageModel, direction_groups,
                                                                       stage_ranges)
    den_cfg, te_cfg = _cfgs()
    rank = dist.get_rank()
    s = stage_ranks.index(rank)
    torch.manual_seed(0)
    te, den = build_models(den_cfg, te_cfg)
    te.init_weights(), den.init_weights()
    for p in list(te.parameters()) + list(den.parameters()):  # no zero-initialised branches: every grad counts
        p.data.add_(0.02 * torch.randn_like(p))
    te_sd, den_sd = te.state_dict(), den.state_dict()
    lo, hi = stage_ranges(den_cfg.depth, pp, 1.0)[s]
    model = StageModel(den_cfg, te_cfg, lo, hi, s == 0, s == pp - 1, device)
    model.load_full_state(te_sd, den_sd)
    links = direction_groups([stage_ranks]) if pp > 1 else None
    g = torch.Generator().manual_seed(7)
    mb, side, C, L = 2, den_cfg.latent_size, den_cfg.latent_channels, te_cfg.max_tokens
    x0 = torch.randn(M * mb, C, side, side, generator=g).to(device)
    eps = torch.randn(M * mb, C, side, side, generator=g).to(device)
    t = torch.rand(M * mb, generator=g).to(device)
    dt = torch.bfloat16 if device.type == "cuda" else torch.float32
    states = torch.randn(M * mb, L, te_cfg.lm_dim, generator=g).to(device, dt)
    inputs, targets = [], []
    for i in range(M):
        sl = slice(i * mb, (i + 1) * mb)
        z_tok, target = Fz.fm_inputs(x0[sl], eps[sl], t[sl])
        kw = dict(lm_states=states[sl], valid=torch.ones(mb, L, dtype=torch.bool, device=device), is_null=None,
                  hw=(side, side))
        inputs.append((z_tok, t[sl], kw))
        targets.append(target.float().contiguous())
    shapes = dict(x=(mb, side * side, den_cfg.dim), t6=(mb, 6, den_cfg.dim), text=(mb, L, den_cfg.text_dim), dtype=dt)
    sched = OneFOneB(model, stage_ranks, s, shapes, device, links=links)
    loss = sched.step(M, (lambda i: inputs[i]) if s == 0 else None, targets if s == pp - 1 else None, side, 1.0 / M)
    grads = {f"{pre}.{n}": p.grad.float().cpu() for pre, n, p in model.full_named_parameters() if p.grad is not None}
    torch.save(dict(loss=None if loss is None else float(loss), grads=grads),
               os.path.join(out_dir, f"{tag}_s{s}.pt"))


def _worker(rank, world, port, out_dir, use_cuda):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    if use_cuda:
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=device)
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    _run([0, 1], 2, device, out_dir, "pp2")
    dist.barrier()
    if rank == 0:  # the unsplit model: one stage holding everything
        solo = dist.new_group([0])
        _run([0], 1, device, out_dir, "pp1")
    else:
        dist.new_group([0])
    dist.barrier()
    if use_cuda:
        torch.cuda.synchronize()
    dist.destroy_process_group()


def _check(d, tol):
    a0, a1 = torch.load(os.path.join(d, "pp2_s0.pt")), torch.load(os.path.join(d, "pp2_s1.pt"))
    ref = torch.load(os.path.join(d, "pp1_s0.pt"))
    assert abs(a1["loss"] - ref["loss"]) <= tol * abs(ref["loss"])
    got = dict(a0["grads"], **a1["grads"])
    assert set(got) == set(ref["grads"])
    for k, v in ref["grads"].items():
        err = ((got[k] - v).norm() / v.norm().clamp_min(1e-12)).item()
        assert err <= tol, (k, err)


def test_pp2_matches_unsplit_cpu():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d, False), nprocs=2, join=True)
        _check(d, 1e-5)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pp2_matches_unsplit_gpu():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d, True), nprocs=2, join=True)
        _check(d, 1e-2)
