"""1F1B pipeline (Gloo on CPU, fp32): loss and every parameter gradient equal the unsplit model's
(the reference's tests/check_pp.py invariant), for 2 and 3 stages."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig, build_models

DEN = DenoiserConfig(dim=128, depth=4, heads=2, mlp_hidden=256, text_dim=128, latent_channels=32, latent_size=8)
TE = LMEncoderConfig(lm_dim=64, dim=128, depth=1, heads=2, kv_heads=1, head_dim=64, mlp_hidden=256, max_tokens=16,
                     backend="states")
M, MB = 4, 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _full():
    torch.manual_seed(0)
    te, den = build_models(DEN, TE)
    with torch.no_grad():  # non-trivial weights everywhere (zero inits hide mistakes)
        for p in list(te.parameters()) + list(den.parameters()):
            p.add_(0.05 * torch.randn_like(p))
    return te, den


def _data():
    g = torch.Generator().manual_seed(1)
    x0 = torch.randn(M, MB, 32, 8, 8, generator=g)
    eps = torch.randn(M, MB, 32, 8, 8, generator=g)
    t = torch.rand(M, MB, generator=g)
    states = torch.randn(M, MB, 16, 64, generator=g)
    valid = torch.ones(M, MB, 16, dtype=torch.bool)
    valid[:, 1, 9:] = False
    return x0, eps, t, states, valid


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.parallel.pipeline import (OneFOneB, StageModel, recv_targets,
                                                                         send_targets, stage_ranges)
    te, den = _full()
    lo, hi = stage_ranges(DEN.depth, world, 1.0)[rank]
    sm = StageModel(DEN, TE, lo, hi, rank == 0, rank == world - 1, "cpu")
    sm.load_full_state(te.state_dict(), den.state_dict())
    x0, eps, t, states, valid = _data()
    T = DEN.latent_size ** 2
    targets = [(eps[i] - x0[i]).flatten(2).transpose(1, 2).contiguous() for i in range(M)]
    pipe = list(range(world))
    if world > 1:
        if rank == 0:
            send_targets(targets, pipe)
        elif rank == world - 1:
            targets = recv_targets(M, targets[0].shape, torch.float32, "cpu", pipe)

    def first_inputs(i):
        tt = t[i].view(-1, 1, 1, 1)
        return (1 - tt) * x0[i] + tt * eps[i], t[i], dict(lm_states=states[i], valid=valid[i])

    shapes = dict(x=(MB, T, DEN.dim), t6=(MB, 6, DEN.dim), text=(MB, 16, DEN.text_dim), dtype=torch.float32)
    sched = OneFOneB(sm, pipe, rank, shapes, "cpu")
    loss = sched.step(M, first_inputs, targets, side=DEN.latent_size, loss_scale=1.0 / M)
    grads = {f"{pre}.{n}": (None if p.grad is None else p.grad.clone()) for pre, n, p in sm.full_named_parameters()}
    torch.save(dict(loss=loss, grads=grads), os.path.join(out, f"s{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_1f1b_matches_unsplit(world):
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"s{r}.pt")) for r in range(world)]
    te, den = _full()
    x0, eps, t, states, valid = _data()
    total = 0.0
    for i in range(M):
        tt = t[i].view(-1, 1, 1, 1)
        text, v = te(lm_states=states[i], valid=valid[i])
        pred = den((1 - tt) * x0[i] + tt * eps[i], t[i], text, v)
        loss = torch.nn.functional.mse_loss(pred, eps[i] - x0[i]) / M
        loss.backward()
        total += loss.item()
    assert abs(res[-1]["loss"].item() - total) < 1e-5 * max(1.0, abs(total))
    ref = {f"te.{n}": p.grad for n, p in te.named_parameters()}
    ref.update({f"den.{n}": p.grad for n, p in den.named_parameters()})
    seen = set()
    for r in res:
        for k, g in r["grads"].items():
            seen.add(k)
            rg = ref[k]
            if g is None or rg is None:  # unused this step (the learned null vector without null prompts)
                assert g is None and rg is None, k
                continue
            assert ((g - rg).norm() / rg.norm().clamp_min(1e-12)).item() < 1e-4, k
    assert seen == set(ref)
