"""MoE MLP: capacity-based dispatch equals the dense top-k oracle when nothing is dropped; expert parallelism over
Gloo ranks equals the local layer (outputs and gradients)."""
import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.models.moe import MoEMLP, moe_dense_reference


def test_moe_matches_dense_oracle():
    torch.manual_seed(0)
    m = MoEMLP(64, 96, experts=4, top_k=2, capacity_factor=4.0)
    h = torch.randn(3, 10, 64)
    out = m(h)
    ref = moe_dense_reference(m, h)
    assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5)
    assert m.aux_loss is not None and m.aux_loss.item() > 0


def test_moe_drops_beyond_capacity():
    torch.manual_seed(0)
    m = MoEMLP(32, 48, experts=2, top_k=1, capacity_factor=0.25)
    with torch.no_grad():
        m.router.weight.zero_()
        m.router.weight[0] = 1.0  # route (almost) everything to expert 0
    h = torch.randn(64, 32).abs()
    out = m(h)
    assert (out.abs().sum(-1) == 0).sum() > 0  # overflow assignments contribute nothing


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, d):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    full = MoEMLP(64, 96, experts=4, top_k=2, capacity_factor=4.0)
    ep = MoEMLP(64, 96, experts=4, top_k=2, capacity_factor=4.0, group=dist.group.WORLD)
    with torch.no_grad():
        ep.router.weight.copy_(full.router.weight)
        L = 4 // world
        ep.w_in.copy_(full.w_in[rank * L:(rank + 1) * L])
        ep.w_out.copy_(full.w_out[rank * L:(rank + 1) * L])
    h = torch.randn(2, 6, 64, generator=torch.Generator().manual_seed(10 + rank)).requires_grad_()
    out = ep(h)
    out.square().sum().backward()
    torch.save(dict(out=out.detach(), gh=h.grad, gw_in=ep.w_in.grad, gw_out=ep.w_out.grad, h=h.detach()),
               os.path.join(d, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_expert_parallel_matches_local():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    torch.manual_seed(0)
    full = MoEMLP(64, 96, experts=4, top_k=2, capacity_factor=4.0)
    gw_in = torch.zeros_like(full.w_in)
    gw_out = torch.zeros_like(full.w_out)
    for r in range(world):
        full.zero_grad()
        h = res[r]["h"].clone().requires_grad_()
        out = full(h)
        out.square().sum().backward()
        assert torch.allclose(out, res[r]["out"], atol=1e-5)
        assert torch.allclose(h.grad, res[r]["gh"], atol=1e-5)
        gw_in += full.w_in.grad
        gw_out += full.w_out.grad
    L = 4 // world
    for r in range(world):  # each rank's expert grads = sum over every rank's tokens routed to them
        assert torch.allclose(res[r]["gw_in"], gw_in[r * L:(r + 1) * L], atol=1e-4)
        assert torch.allclose(res[r]["gw_out"], gw_out[r * L:(r + 1) * L], atol=1e-4)
