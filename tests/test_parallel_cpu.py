"""Multi-process host-side logic on CPU (Gloo, world size 2): sharded Muon equals the unsharded optimizer, and
bucketed gradient reduction averages gradients across ranks."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _muon_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from trenowanie_generatora_obrazkow_b200.optim.muon import Muon
    torch.manual_seed(0)
    shapes = [(64, 32), (64, 32), (64, 32), (32, 96), (48, 48)]
    ps = [torch.nn.Parameter(torch.randn(*s) * 0.1) for s in shapes]
    opt = Muon(ps, lr=0.02, weight_decay=0.01, shard=True)
    for step in range(3):
        g = torch.Generator().manual_seed(100 + step)
        for p in ps:
            p.grad = torch.randn(p.shape, generator=g)
        opt.step()
    torch.save([p.detach() for p in ps], os.path.join(out_dir, f"muon_{rank}.pt"))
    dist.destroy_process_group()


def test_sharded_muon_matches_unsharded():
    from trenowanie_generatora_obrazkow_b200.optim.muon import Muon
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_muon_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        r0 = torch.load(os.path.join(d, "muon_0.pt"))
        r1 = torch.load(os.path.join(d, "muon_1.pt"))
    torch.manual_seed(0)
    shapes = [(64, 32), (64, 32), (64, 32), (32, 96), (48, 48)]
    ps = [torch.nn.Parameter(torch.randn(*s) * 0.1) for s in shapes]
    opt = Muon(ps, lr=0.02, weight_decay=0.01, shard=False)
    for step in range(3):
        g = torch.Generator().manual_seed(100 + step)
        for p in ps:
            p.grad = torch.randn(p.shape, generator=g)
        opt.step()
    for a, b, c in zip(r0, r1, ps):
        assert torch.equal(a, b), "ranks diverged"
        # bf16 Newton-Schulz: batching may change rounding; the error must stay below bf16 noise
        assert (a - c.detach()).abs().max() < 2e-3


def _bucket_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from trenowanie_generatora_obrazkow_b200.parallel.ddp import GradBuckets
    torch.manual_seed(0)
    lin = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8))
    gb = GradBuckets(list(lin.parameters()), bucket_bytes=512, comm="nccl_fp32")
    gb.zero()
    x = torch.randn(4, 16, generator=torch.Generator().manual_seed(7 + rank))
    gb.arm()
    lin(x).square().sum().backward()
    gb.finish()
    torch.save([p.grad.clone() for p in lin.parameters()], os.path.join(out_dir, f"g_{rank}.pt"))
    gb.close()
    dist.destroy_process_group()


def test_grad_buckets_average():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_bucket_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        g0 = torch.load(os.path.join(d, "g_0.pt"))
        g1 = torch.load(os.path.join(d, "g_1.pt"))
    torch.manual_seed(0)
    lin = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8))
    grads = []
    for rank in range(2):
        lin.zero_grad()
        x = torch.randn(4, 16, generator=torch.Generator().manual_seed(7 + rank))
        lin(x).square().sum().backward()
        grads.append([p.grad.clone() for p in lin.parameters()])
    for a, b, r0g, r1g in zip(g0, g1, grads[0], grads[1]):
        assert torch.allclose(a, b)
        assert torch.allclose(a, (r0g + r1g) / 2, atol=1e-5)


def _comm_check_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from trenowanie_generatora_obrazkow_b200.parallel import comm_check
    res = comm_check.main(["--sizes", "0.25", "1", "--iters", "2", "--warmup", "1", "--model-params", "1e6"])
    torch.save(res, os.path.join(out_dir, f"cc_{rank}.pt"))
    dist.destroy_process_group()


def test_comm_check_on_gloo_ranks():
    """parallel/comm_check.py (the reference's tests/check_nccl.py): correctness checks pass, bandwidth rows and a
    per-step gradient estimate are reported, with the same (max-over-ranks) times on every rank."""
    from trenowanie_generatora_obrazkow_b200.parallel import comm_check
    assert comm_check.bus_bandwidth(2 ** 30, 1.0, 8) == pytest.approx(2 ** 30 * 2 * 7 / 8 / 1e9)
    assert comm_check.grad_allreduce_ms(1e9, 100.0, 2) == pytest.approx(1e9 * 2 * 2 * 0.5 / 100e9 * 1e3)
    assert comm_check.grad_allreduce_ms(1e9, 100.0, 1) == 0.0
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_comm_check_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        r0, r1 = (torch.load(os.path.join(d, f"cc_{r}.pt")) for r in range(2))
    assert r0["world"] == 2 and r0["backend"] == "gloo" and [r["mb"] for r in r0["allreduce"]] == [0.25, 1]
    assert all(r["busbw_gbs"] > 0 for r in r0["allreduce"])
    assert [r["ms"] for r in r0["allreduce"]] == [r["ms"] for r in r1["allreduce"]]
    assert r0["grad_allreduce_ms"]["pg:1e+06"] > 0
