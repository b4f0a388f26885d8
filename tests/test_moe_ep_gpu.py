"""Expert parallelism on 2+ GPUs: the peer-memory exchange fused with the expert GEMMs against the NCCL
all_to_all path, outputs and all gradients, over several steps (one process per GPU, NCCL)."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, d):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    from trenowanie_generatora_obrazkow_b200.models.moe import MoEMLP
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    g = dist.group.WORLD
    torch.manual_seed(100 + rank)  # each rank's experts differ; the router is copied below
    ref = MoEMLP(512, 256, experts=2 * world, top_k=2, capacity_factor=1.5, group=g, transport="nccl").cuda()
    fus = MoEMLP(512, 256, experts=2 * world, top_k=2, capacity_factor=1.5, group=g, transport="p2p").cuda()
    with torch.no_grad():
        ref.router.weight.copy_(torch.randn(ref.router.weight.shape, generator=torch.Generator().manual_seed(7)).cuda()
                                * 0.05)
    fus.load_state_dict(ref.state_dict())
    res = []
    for it in range(3):
        h = torch.randn(2, 256, 512, generator=torch.Generator().manual_seed(1000 * it + rank)).cuda().bfloat16()
        row = []
        for m in (ref, fus):
            m.zero_grad(set_to_none=True)
            x = h.clone().requires_grad_()
            o = m(x)
            (o.float().square().mean() + 0.0).backward()
            row.append((o.float().cpu(), x.grad.float().cpu(), m.w_in.grad.cpu(), m.w_out.grad.cpu(),
                        m.router.weight.grad.cpu()))
        torch.cuda.synchronize()
        check_errors()
        res.append(row)
    torch.save(res, os.path.join(d, f"r{rank}.pt"))
    dist.barrier()
    fus.exchange.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_moe_peer_exchange_multi_gpu():
    world = min(8, torch.cuda.device_count())  # every visible GPU (experts = 2 per rank)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        for r in range(world):
            for it, (a, b) in enumerate(torch.load(os.path.join(d, f"r{r}.pt"))):
                for x, y in zip(b, a):
                    rel = ((x - y).norm() / y.norm().clamp(min=1e-12)).item()
                    assert rel < 3e-2, (r, it, rel)
