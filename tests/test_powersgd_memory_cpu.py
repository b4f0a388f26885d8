"""PowerSGD reducer (parallel/powersgd.py) on Gloo ranks: exact averaging during warm-up, rank-r approximations
afterwards that, with error feedback, converge to the true mean over repeated steps; memory diagnostics."""
import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.parallel.ddp import GradBuckets
    from trenowanie_generatora_obrazkow_b200.parallel.powersgd import PowerSGD
    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.zeros(48, 32)), torch.nn.Parameter(torch.zeros(32)),
          torch.nn.Parameter(torch.zeros(40, 24))]
    gb = GradBuckets(ps, comm="nccl_fp32", overlap=False)
    psgd = PowerSGD(gb, rank=4, start_iter=1, seed=3)
    gb.reducer = psgd
    g = torch.Generator().manual_seed(100 + rank)
    fixed = [torch.randn(p.shape, generator=g) for p in ps]  # the same local gradient every step
    res = []
    for step in range(30):
        gb.zero()
        for p, f in zip(ps, fixed):
            p.grad.copy_(f)
        gb.finish()
        psgd.next_step()
        res.append([p.grad.clone() for p in ps])
    torch.save(dict(res=res, fixed=fixed), os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_powersgd_warmup_exact_then_error_feedback_converges():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    mean = [sum(o["fixed"][i] for o in outs) / world for i in range(3)]
    for i in range(3):  # step 0: plain averaging
        assert torch.allclose(outs[0]["res"][0][i], mean[i], atol=1e-6)
    assert torch.allclose(outs[0]["res"][5][1], mean[1], atol=1e-6)  # vectors stay uncompressed
    for i in (0, 2):
        single = (outs[0]["res"][1][i] - mean[i]).norm() / mean[i].norm()
        avg = sum(o for o in (s[i] for s in outs[0]["res"][1:])) / 29  # error feedback: the running mean converges
        assert single > 0.05 and (avg - mean[i]).norm() / mean[i].norm() < single / 3
    for a, b in zip(outs[0]["res"][-1], outs[1]["res"][-1]):
        assert torch.allclose(a, b)


def test_memory_breakdown_and_oom_guard():
    import pytest

    from trenowanie_generatora_obrazkow_b200.utils.memory import breakdown, host_rss_gb, oom_guard, report
    ps = [torch.zeros(1024, 256), torch.zeros(256)]
    opt = torch.optim.AdamW(ps, lr=1e-3)
    for p in ps:
        p.grad = torch.ones_like(p)
    opt.step()
    b = breakdown(params=ps, grads=[p.grad for p in ps], opts=[opt])
    gb = 1024 ** 3
    assert abs(b["weights"] * gb - (1024 * 256 + 256) * 4) < 1 and b["optimizer"] * gb >= 2 * (1024 * 256 + 256) * 4
    assert host_rss_gb() > 0 and "weights" in report(params=ps)
    seen = []
    with pytest.raises(torch.OutOfMemoryError):
        with oom_guard(lambda: "breakdown", log=seen.append):
            raise torch.OutOfMemoryError("simulated")
    assert seen == ["breakdown"]
