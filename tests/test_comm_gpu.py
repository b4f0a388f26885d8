"""Peer-memory all-reduce (csrc/comm.cu): numerics on 2+ GPUs against an fp32 mean, and the bounded flag wait on
one GPU (a peer that never arrives must end the kernel with an error code, not hang it)."""
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


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    from trenowanie_generatora_obrazkow_b200.parallel.comm import PeerAllReduce
    ar = PeerAllReduce(1 << 20, blocks=16, timeout_s=20)
    res = []
    for n in (1000003, 4096, 777):
        g = torch.Generator(device="cuda").manual_seed(100 * rank + n)
        x = torch.randn(n, device="cuda", generator=g)
        ar(x)
        torch.cuda.synchronize()
        res.append(x.cpu())
    check_errors()
    torch.save(res, os.path.join(out, f"r{rank}.pt"))
    ar.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_matches_mean():
    world = torch.cuda.device_count()  # every visible GPU
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    for k, n in enumerate((1000003, 4096, 777)):
        ins = []
        for r in range(world):
            g = torch.Generator(device="cuda").manual_seed(100 * r + n)
            ins.append(torch.randn(n, device="cuda", generator=g).cpu())
        mean = torch.stack(ins).mean(0)
        for r in range(world):
            assert torch.equal(outs[r][k], outs[0][k]), "ranks disagree"
        rel = ((outs[0][k] - mean).norm() / mean.norm()).item()
        assert rel < 1e-2, rel


def test_peer_wait_times_out_with_error_code():
    """One GPU, world 2: the second 'rank' is never launched, so its flags never arrive."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import err_buf, ext
    dev = torch.cuda.current_device()
    blocks, n = 4, 4096
    slice_ = (n // 2 + 7) // 8 * 8
    bufs = [ext().symm_alloc(2 * slice_ * 2, dev)[0] for _ in range(4)]  # staging/result for both "ranks"
    flags = [ext().symm_alloc(3 * blocks * 4, dev)[0] for _ in range(2)]
    err = err_buf(torch.device("cuda", dev))
    err.zero_()
    x = torch.randn(n, device="cuda")
    import time
    t0 = time.time()
    ext().allreduce_bf16(x, [bufs[0], bufs[1]], [bufs[2], bufs[3]], flags, 0, 2, slice_, 1, 0.5, blocks,
                         int(0.2e9), err)
    torch.cuda.synchronize()
    assert time.time() - t0 < 10
    assert int(err[0].item()) == 4  # ERR_PEER_TIMEOUT
    err.zero_()
    for p in bufs + flags:
        ext().symm_free(p, dev)
