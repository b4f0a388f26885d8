"""Owner-sharded Muon over peer memory (csrc/muon_comm.cu): on 2+ GPUs the parameters match the all-reduce +
all-gather sharded Muon and the bf16 shadows the GEMMs read are current; on one GPU the reduce-scatter's flag wait
for a peer that never arrives ends with an error code instead of hanging."""
import os
import socket
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(256, 128), (256, 128), (256, 128), (128, 384), (192, 192), (384, 128), (256, 128), (200, 136)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from trenowanie_generatora_obrazkow_b200.ops import fused as Fz
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    from trenowanie_generatora_obrazkow_b200.optim.muon import Muon
    from trenowanie_generatora_obrazkow_b200.parallel.ddp import GradBuckets
    from trenowanie_generatora_obrazkow_b200.parallel.muon_comm import MuonShardedComm
    torch.manual_seed(0)
    init = [torch.randn(*s, device="cuda") * 0.1 for s in SHAPES]
    pa = [torch.nn.Parameter(t.clone()) for t in init]
    pb = [torch.nn.Parameter(t.clone()) for t in init]
    opt_a = Muon(pa, lr=0.02, weight_decay=0.01, shard=True, splits={pa[5]: [128, 128, 128]})
    opt_b = Muon(pb, lr=0.02, weight_decay=0.01, shard=True, splits={pb[5]: [128, 128, 128]})
    ref = GradBuckets(pa, bucket_bytes=300000, comm="nccl_bf16", overlap=False)
    comm = MuonShardedComm(opt_b, transport="p2p", blocks=16, timeout_s=30)
    buckets = GradBuckets(pb, bucket_bytes=300000, comm="nccl_bf16", reducer=comm.reduce_bucket)
    comm.attach_buckets(buckets)
    norms = []
    for step in range(3):
        g = torch.Generator(device="cuda").manual_seed(100 + 10 * step + rank)
        grads = [torch.randn(s, device="cuda", generator=g) for s in SHAPES]
        ref.zero()
        for p, gr in zip(pa, grads):
            p.grad.copy_(gr)
        ref.finish()
        na = torch.nn.utils.clip_grad_norm_(pa, 20.0)
        opt_a.step()
        buckets.zero()
        comm.begin_step()
        buckets.arm()
        for p, gr in zip(pb, grads):
            p.grad.copy_(gr)
            Fz._notify(p)  # the fused Linear backward announces each finished weight gradient this way
        buckets.finish()
        nb = comm.owned_sumsq().sqrt().reshape(())
        comm.step((20.0 / (nb + 1e-6)).clamp(max=1.0))
        norms.append((float(na), float(nb)))
    torch.cuda.synchronize()
    check_errors()
    shadow_ok = all(torch.equal(Fz.bf16_weight(p), p.detach().bfloat16()) for p in pb)
    torch.save(dict(a=[p.detach().cpu() for p in pa], b=[p.detach().cpu() for p in pb], norms=norms,
                    shadow_ok=shadow_ok), os.path.join(out, f"r{rank}.pt"))
    buckets.close()
    comm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_muon_p2p_matches_gather_path():
    world = torch.cuda.device_count()  # every visible GPU
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    for o in outs:
        assert o["shadow_ok"]
        for na, nb in o["norms"]:
            assert abs(na - nb) < 2e-3 * na
        for a, b in zip(o["a"], o["b"]):
            assert (a - b).abs().max() < 3e-3, (a - b).abs().max()
    for o in outs[1:]:
        for a, b in zip(outs[0]["b"], o["b"]):
            assert torch.equal(a, b)


def test_muon_rs_wait_times_out_with_error_code():
    """One GPU, world 2: the second 'rank' never signals, so the reduce-scatter must give up with an error code."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import err_buf, ext
    dev = torch.cuda.current_device()
    blocks, n = 4, 4096
    staging = [ext().symm_alloc(n * 2, dev)[0] for _ in range(2)]
    flags = [ext().symm_alloc(2 * 2 * blocks * 4, dev)[0] for _ in range(2)]
    err = err_buf(torch.device("cuda", dev))
    err.zero_()
    grads = torch.randn(n, device="cuda")
    segs = torch.tensor([[0, 0, 1024]], dtype=torch.int64, device="cuda")
    g_owned = torch.zeros(1024, device="cuda")
    sumsq = torch.zeros(1, device="cuda")
    t0 = time.time()
    ext().muon_rs(grads, staging, flags, segs, 1024, g_owned, sumsq, 0, 2, 1, 0, blocks, int(0.2e9), err)
    torch.cuda.synchronize()
    assert time.time() - t0 < 10
    assert int(err[0].item()) == 4  # ERR_PEER_TIMEOUT
    err.zero_()
    for p in staging + flags:
        ext().symm_free(p, dev)
