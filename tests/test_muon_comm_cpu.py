"""Owner-sharded Muon data flow (parallel/muon_comm.py, torch transport) on Gloo ranks: the same parameters,
momentum and gradient norm as the all-reduce + all-gather sharded Muon, for an even (2) and an uneven (3) world."""
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


SHAPES = [(64, 32), (64, 32), (64, 32), (32, 96), (48, 48), (96, 32), (64, 32)]


def _worker(rank, world, port, out_dir, momentum_dtype):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.optim.muon import Muon
    from trenowanie_generatora_obrazkow_b200.parallel.ddp import GradBuckets
    from trenowanie_generatora_obrazkow_b200.parallel.muon_comm import MuonShardedComm
    mdt = torch.bfloat16 if momentum_dtype == "bf16" else None
    torch.manual_seed(0)
    init = [torch.randn(*s) * 0.1 for s in SHAPES]
    pa = [torch.nn.Parameter(t.clone()) for t in init]
    pb = [torch.nn.Parameter(t.clone()) for t in init]
    # the 96 x 32 matrix is a fused q/k/v-like matrix split into three 32-row blocks (CMuon)
    opt_a = Muon(pa, lr=0.02, weight_decay=0.01, shard=True, splits={pa[5]: [32, 32, 32]}, momentum_dtype=mdt)
    opt_b = Muon(pb, lr=0.02, weight_decay=0.01, shard=True, splits={pb[5]: [32, 32, 32]}, momentum_dtype=mdt)
    ref_buckets = GradBuckets(pa, bucket_bytes=20000, comm="nccl_bf16", overlap=False)
    comm = MuonShardedComm(opt_b, transport="torch")
    buckets = GradBuckets(pb, bucket_bytes=20000, comm="nccl_bf16", reducer=comm.reduce_bucket)
    comm.attach_buckets(buckets)
    norms = []
    for step in range(3):
        g = torch.Generator().manual_seed(100 + 10 * step + rank)
        grads = [torch.randn(s, generator=g) for s in SHAPES]
        # reference: all-reduce, clip, Muon step
        ref_buckets.zero()
        for p, gr in zip(pa, grads):
            p.grad.copy_(gr)
        ref_buckets.finish()
        na = torch.nn.utils.clip_grad_norm_(pa, 5.0)
        opt_a.step()
        # owner-sharded path
        buckets.zero()
        comm.begin_step()
        buckets.arm()
        for p, gr in zip(pb, grads):
            p.grad.copy_(gr)
        buckets.finish()
        nb = comm.owned_sumsq().sqrt().reshape(())
        coef = (5.0 / (nb + 1e-6)).clamp(max=1.0)
        comm.step(coef)
        norms.append((float(na), float(nb)))
    comm.export_momentum()
    torch.save(dict(a=[p.detach() for p in pa], b=[p.detach() for p in pb], norms=norms,
                    ma=[opt_a.momentum_buffer(p).float() for p in pa],
                    mb=[opt_b.momentum_buffer(p).float() for p in pb]),
               os.path.join(out_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,momentum_dtype", [(2, "fp32"), (3, "fp32"), (2, "bf16")])
def test_sharded_muon_matches_gather_path(world, momentum_dtype):
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _free_port(), d, momentum_dtype), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    for o in outs:
        for na, nb in o["norms"]:
            assert abs(na - nb) < 1e-3 * na
        for a, b in zip(o["a"], o["b"]):
            # the owner path rounds the Nesterov direction to bf16 before the Frobenius normalisation
            assert (a - b).abs().max() < 2e-3, (a - b).abs().max()
        tol = 1e-5 if momentum_dtype == "fp32" else 2e-2
        for a, b in zip(o["ma"], o["mb"]):
            assert (a - b).abs().max() <= tol * max(1.0, a.abs().max()), (a - b).abs().max()
    for o in outs[1:]:  # every rank holds the same parameters
        for a, b in zip(outs[0]["b"], o["b"]):
            assert torch.equal(a, b)


def _trainer_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.models.config import SIZES, TE_SIZES
    from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig, Trainer
    den, te = SIZES["nano"], TE_SIZES["states-nano"]
    res = {}
    for mode in ("gather", "sharded"):
        tr = Trainer(den, te, TrainConfig(global_batch=4, micro_batch=2, steps=10, grad_comm="nccl_bf16",
                                          muon_comm=mode, clip=0.5, cfg_drop=0.0), "cpu")
        assert (tr.muon_comm is not None) == (mode == "sharded")
        for step in range(2):
            g = torch.Generator().manual_seed(1000 * step + rank)
            batch = {"x0": torch.randn(2, den.latent_channels, 8, 8, generator=g),
                     "lm_states": torch.randn(2, 16, te.lm_dim, generator=g)}
            tr.step(batch)
        res[mode] = [p.detach().clone() for p in tr.params]
        res[mode + "_gnorm"] = float(tr.last_gnorm)
        tr.close()
    torch.save(res, os.path.join(out_dir, f"t{rank}.pt"))
    dist.destroy_process_group()


def test_trainer_sharded_muon_matches_gather():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_trainer_worker, args=(world, _free_port(), d), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"t{r}.pt")) for r in range(world)]
    for o in outs:
        assert abs(o["gather_gnorm"] - o["sharded_gnorm"]) < 1e-3 * o["gather_gnorm"]
        for a, b in zip(o["gather"], o["sharded"]):
            assert (a - b).abs().max() < 3e-3, (a - b).abs().max()
    for a, b in zip(outs[0]["sharded"], outs[1]["sharded"]):
        assert torch.equal(a, b)
