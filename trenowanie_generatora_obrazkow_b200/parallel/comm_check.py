"""All-reduce sanity and bandwidth check, independent of training (reference tests/check_nccl.py).

  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m trenowanie_generatora_obrazkow_b200.parallel.comm_check
  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m trenowanie_generatora_obrazkow_b200.parallel.comm_check \\
      --impl pg peer --sizes 1 16 64 256 --model-params 1.55e9
  NCCL_DEBUG=INFO torchrun ...      # shows the transport NCCL picks (P2P / NVLS / SHM / NET)

Every rank first checks a one-element all-reduce (the sum must equal the world size) and a random-tensor all-reduce
against the sum of the ranks' tensors. Then, per message size, it times ``iters`` all-reduces of bf16 data after
``warmup`` untimed ones: on GPUs with CUDA events on the launching stream, the duration the max over ranks; on a CPU
(Gloo) run by wall clock. Bus bandwidth = bytes x 2 (world - 1) / world / time, the usual all-reduce convention.
Implementations: ``pg`` is the process group's all-reduce (NCCL on GPUs), ``peer`` this framework's peer-memory
kernel (parallel/comm.PeerAllReduce: fp32 in and out, bf16 on the wire, the data-parallel gradient transport; GPUs
only). The last lines estimate the gradient all-reduce time of one training step for a model of ``--model-params``
parameters with bf16 gradients at the largest size's bandwidth (it overlaps with the backward pass in training).
Rank 0 prints one JSON line with everything measured.
"""
import argparse
import json
import os
import time

import torch
import torch.distributed as dist


def check_allreduce(device, group=None):
    """Raises AssertionError when the process group's all-reduce returns a wrong sum."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    x = torch.ones(1, device=device)
    dist.all_reduce(x, group=group)
    assert x.item() == world, f"all_reduce of ones gave {x.item()} on {world} ranks"
    g = torch.Generator().manual_seed(1234)
    parts = [torch.randn(4097, generator=g) for _ in range(world)]
    y = parts[rank].to(device, copy=True)
    dist.all_reduce(y, group=group)
    want = torch.stack(parts).sum(0)
    assert torch.allclose(y.cpu(), want, rtol=1e-5, atol=1e-5), "all_reduce of random tensors differs from the sum"
    return True


def bus_bandwidth(nbytes, seconds, world):
    return nbytes * 2 * (world - 1) / world / seconds / 1e9 if world > 1 and seconds > 0 else 0.0


def _max_over_ranks(value, device, group=None):
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def time_allreduce(fn, device, iters=10, warmup=3, group=None):
    """Seconds per call of fn() (max over ranks): CUDA events on GPUs, wall clock on CPUs."""
    for _ in range(warmup):
        fn()
    cuda = torch.device(device).type == "cuda"
    dist.barrier(group=group)
    if cuda:
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize(device)
        sec = a.elapsed_time(b) / 1e3 / iters
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        sec = (time.perf_counter() - t0) / iters
    return _max_over_ranks(sec, device, group)


def measure(sizes_mb, impls, device, iters=10, warmup=3, group=None, log=print):
    """[{impl, mb, ms, busbw_gbs}] for each implementation and size (bf16 payload of ``mb`` MiB)."""
    world = dist.get_world_size(group)
    rows = []
    for impl in impls:
        peer = None
        if impl == "peer":
            if torch.device(device).type != "cuda":
                log("peer: needs GPUs, skipped")
                continue
            from .comm import PeerAllReduce
            peer = PeerAllReduce(int(max(sizes_mb) * 2 ** 20) // 2, group=group, device=device)
        for mb in sizes_mb:
            n = int(mb * 2 ** 20) // 2
            if impl == "peer":
                t = torch.randn(n, device=device)
                fn = (lambda t=t: peer(t))
            else:
                t = torch.randn(n, dtype=torch.bfloat16, device=device)
                fn = (lambda t=t: dist.all_reduce(t, group=group))
            sec = time_allreduce(fn, device, iters, warmup, group)
            row = dict(impl=impl, mb=mb, ms=sec * 1e3, busbw_gbs=bus_bandwidth(n * 2, sec, world))
            rows.append(row)
            log(f"{impl:4s} all_reduce {mb:6g} MB bf16: {row['ms']:8.3f} ms   bus bandwidth {row['busbw_gbs']:7.1f} GB/s")
        if peer is not None:
            peer.close()
    return rows


def grad_allreduce_ms(params, busbw_gbs, world):
    """Milliseconds to all-reduce ``params`` bf16 gradients at a bus bandwidth (0 on one rank)."""
    if world < 2 or busbw_gbs <= 0:
        return 0.0
    return params * 2 * 2 * (world - 1) / world / (busbw_gbs * 1e9) * 1e3


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--sizes", type=float, nargs="+", default=[1, 16, 64, 256], help="MiB of bf16 per all-reduce")
    p.add_argument("--impl", nargs="+", default=["pg"], choices=["pg", "peer"])
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--model-params", type=float, nargs="*", default=[63e6, 116e6, 1.55e9],
                   help="parameter counts for the per-step gradient all-reduce estimate")
    p.add_argument("--timeout", type=float, default=120.0, help="process-group timeout, seconds")
    a = p.parse_args(argv)
    from datetime import timedelta
    cuda = torch.cuda.is_available() and not os.environ.get("PP_CPU")
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    backend = os.environ.get("DIST_BACKEND", "nccl" if cuda else "gloo")
    own = not dist.is_initialized()
    if own:
        dist.init_process_group(backend, timeout=timedelta(seconds=a.timeout))
    rank, world = dist.get_rank(), dist.get_world_size()
    device = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    log = print if rank == 0 else (lambda *x, **k: None)
    check_allreduce(device)
    name = torch.cuda.get_device_name(device) if cuda else "CPU"
    log(f"all_reduce OK on {world} ranks ({name}, {dist.get_backend()})", flush=True)
    rows = measure(a.sizes, a.impl, device, a.iters, a.warmup, log=lambda s: log(s, flush=True))
    est = {}
    for impl in a.impl:
        mine = [r for r in rows if r["impl"] == impl]
        if not mine:
            continue
        top = max(mine, key=lambda r: r["mb"])
        for n in a.model_params:
            ms = grad_allreduce_ms(n, top["busbw_gbs"], world)
            est[f"{impl}:{n:.3g}"] = ms
            if world > 1:
                log(f"~{ms:.1f} ms of bf16 gradient all-reduce per step for {n / 1e6:.0f}M parameters ({impl}, "
                    f"{top['busbw_gbs']:.0f} GB/s; overlapped with the backward pass in training)")
    result = dict(world=world, backend=dist.get_backend(), device=name, allreduce=rows, grad_allreduce_ms=est)
    log(json.dumps(result))
    if own:
        dist.destroy_process_group()
    return result


if __name__ == "__main__":
    main()
