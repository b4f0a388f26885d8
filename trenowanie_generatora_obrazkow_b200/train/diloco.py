"""DiLoCo / MuLoCo local-SGD outer step (reference train.py:381-412, train_pp.py:429-443).

Every worker trains its own copy for H inner steps (unsharded Muon); then the pseudo-gradient
``global - local`` is averaged over the workers (bucketed; bf16 or fp32 on the wire) and applied to the global
weights by an outer optimizer (Nesterov SGD; lr 1 / momentum 0 is plain weight averaging); the new global weights
replace every local copy. Global weights may live in pinned host memory (``offload``): each bucket is moved to the
GPU only for its own update.
"""
import torch
import torch.distributed as dist


def make_global(live, offload=False):
    """fp32 global copies of the live parameters (pinned host memory with offload) + their outer optimizer."""
    out = []
    for p in live:
        g = p.detach().float().cpu().pin_memory() if offload else p.detach().clone().float()
        out.append(torch.nn.Parameter(g, requires_grad=False))
    return out


def make_outer_opt(global_params, lr=0.7, momentum=0.9):
    return torch.optim.SGD(global_params, lr=lr, momentum=momentum, nesterov=momentum > 0)


def _buckets(params, bucket):
    idx, out, size = [], [], 0
    for i, p in enumerate(params):
        idx.append(i)
        size += p.numel()
        if size >= bucket or i == len(params) - 1:
            out.append(idx)
            idx, size = [], 0
    return out


@torch.no_grad()
def outer_sync(global_params, live, outer_opt, n, comm="bf16", group=None, bucket=64 * 2 ** 20):
    for chunk in _buckets(global_params, bucket):
        dev = live[chunk[0]].device
        flat = torch.cat([(global_params[i].to(dev, non_blocking=True) - live[i].detach().float()).flatten()
                          for i in chunk])
        if dist.is_available() and dist.is_initialized() and n > 1:
            if comm == "bf16":
                lo = flat.bfloat16()
                dist.all_reduce(lo, group=group)
                flat.copy_(lo)
            else:
                dist.all_reduce(flat, group=group)
            flat /= n
        flat = flat.to(global_params[chunk[0]].device)
        for i, d in zip(chunk, flat.split([global_params[i].numel() for i in chunk])):
            global_params[i].grad = d.view_as(global_params[i])
        outer_opt.step()
        outer_opt.zero_grad(set_to_none=True)
        for i in chunk:
            live[i].copy_(global_params[i], non_blocking=True)


def ema_decay_at_sync(ema, H, n_syncs):
    """EMA decay at an outer sync: the same window in samples as the per-step EMA (reference train.py:955-957)."""
    return min(ema ** H, (1 + n_syncs) / (10 + n_syncs))
