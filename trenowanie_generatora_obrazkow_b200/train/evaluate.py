"""Held-out evaluation and training statistics.

evaluate(): velocity MSE on a fixed held-out set with fixed t and noise (reference train.py:415-473): t from a
seeded CPU generator (logit-normal), every 8th sample instead uniform in [0.9, 1) and reported only as
val/loss_t0.90-1.00; the rest reported overall and in four t buckets; optional per-group losses.
weight_sq(): per-kind sum of squares of the hidden matrices (reference train.py:230-257).
grad_sq_norms() / noise_scale(): gradient-noise-scale estimate (McCandlish et al. 2018; reference
train.py:260-281).
"""
import torch
import torch.distributed as dist

from ..models.text import LMTextEncoder


@torch.no_grad()
def evaluate(te, den, val, device, seed=1234, chunk=256, groups=(), den_chunk=0, lm_states=None, t_shift=1.0):
    """val = (latents (N, C, h, w), ids (N, L)) or (latents, LM states (N, L, D)) for an LM refiner."""
    lat, ids = val
    g = torch.Generator(device="cpu").manual_seed(seed)
    t_all = torch.sigmoid(torch.randn(len(lat), generator=g))
    if t_shift != 1.0:
        t_all = t_shift * t_all / (1 + (t_shift - 1) * t_all)
    eps_all = torch.randn(lat.shape, generator=g)
    hi_mask = torch.arange(len(lat)) % 8 == 7
    t_all[hi_mask] = 0.9 + 0.1 * torch.rand(int(hi_mask.sum()), generator=torch.Generator().manual_seed(seed + 7))
    was_training = te.training, den.training
    te.eval(), den.eval()
    buckets = torch.zeros(2, 4)
    hi = torch.zeros(2)
    tot, n = 0.0, 0
    per_all = []
    for i in range(0, len(lat), chunk):
        x0 = lat[i:i + chunk].to(device).float()
        t, eps = t_all[i:i + chunk].to(device), eps_all[i:i + chunk].to(device)
        if isinstance(te, LMTextEncoder):
            states = (lm_states[i // chunk] if lm_states is not None else ids[i:i + chunk]).to(device)
            text, valid = te(lm_states=states)
        else:
            text, valid = te(ids[i:i + chunk].to(device))
        tt = t.view(-1, 1, 1, 1)
        zt = (1 - tt) * x0 + tt * eps
        dc = den_chunk or len(x0)
        v = torch.cat([den(zt[j:j + dc], t[j:j + dc], text[j:j + dc], valid[j:j + dc]).float()
                       for j in range(0, len(x0), dc)])
        per = (v - (eps - x0)).pow(2).mean(dim=(1, 2, 3)).cpu()
        per_all.append(per)
        m = hi_mask[i:i + chunk]
        hi += torch.stack([per[m].sum(), m.sum().float()])
        keep, tc = per[~m], t.cpu()[~m]
        tot += keep.sum().item()
        n += len(keep)
        b = (tc * 4).long().clamp(max=3)
        buckets[0].index_add_(0, b, keep)
        buckets[1].index_add_(0, b, torch.ones_like(keep))
    te.train(was_training[0]), den.train(was_training[1])
    out = {"val/loss": tot / max(n, 1)}
    for k in range(4):  # a bucket without samples (small validation sets) reads nan, not a zero loss
        out[f"val/loss_t{k / 4:.2f}-{(k + 1) / 4:.2f}"] = (buckets[0][k] / buckets[1][k]).item() \
            if buckets[1][k] > 0 else float("nan")
    out["val/loss_t0.90-1.00"] = (hi[0] / hi[1]).item() if hi[1] > 0 else float("nan")
    per_all, i = torch.cat(per_all), 0
    for label, count in groups:
        keep = ~hi_mask[i:i + count]
        out[f"val_{label}/loss"] = per_all[i:i + count][keep].mean().item()
        i += count
    return out


WRMS_KINDS = ("attn.qkv", "attn.out", "cross.q", "cross.kv", "cross.out", "mlp.in_proj", "mlp.out_proj")
WRMS_KEYS = [f"den_{k}" for k in WRMS_KINDS] + ["te_refiner", "hidden"]


@torch.no_grad()
def weight_sq(named, device):
    """(len(WRMS_KEYS), 2) tensor of (sum of squares, count) per kind of hidden block matrix."""
    acc = torch.zeros(len(WRMS_KEYS), 2, device=device)
    for prefix, name, p in named:
        if p.ndim != 2 or ".blocks." not in f".{name}" or name.endswith("mod_table") or not p.requires_grad:
            continue
        sq = torch.linalg.vector_norm(p.detach(), dtype=torch.float32).square()
        if prefix == "te":
            rows = [WRMS_KEYS.index("te_refiner")]
        else:
            kind = next((k for k in WRMS_KINDS if name.endswith(f"{k}.weight")), None)
            rows = [WRMS_KEYS.index(f"den_{kind}")] if kind else []
        for r in rows + [WRMS_KEYS.index("hidden")]:
            acc[r, 0] += sq
            acc[r, 1] += p.numel()
    return acc


def wrms_stats(acc):
    acc = acc.cpu()
    return {f"weights/rms_{k}": (acc[i, 0] / acc[i, 1]).sqrt().item() for i, k in enumerate(WRMS_KEYS)
            if acc[i, 1] > 0}


@torch.no_grad()
def grad_sq_norms(grads, n, bucket=64 * 2 ** 20, group=None):
    """(mean over workers of |local grad|^2, |mean grad|^2) with one bucketed bf16 all-reduce."""
    small = torch.stack(torch._foreach_norm(grads)).float().square().sum()
    dist.all_reduce(small, group=group)
    big = torch.zeros((), device=small.device)
    chunk, size = [], 0
    for i, g in enumerate(grads):
        chunk.append(g)
        size += g.numel()
        if size >= bucket or i == len(grads) - 1:
            flat = torch.cat([c.flatten() for c in chunk]).bfloat16()
            dist.all_reduce(flat, group=group)
            big += (flat.float() / n).square().sum()
            chunk, size = [], 0
    return small / n, big


def noise_scale(small_sq, big_sq, b_small, b_big):
    """Unbiased |G|^2 and tr(Sigma) from gradient norms at two batch sizes; B_noise = tr(Sigma) / |G|^2."""
    g2 = (b_big * big_sq - b_small * small_sq) / (b_big - b_small)
    s = (small_sq - big_sq) / (1 / b_small - 1 / b_big)
    return g2, s
