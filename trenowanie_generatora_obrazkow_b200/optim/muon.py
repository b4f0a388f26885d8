"""Muon for 2D hidden matrices: momentum, Nesterov direction, decoupled weight decay, batched Newton-Schulz per
shape bucket, shape scale sqrt(max(1, rows / cols)).

Semantics follow the reference optimizer (aurora/muon.py:89-194):
  * momentum ``buf.lerp_(g, 1 - mu)``; direction ``g.lerp(buf, mu)`` (Nesterov) or ``buf``;
  * ``p *= 1 - lr * wd``; ``p -= lr * scale * NS5(direction)``;
  * CMuon ``splits`` (row blocks of fused matrices orthogonalised separately, keeping the fused shape scale);
  * periodic row-wise Muon (``period``, ``gamma``);
  * bf16 momentum with stochastic rounding (``momentum_dtype=torch.bfloat16``).

Distribution: with ``shard=True`` under torch.distributed, every shape bucket is split into contiguous per-rank
slices; each rank orthogonalises its slice and the bf16 updates are gathered (``gather`` hook: NCCL
all_gather_into_tensor by default; parallel/muon_comm.py supplies the fused peer-memory path). ``shard=False``
orthogonalises everything locally (DiLoCo, where replicas differ).
"""
import math

import torch
import torch.distributed as dist

from .newton_schulz import rownorm, zeropower


def stochastic_round_bf16(x, generator=None):
    """fp32 -> bf16, rounding up or down with probability proportional to the distance (unbiased): uniform noise
    on the 16 dropped mantissa bits, then truncation."""
    bits = x.contiguous().view(torch.int32)
    noise = torch.randint(0, 1 << 16, bits.shape, dtype=torch.int32, device=x.device, generator=generator)
    return ((bits + noise) & -65536).view(torch.float32).to(torch.bfloat16)


def default_gather(out, local, group=None):
    """All-gather of equal bf16 slices (NCCL; Gloo gathers through host memory)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        world = dist.get_world_size(group)
        parts = [torch.empty_like(local, device="cpu") for _ in range(world)]
        dist.all_gather(parts, local.cpu(), group=group)
        out.copy_(torch.cat(parts).to(out.device))


class Muon(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-2, momentum=0.95, nesterov=True, ns_steps=5, weight_decay=0.0, shard=True,
                 splits=None, period=1, gamma=0.15, momentum_dtype=None, group=None, gather=None, chunk_elems=None):
        self.momentum_dtype = momentum_dtype
        self.chunk_elems = chunk_elems or 64 * 2 ** 20
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                                      weight_decay=weight_decay))
        distributed = shard and dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        self.gather = gather or default_gather
        self.period, self.gamma, self._t = period, gamma, 0
        splits = splits or {}
        self._buckets = []
        for g in self.param_groups:
            by_shape = {}
            for p in g["params"]:
                assert p.ndim == 2, "Muon is only for 2D weight matrices"
                rows, cols = p.shape
                scale = max(1.0, rows / cols) ** 0.5
                sizes = splits.get(p, [rows])
                assert sum(sizes) == rows, (p.shape, sizes)
                r0 = 0
                for n in sizes:
                    by_shape.setdefault((n, cols), []).append((p, r0, r0 + n, scale))
                    r0 += n
            self._buckets.append(list(by_shape.values()))

    def load_state_dict(self, state_dict):
        """Keep the momentum in ``momentum_dtype`` (torch would cast it to the parameter's dtype)."""
        super().load_state_dict(state_dict)
        if self.momentum_dtype is not None:
            for st in self.state.values():
                if "momentum_buffer" in st:
                    st["momentum_buffer"] = st["momentum_buffer"].to(self.momentum_dtype)

    def _ns(self, X, steps):
        return zeropower(X, steps)

    @torch.no_grad()
    def step(self):
        refresh = self._t % self.period == 0
        self._t += 1
        for group, buckets in zip(self.param_groups, self._buckets):
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            ps = [p for p in group["params"]]
            grads = [p.grad for p in ps]
            assert all(g is not None for g in grads), "Muon expects a gradient for every matrix"
            for p in ps:
                if "momentum_buffer" not in self.state[p]:
                    self.state[p]["momentum_buffer"] = torch.zeros_like(p, dtype=self.momentum_dtype or p.dtype)
            bufs = [self.state[p]["momentum_buffer"] for p in ps]
            if all(b.dtype == g.dtype for b, g in zip(bufs, grads)):
                torch._foreach_lerp_(bufs, grads, 1 - mom)
            else:  # bf16 momentum: EMA step in fp32, stored with stochastic rounding
                for b, g in zip(bufs, grads):
                    b.copy_(stochastic_round_bf16(b.float().lerp(g.float(), 1 - mom)))
            if wd:
                torch._foreach_mul_(ps, 1 - lr * wd)
            for entries in buckets:
                rows, cols = entries[0][2] - entries[0][1], entries[0][0].shape[1]

                def direction(i):
                    p, r0, r1, _ = entries[i]
                    buf = self.state[p]["momentum_buffer"][r0:r1]
                    g = p.grad[r0:r1]
                    return g.lerp(buf.to(g.dtype), mom) if group["nesterov"] else buf

                if self.world == 1:
                    step_n = max(1, self.chunk_elems // (rows * cols))
                    for c0 in range(0, len(entries), step_n):
                        idx = range(c0, min(len(entries), c0 + step_n))
                        X = torch.stack([direction(i) for i in idx])
                        X = self._ns(X, group["ns_steps"]) if refresh else rownorm(X) * self.gamma
                        for j, i in enumerate(idx):
                            p, r0, r1, s = entries[i]
                            p[r0:r1].add_(X[j].float(), alpha=-lr * s)
                        del X
                    continue
                if refresh:
                    per = math.ceil(len(entries) / self.world)
                    lo, hi = min(len(entries), self.rank * per), min(len(entries), (self.rank + 1) * per)
                    local = torch.zeros(per, rows, cols, dtype=torch.bfloat16, device=entries[0][0].device)
                    if hi > lo:
                        local[: hi - lo] = self._ns(torch.stack([direction(i) for i in range(lo, hi)]),
                                                    group["ns_steps"])
                    out = torch.empty(self.world * per, rows, cols, dtype=torch.bfloat16, device=local.device)
                    self.gather(out, local, self.group)
                    out = out[: len(entries)]
                else:
                    out = rownorm(torch.stack([direction(i) for i in range(len(entries))])) * self.gamma
                updates = list(out.float().unbind(0))
                torch._foreach_mul_(updates, [e[3] for e in entries])
                torch._foreach_add_([p[r0:r1] for p, r0, r1, _ in entries], updates, alpha=-lr)


def muon_splits(named):
    """CMuon row blocks of the fused matrices: {param: [sizes]} from (prefix, name, param) triples
    (qkv -> q, k, v; cross kv -> k, v; SwiGLU in_proj -> gate, up)."""
    out = {}
    for _, name, p in named:
        if p.ndim != 2:
            continue
        rows, cols = p.shape
        if name.endswith("attn.qkv.weight") and (rows - cols) > 0 and (rows - cols) % 2 == 0:
            out[p] = [cols, (rows - cols) // 2, (rows - cols) // 2]
        elif name.endswith(("cross.kv.weight", "mlp.in_proj.weight")) and rows % 2 == 0:
            out[p] = [rows // 2, rows // 2]
    return out
