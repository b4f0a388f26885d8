"""Muon for 2-D hidden matrices, built on one flat Muon space that the owner-sharded path (parallel/muon_comm.py)
shares.

Update rule (the published Muon recipe, with the reference optimizer's options, aurora/muon.py:89-194):
  momentum  m <- lerp(m, g, 1 - mu)                   (fp32, or bf16 stored with stochastic rounding)
  direction d  = lerp(g, m, mu)  (Nesterov)  or  m
  p <- p (1 - lr wd) - lr s NS5(d),  s = sqrt(max(1, rows / cols))
with CMuon ``splits`` (row blocks of fused matrices orthogonalised separately, keeping the fused matrix's shape
scale) and periodic row-wise steps (``period``, ``gamma``: every step not divisible by ``period`` uses a row
normalisation instead of Newton-Schulz).

Layout (``MuonLayout``): every row block ("entry") of every Muon matrix is a slot of a flat, bucket-major space:
entries of one (param group, rows, cols) bucket are consecutive, so a bucket's Newton-Schulz input is a contiguous
[k, rows, cols] view, never a stacked copy. Entry i of a bucket is owned by rank i // ceil(len / world).

The optimizer is the single-owner case of that design:
  * one fused launch (``muon_seg_momentum``) reads every gradient in place through a segment table, updates the
    flat momentum and writes the bf16 Newton-Schulz input;
  * Newton-Schulz runs per bucket on the owned entries (tcgen05 GEMMs) into a flat bf16 update buffer;
  * with ``shard=True`` on W > 1 ranks (gradients already all-reduced), each bucket's updates are all-gathered in
    place (its span is padded to W x ceil(len / W) entries, so rank r's entries are exactly its chunk);
  * one fused launch (``muon_apply``) applies decay and update to every fp32 master and refreshes its bf16 shadow.
CPU tensors run the same flow with torch ops (tests). The full momentum lives in this flat buffer on every rank
(``state_dict`` materialises per-parameter ``momentum_buffer`` tensors, so checkpoints keep the usual layout);
the peer-memory sharded path keeps only the owners' momentum and exports / imports it through this buffer.
"""
import math
from dataclasses import dataclass

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
    """All-gather of equal bf16 chunks into `out` (NCCL in place; Gloo through host memory)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
        return
    parts = [torch.empty_like(local, device="cpu") for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, local.cpu(), group=group)
    out.copy_(torch.cat(parts).to(out.device))


@dataclass
class MuonEntry:
    p: torch.Tensor
    r0: int
    r1: int
    scale: float     # shape scale of the whole (fused) matrix
    group: int       # param group index
    bucket: int
    slot: int        # index within the bucket
    off: int         # first element in the flat Muon space
    n: int
    owner: int


@dataclass
class MuonBucket:
    group: int
    rows: int
    cols: int
    entries: list    # entry indices, in slot order
    off: int         # flat offset of slot 0
    per: int         # entries per rank (ceil(len / world))
    span: int        # flat elements reserved for the bucket (padded to world * per slots when padding)

    def owned_slots(self, rank):
        return rank * self.per, min(len(self.entries), (rank + 1) * self.per)


class MuonLayout:
    """Entries and shape buckets of the Muon matrices of `param_groups` in one flat space (module docstring)."""

    def __init__(self, param_groups, splits=None, world=1, rank=0, pad=False):
        splits = splits or {}
        self.world, self.rank = world, rank
        self.entries, self.buckets = [], []
        off = 0
        for gi, g in enumerate(param_groups):
            keyed = {}
            for p in g["params"]:
                if p.ndim != 2:
                    raise ValueError(f"Muon orthogonalises 2-D matrices only, got a tensor of shape {tuple(p.shape)}")
                rows, cols = p.shape
                scale = math.sqrt(max(1.0, rows / cols))
                blocks = splits.get(p, [rows])
                if sum(blocks) != rows:
                    raise ValueError(f"row splits {blocks} do not cover a {tuple(p.shape)} matrix")
                r0 = 0
                for n in blocks:
                    keyed.setdefault((n, cols), []).append((p, r0, r0 + n, scale))
                    r0 += n
            for (rows, cols), members in keyed.items():
                per = math.ceil(len(members) / world)
                b = MuonBucket(gi, rows, cols, [], off, per, 0)
                for slot, (p, r0, r1, scale) in enumerate(members):
                    e = MuonEntry(p, r0, r1, scale, gi, len(self.buckets), slot, off + slot * rows * cols,
                                  rows * cols, slot // per)
                    b.entries.append(len(self.entries))
                    self.entries.append(e)
                b.span = (world * per if pad else len(members)) * rows * cols
                off += b.span
                self.buckets.append(b)
        self.total = off

    def bucket_entries(self, b):
        return [self.entries[i] for i in b.entries]


class Muon(torch.optim.Optimizer):
    """Muon over the flat layout (module docstring). ``gather`` replaces the update all-gather (default: NCCL in
    place); ``chunk_elems`` bounds the Newton-Schulz working set per launch sequence."""

    def __init__(self, params, lr=1e-2, momentum=0.95, nesterov=True, ns_steps=5, weight_decay=0.0, shard=True,
                 splits=None, period=1, gamma=0.15, momentum_dtype=None, group=None, gather=None, chunk_elems=None):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                                      weight_decay=weight_decay))
        distributed = shard and dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        self.momentum_dtype = momentum_dtype
        self.gather = gather or default_gather
        self.chunk_elems = chunk_elems or 512 * 2 ** 20
        self.period, self.gamma, self._t = period, gamma, 0
        self.splits = splits or {}
        self.layout = MuonLayout(self.param_groups, self.splits, self.world, self.rank, pad=self.world > 1)
        self._momentum = None  # flat momentum, allocated on first use
        self._x = None       # flat Newton-Schulz input (bf16), allocated on first step
        self._upd = None     # flat updates (bf16)
        self._tables = {}    # cached device segment tables, keyed by the pointers they hold
        self._steps = 0

    @property
    def momentum(self):
        if self._momentum is None:
            self._momentum = torch.zeros(self.layout.total, dtype=self.momentum_dtype or torch.float32,
                                         device=self.layout.entries[0].p.device)
        return self._momentum

    # ---------------------------------------------------------------------------------------------------------
    # checkpoints: per-parameter momentum buffers <-> the flat momentum
    # ---------------------------------------------------------------------------------------------------------
    def _momentum_view(self, e):
        return self.momentum[e.off:e.off + e.n].view(e.r1 - e.r0, -1)

    @torch.no_grad()
    def momentum_buffer(self, p):
        """The momentum of parameter p assembled from its entries (a copy)."""
        out = torch.zeros_like(p, dtype=self.momentum.dtype)
        for e in self.layout.entries:
            if e.p is p:
                out[e.r0:e.r1] = self._momentum_view(e)
        return out

    @torch.no_grad()
    def state_dict(self):
        for e in self.layout.entries:
            st = self.state[e.p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(e.p, dtype=self.momentum.dtype)
            st["momentum_buffer"][e.r0:e.r1] = self._momentum_view(e)
        sd = super().state_dict()
        sd["state"] = {k: dict(v) for k, v in sd["state"].items()}  # packed dicts are the live ones: detach them
        for e in self.layout.entries:  # the flat buffer stays the only live copy
            self.state[e.p].pop("momentum_buffer", None)
        return sd

    @torch.no_grad()
    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        bufs = {}
        for e in self.layout.entries:  # a split matrix has several entries: take its buffer once, use it for all
            if id(e.p) not in bufs:
                bufs[id(e.p)] = self.state.get(e.p, {}).pop("momentum_buffer", None)
            buf = bufs[id(e.p)]
            if buf is not None:
                self._momentum_view(e).copy_(buf[e.r0:e.r1])

    # ---------------------------------------------------------------------------------------------------------
    # step
    # ---------------------------------------------------------------------------------------------------------
    def _device_path(self):
        return self.momentum.is_cuda and all(
            e.p.grad is not None and e.p.grad.dtype == torch.float32 and e.p.grad.is_contiguous()
            and e.p.dtype == torch.float32 for e in self.layout.entries)

    def _table(self, key, rows, dtype=torch.int64):
        """Device copy of a small host table, re-uploaded only when its contents change."""
        t = self._tables.get(key)
        if t is None or t[0] != rows:
            t = (rows, torch.tensor(rows, dtype=dtype).reshape(-1, len(rows[0]) if rows else 1)
                 .to(self.momentum.device))
            self._tables[key] = t
        return t[1]

    def _grad_rows(self, gi):
        return [(e.p.grad.data_ptr() + e.r0 * e.p.shape[1] * 4, e.off, e.n)
                for e in self.layout.entries if e.group == gi]

    def _apply_rows(self, ema):
        from ..ops.fused import bf16_weight
        rows = []
        for e in self.layout.entries:
            cols = e.p.shape[1]
            ev = ema.lookup(e.p) if ema is not None else None
            rows.append((e.p.data_ptr() + e.r0 * cols * 4, bf16_weight(e.p).data_ptr() + e.r0 * cols * 2, e.off, e.n,
                         0 if ev is None else ev.data_ptr() + e.r0 * cols * 4))
        return rows

    def _momentum_torch(self, gi, g, coef=1.0):
        """CPU / fallback path of the fused momentum kernel for param group gi."""
        mu, nesterov = g["momentum"], g["nesterov"]
        for e in self.layout.entries:
            if e.group != gi:
                continue
            grad = e.p.grad[e.r0:e.r1].reshape(-1).float() * coef
            m = self.momentum[e.off:e.off + e.n]
            if m.dtype == torch.float32:
                m.lerp_(grad, 1 - mu)
                mq = m
            else:
                m.copy_(stochastic_round_bf16(m.float().lerp(grad, 1 - mu)))
                mq = m.float()
            self._x[e.off:e.off + e.n] = (grad.lerp(mq, mu) if nesterov else mq).to(torch.bfloat16)

    @torch.no_grad()
    def step(self, closure=None, coef=None, ema=None, ema_rate=0.0, timer=None):
        """One Muon step. ``coef`` (float or device scalar) scales the gradients first (the clip coefficient);
        ``ema`` (optim.groups.EMA): its tensors of these matrices get e += ema_rate (p - e) after the update, in the
        same launch on the device (and are marked done for this step)."""
        if closure is not None:
            with torch.enable_grad():
                closure()
        for e in self.layout.entries:
            if e.p.grad is None:
                raise RuntimeError("Muon needs a gradient for every matrix it optimises")
        refresh = self._t % self.period == 0
        self._t += 1
        self._steps += 1
        L = self.layout
        dev = self.momentum.device
        if self._x is None:
            self._x = torch.zeros(L.total, dtype=torch.bfloat16, device=dev)
            self._upd = torch.zeros(L.total, dtype=torch.bfloat16, device=dev)
        fused = self._device_path()
        if fused:
            from ..ops._ext import ext
            coef_t = coef.reshape(1).float() if torch.is_tensor(coef) else \
                torch.full((1,), 1.0 if coef is None else float(coef), device=dev)
            blocks = 148 * 4
            for gi, g in enumerate(self.param_groups):
                rows = self._grad_rows(gi)
                if rows:
                    seed = (self._steps * 0x9E3779B1 + gi * 0x85EBCA77) & 0x7FFFFFFFFFFFFFFF
                    ext().muon_seg_momentum(self._table(("grad", gi), rows), self.momentum, self._x, coef_t,
                                            g["momentum"], bool(g["nesterov"]), seed, blocks)
        else:
            for gi, g in enumerate(self.param_groups):
                self._momentum_torch(gi, g, 1.0 if coef is None else coef)

        if timer is not None:
            timer.mark("muon_momentum")
        # Newton-Schulz (or the row-wise step) of the owned entries of every bucket, into the update buffer
        for b in L.buckets:
            lo, hi = b.owned_slots(self.rank)
            size = b.rows * b.cols
            per_launch = max(1, self.chunk_elems // size)
            steps = self.param_groups[b.group]["ns_steps"]
            for s0 in range(lo, hi, per_launch):
                s1 = min(hi, s0 + per_launch)
                a, z = b.off + s0 * size, b.off + s1 * size
                X = self._x[a:z].view(s1 - s0, b.rows, b.cols)
                if refresh:  # the flat input is scratch: normalised in place, result straight into the updates
                    zeropower(X, steps, out=self._upd[a:z].view(s1 - s0, b.rows, b.cols), scratch_ok=True)
                else:
                    self._upd[a:z].copy_((rownorm(X) * self.gamma).reshape(-1))
            if self.world > 1:  # in place: rank r's owned slots are chunk r of the bucket's padded span
                span = self._upd[b.off:b.off + b.span]
                chunk = b.per * size
                self.gather(span, span[self.rank * chunk:(self.rank + 1) * chunk], self.group)

        if timer is not None:
            timer.mark("muon_newton_schulz")  # with W > 1: and the update all-gather
        # p <- p (1 - lr wd) - lr s U, and the bf16 shadow
        coefs = [(-self.param_groups[e.group]["lr"] * e.scale,
                  1 - self.param_groups[e.group]["lr"] * self.param_groups[e.group]["weight_decay"])
                 for e in L.entries]
        if fused:  # raw-pointer writes: the parameters' versions stay, so their bf16 shadows stay valid
            from ..ops._ext import ext
            from .adamw import after_raw_update
            ext().muon_apply(self._upd, self._table("apply", self._apply_rows(ema)),
                             self._table("coefs", coefs, torch.float32), float(ema_rate), 148 * 4)
            after_raw_update(e.p for e in L.entries)
        else:
            for e, (alpha, decay) in zip(L.entries, coefs):
                blk = e.p[e.r0:e.r1]  # a view: the in-place update bumps the parameter's version
                blk.mul_(decay).add_(self._upd[e.off:e.off + e.n].view_as(blk).float(), alpha=alpha)
        if timer is not None:
            timer.mark("muon_apply")
        if ema is not None:
            done = set()
            for e in L.entries:
                ev = ema.lookup(e.p)
                if ev is None or id(e.p) in done:
                    continue
                if not fused:
                    ev.lerp_(e.p.detach().float(), ema_rate)
                ema.mark_fused(e.p)
                done.add(id(e.p))


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
