"""Owner-sharded Muon: gradient reduce-scatter to the owner of each matrix, owner-only momentum and Newton-Schulz,
and the update all-gather fused with the parameter update.

Reference behaviour (aurora/muon.py:89-194, train.py:774-791): DDP all-reduces every gradient (bf16 compress hook),
every rank keeps the full momentum, runs Newton-Schulz on its contiguous slice of each shape bucket and the bf16
updates are all-gathered (``all_gather_into_tensor``). Ownership is the same here (entry i of a bucket belongs to
rank i // ceil(len / world)), and so is the math; the data flow is cut down to what the owners need:

* Muon matrices get their own gradient buckets (``GradBuckets(..., reducer=MuonShardedComm.reduce_bucket)``). As
  soon as a bucket's gradients are complete in the last backward, ``muon_rs`` (csrc/muon_comm.cu) casts it to bf16
  in peer-visible staging and every owner pulls and sums the rows of its matrices from all peers over NVLink into
  an fp32 owned-gradient buffer (plus its sum of squares). The NCCL all-reduce moves 2 (W-1)/W of the bytes; this
  moves (W-1)/W.
* The global gradient norm is the AdamW gradients' norm plus the all-reduced owned sums of squares; the clip
  coefficient is applied inside ``muon_momentum`` (momentum lerp, Nesterov lerp, bf16 Newton-Schulz input; bf16
  momentum with stochastic rounding when requested). Momentum exists only on the owner.
* Newton-Schulz runs batched per shape bucket on the owned slice (tcgen05 GEMMs), the result lands in the owner's
  part of a peer-visible update buffer that spans the whole Muon space.
* ``muon_ag_apply`` pushes every owner's updates into every peer's update buffer and, in the same launch, applies
  ``p = p (1 - lr wd) - lr s U`` to every fp32 master matrix and writes its bf16 shadow (the copy the next forward's
  GEMMs read), so no separate weight cast runs before the next forward.

``transport="torch"`` runs the same data flow with torch.distributed collectives (CPU / Gloo tests, or NCCL
without peer mappings): an all-reduce of the bf16 bucket stands in for the reduce-scatter and an all-reduce of the
zero-padded update buffer for the all-gather.
"""
import math

import torch
import torch.distributed as dist

from ..ops import fused as Fz
from ..optim.muon import stochastic_round_bf16
from ..optim.newton_schulz import rownorm, zeropower


class MuonShardedComm:
    def __init__(self, muon, group=None, device=None, transport="p2p", blocks=32, timeout_s=60.0, ag_blocks=None):
        self.muon, self.group = muon, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world == muon.world, "the optimizer must be built with the same group (shard=True)"
        first = muon.param_groups[0]["params"][0]
        self.device = torch.device(device) if device is not None else first.device
        self.transport = transport if self.device.type == "cuda" else "torch"
        # reduce-scatter: few CTAs (it runs beside the backward's kernels); all-gather + apply: enough CTAs to keep
        # HBM and NVLink busy (it streams every master weight), within the flag array's limit
        self.blocks, self.timeout_ns = blocks, int(timeout_s * 1e9)
        self.ag_blocks = ag_blocks or max(1, min(296, 1024 // max(1, self.world)))
        # ---- the Muon space: the optimizer's layout without padding (same entries, order and owners) ----
        from ..optim.muon import MuonLayout
        self.layout = MuonLayout(muon.param_groups, muon.splits, self.world, self.rank, pad=False)
        self.entries = []       # dict(p, r0, r1, scale, gi, off, n, owner, oown)
        self.bucket_views = []  # (gi, rows, cols, lo, hi, off_lo, own_lo): owned slice of each shape bucket
        own = 0
        for b in self.layout.buckets:
            lo, hi = b.owned_slots(self.rank)
            own_lo = own
            for k in b.entries:
                le = self.layout.entries[k]
                e = dict(p=le.p, r0=le.r0, r1=le.r1, scale=le.scale, gi=le.group, off=le.off, n=le.n,
                         owner=le.owner, oown=None)
                if le.owner == self.rank:
                    e["oown"] = own
                    own += le.n
                self.entries.append(e)
            if hi > lo:
                self.bucket_views.append((b.group, b.rows, b.cols, lo, hi, b.off + lo * b.rows * b.cols, own_lo))
        off = self.layout.total
        self.total, self.owned = off, own
        self.own_ranges = [(v[5], (v[4] - v[3]) * v[1] * v[2]) for v in self.bucket_views]
        # owned elements per param group (contiguous: buckets are laid out group by group)
        self.group_owned = []
        for gi in range(len(muon.param_groups)):
            es = [e for e in self.entries if e["gi"] == gi and e["owner"] == self.rank]
            self.group_owned.append((es[0]["oown"], es[-1]["oown"] + es[-1]["n"]) if es else (0, 0))
        dev = self.device
        self.g_owned = torch.zeros(max(1, self.owned), dtype=torch.float32, device=dev)
        self.x_in = torch.zeros(max(1, self.owned), dtype=torch.bfloat16, device=dev)
        mdt = muon.momentum_dtype or torch.float32
        self.momentum = torch.zeros(max(1, self.owned), dtype=mdt, device=dev)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.step_count = 0
        self.rs_epoch = 0
        self.ag_epoch = 0
        self.bucket_segs = {}
        self.params = [e["p"] for e in self.entries]
        self._peer = None
        if self.transport == "p2p":
            self._init_peer()
        else:
            self.update = torch.zeros(self.total, dtype=torch.bfloat16, device=dev)

    # ------------------------------------------------------------------------------------------------------------
    def _init_peer(self):
        self._peer_sizes = dict(update=self.total * 2,
                                rs_flags=2 * self.world * self.blocks * 4, ag_flags=self.world * self.ag_blocks * 4)

    def attach_buckets(self, buckets):
        """Build the per-bucket segment tables from the gradient buckets of the Muon matrices (``GradBuckets``):
        for every owned entry, (offset in the bucket, offset in the owned-gradient buffer, length)."""
        where = {}
        for bi, ps in enumerate(buckets.buckets):
            o = 0
            for p in ps:
                where[p] = (bi, o)
                o += p.numel()
        segs = {}
        for e in self.entries:
            if e["owner"] != self.rank:
                continue
            bi, o = where[e["p"]]
            cols = e["p"].shape[1]
            segs.setdefault(bi, []).append((o + e["r0"] * cols, e["oown"], e["n"]))
        self.bucket_segs = {}
        for bi in range(len(buckets.buckets)):
            s = sorted(segs.get(bi, []))
            t = torch.tensor(s if s else [[0, 0, 0]], dtype=torch.int64).reshape(-1, 3)
            owned = sum(x[2] for x in s)
            if self.transport == "p2p":
                t = t.to(self.device)
            self.bucket_segs[bi] = (t if s else t[:0], owned)
        if self.transport == "p2p" and self._peer is None:
            from .comm import PeerBuffers
            stage = max(buf.numel() for buf in buckets.flat)
            sizes = dict(self._peer_sizes, staging=stage * 2)
            self._peer = PeerBuffers(sizes, self.group, self.device)
            self.update = None
            self._build_apply_tables()
        return self

    def _apply_rows(self, ema=None):
        """(fp32 master, bf16 shadow, offset, length, EMA) rows of every entry. ``bf16_weight`` re-creates a shadow
        whose master was changed by torch in place (load_state_dict, DiLoCo outer step), so the rows are rebuilt
        and compared every step."""
        rows = []
        for e in self.entries:
            cols = e["p"].shape[1]
            ev = ema.lookup(e["p"]) if ema is not None else None
            rows.append((e["p"].data_ptr() + e["r0"] * cols * 4, Fz.bf16_weight(e["p"]).data_ptr() + e["r0"] * cols * 2,
                         e["off"], e["n"], 0 if ev is None else ev.data_ptr() + e["r0"] * cols * 4))
        return rows

    def _build_apply_tables(self, ema=None):
        self._rows = self._apply_rows(ema)
        self.apply_segs = torch.tensor(self._rows, dtype=torch.int64, device=self.device).reshape(-1, 5)
        self.own_t = torch.tensor(self.own_ranges if self.own_ranges else [[0, 0]], dtype=torch.int64,
                                  device=self.device).reshape(-1, 2)
        if not self.own_ranges:
            self.own_t = self.own_t[:0]
        self.coefs = torch.zeros(len(self.entries), 2, dtype=torch.float32, device=self.device)

    def close(self):
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    # ------------------------------------------------------------------------------------------------------------
    # reduce-scatter (called per gradient bucket by GradBuckets, on its reduction stream)
    # ------------------------------------------------------------------------------------------------------------
    def begin_step(self):
        self.sumsq.zero_()

    def reduce_bucket(self, bi, buf):
        segs, owned = self.bucket_segs[bi]
        if self.transport == "p2p":
            from ..ops._ext import err_buf, ext
            prev = self.rs_epoch
            self.rs_epoch = (self.rs_epoch + 1) & 0xFFFFFFFF or 1
            pp = self._peer.ptrs
            ext().muon_rs(buf, pp["staging"], pp["rs_flags"], segs, owned, self.g_owned, self.sumsq, self.rank,
                          self.world, self.rs_epoch, prev, self.blocks, self.timeout_ns, err_buf(buf.device))
            return
        lo = buf.to(torch.bfloat16)
        dist.all_reduce(lo, group=self.group)
        red = lo.float().div_(self.world)
        for src, dst, n in segs.tolist():
            v = red[src:src + n]
            self.g_owned[dst:dst + n] = v
            self.sumsq += v.square().sum()

    def owned_sumsq(self):
        """Sum over ranks of the owned reduced gradients' squares (the Muon part of the global gradient norm)."""
        s = self.sumsq.clone()
        dist.all_reduce(s, group=self.group)
        return s

    # ------------------------------------------------------------------------------------------------------------
    # optimizer step
    # ------------------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def step(self, coef=1.0, ema=None, ema_rate=0.0, timer=None):
        """One Muon step from the owned reduced gradients; ``coef`` is the gradient-clip coefficient (float or
        device scalar); ``ema`` (optim.groups.EMA, where this rank keeps one): updated inside the apply launch."""
        m = self.muon
        refresh = m._t % m.period == 0
        m._t += 1
        self.step_count += 1
        coef_t = (coef.reshape(1).float() if torch.is_tensor(coef) else torch.tensor([float(coef)])).to(self.device)
        for gi, g in enumerate(m.param_groups):
            a, b = self.group_owned[gi]
            if b <= a:
                continue
            self._momentum(self.g_owned[a:b], self.momentum[a:b], self.x_in[a:b], coef_t, g["momentum"],
                           g["nesterov"])
        if timer is not None:
            timer.mark("muon_momentum")
        upd_local = self._local_update_view()
        for gi, rows, cols, lo, hi, off_lo, own_lo in self.bucket_views:
            n = (hi - lo) * rows * cols
            X = self.x_in[own_lo:own_lo + n].view(hi - lo, rows, cols)
            steps = m.param_groups[gi]["ns_steps"]
            dst = upd_local[off_lo:off_lo + n].view(hi - lo, rows, cols)
            if refresh:  # x_in is scratch: normalised in place, the result lands in the peer-visible update buffer
                zeropower(X, steps, out=dst, scratch_ok=True)
            else:
                dst.copy_(rownorm(X) * m.gamma)
        if timer is not None:
            timer.mark("muon_newton_schulz")
        self._gather_apply(ema, ema_rate)
        if timer is not None:
            timer.mark("muon_allgather_apply")

    def _momentum(self, g, buf, x, coef, mu, nesterov):
        if self.transport == "p2p":
            from ..ops._ext import ext
            seed = (self.step_count * 0x9E3779B1 + self.rank * 0x85EBCA77) & 0x7FFFFFFFFFFFFFFF
            ext().muon_momentum(g, buf, x, coef, mu, bool(nesterov), seed)
            return
        gs = g * coef.to(g.device)
        if buf.dtype == torch.float32:
            buf.lerp_(gs, 1 - mu)
            mq = buf
        else:
            buf.copy_(stochastic_round_bf16(buf.float().lerp(gs, 1 - mu)))
            mq = buf.float()
        x.copy_(gs.lerp(mq, mu) if nesterov else mq)

    def _local_update_view(self):
        if self.transport == "p2p":
            ptr = self._peer.local["update"]
            return _wrap_bf16(ptr, self.total, self.device)
        self.update.zero_()
        return self.update

    def _gather_apply(self, ema=None, ema_rate=0.0):
        m = self.muon
        coefs = []
        for e in self.entries:
            g = m.param_groups[e["gi"]]
            coefs.append([-g["lr"] * e["scale"], 1 - g["lr"] * g["weight_decay"]])
        if self.transport == "p2p":
            from ..ops._ext import err_buf, ext
            if self._apply_rows(ema) != self._rows:
                self._build_apply_tables(ema)
            self.coefs.copy_(torch.tensor(coefs, dtype=torch.float32), non_blocking=False)
            self.ag_epoch = (self.ag_epoch + 1) & 0xFFFFFFFF or 1
            pp = self._peer.ptrs
            ext().muon_ag_apply(pp["update"], pp["ag_flags"], self.own_t, self.owned, self.apply_segs, self.coefs,
                                float(ema_rate), self.rank, self.world, self.ag_epoch, self.ag_blocks, self.timeout_ns,
                                err_buf(self.device))
            from ..optim.adamw import after_raw_update
            after_raw_update(e["p"] for e in self.entries)
            self._mark_ema(ema)
            return
        dist.all_reduce(self.update, group=self.group)  # every owner contributed its ranges, zeros elsewhere
        U = self.update.float()
        for e, (alpha, decay) in zip(self.entries, coefs):
            blk = e["p"][e["r0"]:e["r1"]]  # a view: the in-place update bumps the parameter's version
            blk.mul_(decay).add_(U[e["off"]:e["off"] + e["n"]].view_as(blk), alpha=alpha)
        if ema is not None:
            for p in {id(e["p"]): e["p"] for e in self.entries}.values():
                ev = ema.lookup(p)
                if ev is not None:
                    ev.lerp_(p.detach().float(), ema_rate)
        self._mark_ema(ema)

    def _mark_ema(self, ema):
        if ema is not None:
            for e in self.entries:
                if ema.lookup(e["p"]) is not None:
                    ema.mark_fused(e["p"])

    # ------------------------------------------------------------------------------------------------------------
    # checkpoints: the optimizer's per-parameter momentum buffers <-> the owners' shards
    # ------------------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def export_momentum(self):
        """Assemble the full momentum (all ranks take part) into the optimizer's flat momentum, from which its
        ``state_dict`` materialises per-parameter buffers."""
        full = torch.zeros(self.total, dtype=torch.float32, device=self.device)
        for e in self.entries:
            if e["owner"] == self.rank:
                full[e["off"]:e["off"] + e["n"]] = self.momentum[e["oown"]:e["oown"] + e["n"]].float()
        dist.all_reduce(full, group=self.group)
        flat = self.muon.momentum
        for e, me in zip(self.entries, self.muon.layout.entries):
            flat[me.off:me.off + me.n] = full[e["off"]:e["off"] + e["n"]].to(flat.dtype)

    @torch.no_grad()
    def import_momentum(self):
        """Take this rank's shards from the optimizer's flat momentum (after its ``load_state_dict``)."""
        flat = self.muon.momentum
        for e, me in zip(self.entries, self.muon.layout.entries):
            if e["owner"] == self.rank:
                self.momentum[e["oown"]:e["oown"] + e["n"]] = flat[me.off:me.off + me.n].to(self.momentum.dtype)


def _wrap_bf16(ptr, n, device):
    """A bf16 tensor view of raw device memory owned elsewhere (the peer-visible update buffer)."""
    from ..ops._ext import ext
    return ext().tensor_from_ptr(ptr, n, device.index)
