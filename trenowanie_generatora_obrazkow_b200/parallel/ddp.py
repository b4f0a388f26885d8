"""Data-parallel gradient reduction with flat gradient buckets.

Reference: DDP with 64 MB buckets, ``gradient_as_bucket_view`` and the bf16 compress hook (train.py:774-791):
gradients are cast to bf16, all-reduced, divided by the world size and written back in fp32.

Here every trainable parameter's ``.grad`` is a view into one of a few flat fp32 bucket buffers allocated once
(the fused Linear backward accumulates weight gradients into them directly). Buckets are ordered by reverse
registration order, i.e. roughly the order backward produces them, and each bucket is reduced as soon as its last
gradient has been accumulated on the last micro-batch, on a side stream, so the reduction overlaps the rest of the
backward pass. The transport is pluggable: ``nccl_bf16`` (cast + NCCL all_reduce + scale, the reference's hook),
``nccl_fp32``, or ``p2p``: the fused peer-memory kernel of parallel/comm.py (one launch per bucket does the bf16
cast, the reduce-scatter over NVLink loads, the scaled all-gather over NVLink stores and the cast back).
"""
import torch
import torch.distributed as dist

from ..ops import fused as Fz


class GradBuckets:
    def __init__(self, params, bucket_bytes=256 * 2 ** 20, group=None, comm="nccl_bf16", overlap=True, reducer=None):
        """``reducer(bucket_index, flat_fp32)`` replaces the all-reduce (e.g. the sharded-Muon reduce-scatter)."""
        self.params = [p for p in params if p.requires_grad]
        self.reducer = reducer
        self.group = group
        # comm "none": local gradients only (DiLoCo inner steps)
        self.world = dist.get_world_size(group) if (dist.is_initialized() and comm != "none") else 1
        self.comm = comm
        self.overlap = overlap and self.world > 1
        dev = self.params[0].device
        # buckets in reverse order (backward produces the last layers' gradients first)
        order = list(reversed(self.params))
        self.buckets, cur, size = [], [], 0
        for p in order:
            cur.append(p)
            size += p.numel() * 4
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.p2p = None
        if comm == "p2p" and self.world > 1:
            from .comm import PeerAllReduce
            self.p2p = PeerAllReduce(max(sum(p.numel() for p in ps) for ps in self.buckets), group=group, device=dev)
        self.flat = []
        self.bucket_of = {}
        for bi, ps in enumerate(self.buckets):
            n = sum(p.numel() for p in ps)
            buf = torch.zeros(n, dtype=torch.float32, device=dev)
            off = 0
            for p in ps:
                p.grad = buf[off:off + p.numel()].view_as(p)
                self.bucket_of[p] = bi
                off += p.numel()
            self.flat.append(buf)
        self.pending = [0] * len(self.buckets)
        self.next_launch = len(self.buckets)
        self.armed = False
        self.stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" and self.overlap else None
        self.events = []
        self._handles = []
        if self.overlap:
            Fz.add_grad_ready_hook(self._on_ready)
            for p in self.params:
                self._handles.append(p.register_post_accumulate_grad_hook(self._on_ready))

    def close(self):
        if self.p2p is not None:
            self.p2p.close()
            self.p2p = None
        Fz.remove_grad_ready_hook(self._on_ready)
        for h in self._handles:
            h.remove()

    def zero(self):
        for b in self.flat:
            b.zero_()
        # autograd may have replaced a .grad it could not accumulate into in place: re-point at the buckets
        for bi, ps in enumerate(self.buckets):
            off = 0
            for p in ps:
                view = self.flat[bi][off:off + p.numel()].view_as(p)
                if p.grad is None or p.grad.data_ptr() != view.data_ptr():
                    p.grad = view
                off += p.numel()

    def arm(self):
        """Call before the backward of the last micro-batch: buckets reduce as their gradients complete."""
        self.pending = [len(ps) for ps in self.buckets]
        self.next_launch = 0
        self.armed = True
        self.events = []

    def _on_ready(self, p):
        if not self.armed:
            return
        bi = self.bucket_of.get(p)
        if bi is None:
            return
        self.pending[bi] -= 1
        # launch in bucket order, so every rank issues its collectives (or peer-memory launches) in the same order
        while self.next_launch < len(self.buckets) and self.pending[self.next_launch] == 0:
            self._launch(self.next_launch)
            self.next_launch += 1

    def _launch(self, bi):
        buf = self.flat[bi]
        if self.stream is not None:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ev)
                self._reduce(buf, bi)
                done = torch.cuda.Event()
                done.record()
            self.events.append(done)
        else:
            self._reduce(buf, bi)

    def _reduce(self, buf, bi):
        if self.world == 1:
            return
        if self.reducer is not None:
            self.reducer(bi, buf)
            return
        if self.p2p is not None:  # fused cast + reduce-scatter + all-gather over NVLink peer memory
            self.p2p(buf)
        elif self.comm == "nccl_fp32":
            dist.all_reduce(buf, group=self.group)
            buf.div_(self.world)
        else:
            lo = buf.to(torch.bfloat16)
            dist.all_reduce(lo, group=self.group)
            buf.copy_(lo).div_(self.world)

    def finish(self):
        """Wait for the reductions (reduce any bucket that did not fire) before the optimizer reads the grads."""
        if self.world == 1:
            self.armed = False
            return
        if self.overlap:
            while self.next_launch < len(self.buckets):  # buckets with a parameter that got no gradient this step
                self.pending[self.next_launch] = 0
                self._launch(self.next_launch)
                self.next_launch += 1
            if self.stream is not None:
                cur = torch.cuda.current_stream()
                for ev in self.events:
                    cur.wait_event(ev)
        else:
            for bi, buf in enumerate(self.flat):
                self._reduce(buf, bi)
        self.armed = False
