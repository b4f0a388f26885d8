"""PowerSGD gradient compression for the data-parallel reduction (Vogels et al. 2019; the reference enables
torch's DDP powerSGD hook with --grad-comm powersgd, train.py:780-791).

For every gradient matrix M (rows x cols, both larger than the rank r) of a bucket, one power-iteration step per
optimizer step with error feedback:
    M <- M + E                      (residual of the previous step)
    P = M Q ; all-reduce(P) / W ; P = orthonormalise(P)
    Q = M^T P ; all-reduce(Q) / W
    M_hat = P Q^T ; E = M - M_hat ; M <- M_hat
Q is kept between steps (warm start) and starts from the same seeded Gaussian on every rank. Vectors, small matrices
and every gradient during the first ``start_iter`` steps are averaged uncompressed (fp32). The wire carries
r (rows + cols) values per matrix instead of rows x cols. Used as the ``reducer`` of ``GradBuckets``.
"""
import torch
import torch.distributed as dist


class PowerSGD:
    def __init__(self, buckets, rank=4, start_iter=10, group=None, seed=0):
        self.buckets, self.r, self.start_iter, self.group = buckets, rank, start_iter, group
        self.world = dist.get_world_size(group)
        self.step = 0
        self.err, self.q = {}, {}
        g = torch.Generator().manual_seed(seed + 29)
        for ps in buckets.buckets:
            for p in ps:
                if p.ndim == 2 and min(p.shape) > rank:
                    self.q[p] = torch.randn(p.shape[1], rank, generator=g).to(p.device)

    def next_step(self):
        self.step += 1

    @torch.no_grad()
    def __call__(self, bi, buf):
        ps = self.buckets.buckets[bi]
        if self.step < self.start_iter:
            dist.all_reduce(buf, group=self.group)
            buf.div_(self.world)
            return
        small, mats, off = [], [], 0
        for p in ps:
            n = p.numel()
            view = buf[off:off + n]
            (mats if p in self.q else small).append((p, view))
            off += n
        if small:
            flat = torch.cat([v for _, v in small])
            dist.all_reduce(flat, group=self.group)
            flat.div_(self.world)
            o = 0
            for _, v in small:
                v.copy_(flat[o:o + v.numel()])
                o += v.numel()
        if not mats:
            return
        Ms = []
        for p, v in mats:
            M = v.view(p.shape)
            if p in self.err:
                M.add_(self.err[p])
            Ms.append(M)
        Ps = [M @ self.q[p] for (p, _), M in zip(mats, Ms)]
        flat = torch.cat([P.reshape(-1) for P in Ps])
        dist.all_reduce(flat, group=self.group)
        flat.div_(self.world)
        o = 0
        for i, P in enumerate(Ps):
            Ps[i] = torch.linalg.qr(flat[o:o + P.numel()].view_as(P)).Q
            o += P.numel()
        Qs = [M.mT @ P for M, P in zip(Ms, Ps)]
        flat = torch.cat([Q.reshape(-1) for Q in Qs])
        dist.all_reduce(flat, group=self.group)
        flat.div_(self.world)
        o = 0
        for (p, _), M, P, Q in zip(mats, Ms, Ps, Qs):
            Qr = flat[o:o + Q.numel()].view_as(Q)
            o += Q.numel()
            approx = P @ Qr.mT
            self.err[p] = M - approx
            M.copy_(approx)
            self.q[p] = Qr.clone()
