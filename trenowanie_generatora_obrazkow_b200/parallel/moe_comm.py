"""Expert-parallel MoE exchange fused with the expert GEMMs over NVLink peer memory (one expert group per GPU).

Per MoE layer and micro-batch, with static capacity C (a multiple of 128) and E = world * local experts:

  forward   dispatch kernel  gathers this rank's token rows slot by slot and stores them straight into each
                             owner's receive buffer [local][world][C][D] (zeros for empty slots), then raises the
                             owner's arrive flag for this source;
            GEMM 1 (owner)   x_recv @ w_in^T: the TMA producer waits for a source's arrive flag before it loads
                             that source's 128-row tiles, so tiles of early sources run while others are in flight;
            SwiGLU           local;
            GEMM 2 (owner)   h @ w_out^T: the epilogue stores every output row into its source's combine buffer
                             [E][C][D] on that GPU and the last tile warp of a source raises its done flag;
            combine kernel   out[t] = sum_k w[t, k] * y[slot(t, k)] once every owner is done.
  backward  the same in reverse: the routing-weighted output gradient is dispatched to the owners, dgrad 2 waits
            for it tile by tile, the weight gradients accumulate in fp32, dgrad 1 scatters dx rows back to the
            sources, and an unweighted combine sums them per token. The router weights' gradient is
            <dout[t], y[slot(t, k)]>. After its weight gradients the owner releases its receive rows to the sources
            (the next forward dispatch of the layer waits for that).

No NCCL call is on this path; every wait is a bounded flag wait (a time-out raises through ``check_errors``).
The receive and combine buffers of a layer are its own (the backward reads them); the backward exchange buffers
are shared by all layers of the same shape, which the layer order makes safe: a source sends a layer's output
gradient only after it combined the previous layer's dx, which its owner scattered after the weight-gradient
GEMM that last read the shared gradient buffer.
"""
import torch
import torch.distributed as dist

from ..ops._ext import err_buf, ext

_ARRIVE_X, _DONE_Y, _FREE, _ARRIVE_DY, _DONE_DX = range(5)


class MoEPeerExchange:
    _shared = {}

    def __init__(self, E, local, C, D, H, group=None, device=None, timeout_s=60.0):
        from .comm import PeerBuffers
        assert C % 128 == 0, "capacity must be a multiple of the 128-row GEMM tile"
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        assert E == local * self.world
        self.E, self.local, self.C, self.D, self.H = E, local, C, D, H
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.timeout_ns = int(timeout_s * 1e9)
        W = self.world
        self.buf = PeerBuffers({"x_recv": local * W * C * D * 2, "y_comb": E * C * D * 2, "flags": 5 * W * 4},
                               group, self.device)
        key = (E, local, C, D, W, id(group))
        if key not in MoEPeerExchange._shared:
            MoEPeerExchange._shared[key] = PeerBuffers({"dy_recv": local * W * C * D * 2,
                                                        "dx_comb": E * C * D * 2}, group, self.device)
        self.shared = MoEPeerExchange._shared[key]
        self.counter = torch.zeros(2 * W, dtype=torch.int32, device=self.device)
        self.fwd_epoch = self.bwd_epoch = 0
        self.blocks = max(1, min(64, (local * C) // 8))

    # ---- addresses
    def _flags(self, kind, peer=None):
        """Flag array `kind` ([world] words) on `peer` (default: this rank)."""
        peer = self.rank if peer is None else peer
        return self.buf.ptrs["flags"][peer] + kind * self.world * 4

    def _flag_word(self, kind, peer, index):
        return self._flags(kind, peer) + index * 4

    def _view(self, ptr, n, shape):
        return ext().tensor_from_ptr(ptr, n, self.device.index).view(*shape)

    def x_recv(self):
        L, W, C, D = self.local, self.world, self.C, self.D
        return self._view(self.buf.local["x_recv"], L * W * C * D, (L, W * C, D))

    def y_comb(self):
        return self._view(self.buf.local["y_comb"], self.E * self.C * self.D, (self.E * self.C, self.D))

    def dy_recv(self):
        L, W, C, D = self.local, self.world, self.C, self.D
        return self._view(self.shared.local["dy_recv"], L * W * C * D, (L, W * C, D))

    # ---- steps
    def dispatch(self, x, src_tok, scale, recv, arrive_kind, epoch, back_pressure):
        W = self.world
        ext().moe_dispatch(x, src_tok, scale, recv, [self._flags(arrive_kind, r) for r in range(W)],
                           self._flags(_FREE) if back_pressure else 0, self.counter, self.E, self.local, self.C,
                           self.rank, epoch, self.timeout_ns, self.blocks, err_buf(x.device))

    def gemm_wait(self, a, b, out, b_mn, arrive_kind, epoch):
        ext().gemm_peer(a, b, out, b_mn, 1, self.C, epoch, self._flags(arrive_kind), [], 0, None, [],
                        self.timeout_ns, err_buf(a.device))

    def gemm_scatter(self, a, b, b_mn, dests, done_kind, epoch):
        W = self.world
        ext().gemm_peer(a, b, None, b_mn, 2, self.C, epoch, 0, dests, self.rank * self.local,
                        self.counter[W:], [self._flag_word(done_kind, s, self.rank) for s in range(W)],
                        self.timeout_ns, err_buf(a.device))

    def combine(self, ybuf_ptr, slot, w, done_kind, epoch, N):
        out = torch.empty(N, self.D, dtype=torch.bfloat16, device=self.device)
        ext().moe_combine(ybuf_ptr, slot, w, self._flags(done_kind), out, self.world, epoch, self.timeout_ns,
                          err_buf(self.device))
        return out

    def release(self, epoch):
        ext().moe_release([self._flags(_FREE, s) for s in range(self.world)], self.rank, epoch)

    def close(self):
        self.buf.close()


def _accumulate_grad(w, fn):
    from ..ops import fused as Fz
    if w.grad is None:
        w.grad = torch.zeros_like(w, dtype=torch.float32)
    fn(w.grad)
    Fz._notify(w)


class _ExchangeExperts(torch.autograd.Function):
    """out [N, D] = sum_k wts[t, k] * expert_{e(t, k)}(x2[t]) with the experts spread over the group."""

    @staticmethod
    def forward(ctx, x2, wts, w_in, w_out, ex, src_tok, slot, slot_w, training):
        ex.fwd_epoch += 1
        e = ex.fwd_epoch
        W = ex.world
        x2 = x2.to(torch.bfloat16).contiguous()
        w_in_b = w_in.detach().to(torch.bfloat16).contiguous()
        w_out_b = w_out.detach().to(torch.bfloat16).contiguous()
        ex.dispatch(x2, src_tok, None, ex.buf.ptrs["x_recv"], _ARRIVE_X, e, back_pressure=True)
        xr = ex.x_recv()
        ab = torch.empty(ex.local, W * ex.C, 2 * ex.H, dtype=torch.bfloat16, device=x2.device)
        ex.gemm_wait(xr, w_in_b, ab, False, _ARRIVE_X, e)
        h = ext().swiglu_fwd(ab)
        ex.gemm_scatter(h, w_out_b, False, ex.buf.ptrs["y_comb"], _DONE_Y, e)
        out = ex.combine(ex.buf.local["y_comb"], slot, wts.detach().float().contiguous(), _DONE_Y, e, x2.shape[0])
        if not training:
            ex.release(e)  # no backward will read the receive rows
        ctx.ex, ctx.epoch, ctx.training = ex, e, training
        ctx.w_in, ctx.w_out = w_in, w_out
        ctx.save_for_backward(ab, w_in_b, w_out_b, src_tok, slot, slot_w)
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops.gemm import gemm
        ex = ctx.ex
        ab, w_in_b, w_out_b, src_tok, slot, slot_w = ctx.saved_tensors
        dout = dout.to(torch.bfloat16).contiguous()
        W = ex.world
        ex.bwd_epoch += 1
        eb = ex.bwd_epoch
        # router weights: d wts[t, k] = <dout[t], y[slot(t, k)]> (y: this layer's combine buffer, still intact)
        keep = slot >= 0
        y = ex.y_comb()
        dw = torch.bmm(y[slot.clamp(min=0).long()], dout.unsqueeze(-1)).squeeze(-1).float() * keep
        # output gradient rows (scaled by the routing weights) -> the owners
        ex.dispatch(dout, src_tok, slot_w, ex.shared.ptrs["dy_recv"], _ARRIVE_DY, eb, back_pressure=False)
        dyr = ex.dy_recv()
        dh = torch.empty(ex.local, W * ex.C, ex.H, dtype=torch.bfloat16, device=dout.device)
        ex.gemm_wait(dyr, w_out_b, dh, True, _ARRIVE_DY, eb)
        h = ext().swiglu_fwd(ab)
        if ctx.w_out.requires_grad:
            _accumulate_grad(ctx.w_out, lambda g: gemm(dyr, h, out=g, a_mn=True, b_mn=True, accumulate=True))
        dab = ext().swiglu_bwd(ab, dh)
        ex.gemm_scatter(dab, w_in_b, True, ex.shared.ptrs["dx_comb"], _DONE_DX, eb)
        if ctx.w_in.requires_grad:
            _accumulate_grad(ctx.w_in, lambda g: gemm(dab, ex.x_recv(), out=g, a_mn=True, b_mn=True,
                                                       accumulate=True))
        ex.release(ctx.epoch)  # the weight gradients were the last readers of the receive rows
        dx2 = ex.combine(ex.shared.local["dx_comb"], slot, None, _DONE_DX, eb, dout.shape[0])
        return dx2, dw, None, None, None, None, None, None, None


def exchange_experts(x2, wts, w_in, w_out, ex, src_tok, slot, slot_w):
    """A backward must follow every forward taken with gradients (it releases the layer's receive rows)."""
    training = torch.is_grad_enabled() and any(t.requires_grad for t in (x2, wts, w_in, w_out))
    return _ExchangeExperts.apply(x2, wts, w_in, w_out, ex, src_tok, slot, slot_w, training)
