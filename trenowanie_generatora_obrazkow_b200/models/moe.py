"""Mixture-of-experts DiT variant: every other block's SwiGLU MLP becomes E experts with top-k token-choice routing,
optionally expert-parallel (one expert group per GPU).

There is no MoE denoiser in the reference (its only MoE is inside the frozen Poziomka LM, aurora/hf_compat.py and
the Triton grouped GEMM aurora/moe_triton.py); this is the benchmark's MoE-DiT configuration built B200-first:

* Routing: router logits in fp32, softmax, top-k, weights renormalised over the k picks; a Switch-style load
  balancing loss E * sum_e f_e p_e is exposed as ``aux_loss``.
* Static shapes: every expert has a fixed capacity C = ceil(capacity_factor * tokens * k / E) rows (assignments
  beyond it are dropped, as in GShard / Switch). Dispatch is an index copy into [E, C, D]; the experts run as ONE
  batched tcgen05 GEMM per projection (E is the batch dimension), so there is no host synchronisation and no
  per-expert launch.
* Expert parallelism: with a process group of size W (E % W == 0), rank r owns experts [r E/W, (r+1) E/W).
  ``transport="p2p"`` (CUDA): the dispatch and combine run over NVLink peer memory, fused with the token gather,
  the expert GEMMs (which wait for arriving rows tile by tile and store their outputs into the sources' memory)
  and the weighted sum (parallel/moe_comm.py). ``transport="nccl"``: the [E, C, D] dispatch buffer is exchanged
  with one all_to_all (fixed splits: no count exchange needed), the local experts run on [W, C, D] rows each, and
  a second all_to_all returns the outputs for the weighted combine.
"""
import math

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..ops import fused as Fz
from ..ops.gemm import gemm


class _BatchedLinear(torch.autograd.Function):
    """y[e] = x[e] @ w[e]^T for e in the batch; w fp32 master (grad accumulated in fp32), bf16 compute on CUDA."""

    @staticmethod
    def forward(ctx, x, w):
        xb = x.to(torch.bfloat16).contiguous()
        wb = w.detach().to(torch.bfloat16).contiguous()
        ctx.save_for_backward(xb, wb)
        ctx.w = w
        return gemm(xb, wb)

    @staticmethod
    def backward(ctx, dy):
        xb, wb = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        dx = gemm(dy, wb, b_mn=True)
        w = ctx.w
        if w.requires_grad:
            if w.grad is None:
                w.grad = torch.zeros_like(w, dtype=torch.float32)
            gemm(dy, xb, out=w.grad, a_mn=True, b_mn=True, accumulate=True)
            Fz._notify(w)
        return dx, None


def batched_linear(x, w):
    if not x.is_cuda:
        return torch.bmm(x.float(), w.float().transpose(1, 2))
    return _BatchedLinear.apply(x, w)


class MoEMLP(nn.Module):
    def __init__(self, dim, hidden, experts=8, top_k=2, capacity_factor=1.25, group=None, transport="p2p"):
        super().__init__()
        self.dim, self.hidden, self.E, self.k, self.cf = dim, hidden, experts, top_k, capacity_factor
        self.group, self.transport, self.exchange = group, transport, None
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        assert experts % self.world == 0
        self.local = experts // self.world
        self.router = nn.Linear(dim, experts, bias=False)
        self.w_in = nn.Parameter(torch.empty(self.local, 2 * hidden, dim))
        self.w_out = nn.Parameter(torch.empty(self.local, dim, hidden))
        self.aux_loss = None
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        nn.init.normal_(self.router.weight, std=0.02)
        nn.init.normal_(self.w_in, std=self.dim ** -0.5)
        nn.init.normal_(self.w_out, std=self.hidden ** -0.5)

    def capacity(self, n_tokens, multiple=8):
        return max(multiple, int(math.ceil(self.cf * n_tokens * self.k / self.E / multiple)) * multiple)

    def _fused(self, x):
        return self.transport == "p2p" and x.is_cuda and self.dim % 64 == 0 and self.hidden % 64 == 0

    def _forward_fused(self, x2, w, idx):
        """Peer-memory exchange fused with the expert GEMMs (parallel/moe_comm.py)."""
        from ..parallel.moe_comm import MoEPeerExchange, exchange_experts
        N = x2.shape[0]
        C = self.capacity(N, 128)
        if self.exchange is None or self.exchange.C != C:
            self.exchange = MoEPeerExchange(self.E, self.local, C, self.dim, self.hidden, self.group, x2.device)
        flat_e = idx.reshape(-1)
        onehot = F.one_hot(flat_e, self.E)
        pos = (onehot.cumsum(0) - onehot).gather(1, flat_e[:, None]).squeeze(1)
        keep = pos < C
        slot = torch.where(keep, flat_e * C + pos, torch.full_like(pos, -1))
        tok = torch.arange(N, device=x2.device).repeat_interleave(self.k)
        src_tok = torch.full((self.E * C,), -1, dtype=torch.int32, device=x2.device)
        src_tok[slot[keep]] = tok[keep].to(torch.int32)
        slot_w = torch.zeros(self.E * C, dtype=torch.float32, device=x2.device)
        slot_w[slot[keep]] = w.detach().reshape(-1)[keep].float()
        return exchange_experts(x2, w, self.w_in, self.w_out, self.exchange, src_tok,
                                slot.view(N, self.k).to(torch.int32).contiguous(), slot_w)

    def route(self, x2):
        logits = F.linear(x2.float(), self.router.weight.float())
        probs = logits.softmax(-1)
        w, idx = probs.topk(self.k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        # Switch load-balancing loss: E * sum_e (fraction of assignments to e) * (mean router prob of e)
        frac = F.one_hot(idx, self.E).float().sum(1).mean(0) / self.k
        self.aux_loss = self.E * (frac * probs.mean(0)).sum()
        return w, idx

    def experts(self, buf):
        """buf [local, rows, D] -> [local, rows, D] through the local experts' SwiGLU."""
        ab = batched_linear(buf, self.w_in)
        h = Fz.swiglu(ab.contiguous()) if ab.is_cuda else Fz.swiglu(ab)
        return batched_linear(h, self.w_out)

    def forward(self, h):
        shape = h.shape
        x2 = h.reshape(-1, self.dim)
        N = x2.shape[0]
        w, idx = self.route(x2)
        if self._fused(x2):
            return self._forward_fused(x2, w, idx).view(shape)
        C = self.capacity(N)
        flat_e = idx.reshape(-1)                                    # [N k]
        onehot = F.one_hot(flat_e, self.E)
        pos = (onehot.cumsum(0) - onehot).gather(1, flat_e[:, None]).squeeze(1)  # rank of each assignment
        keep = pos < C
        tok = torch.arange(N, device=x2.device).repeat_interleave(self.k)
        slot = flat_e * C + pos
        buf = x2.new_zeros(self.E * C, self.dim)
        buf = buf.index_copy(0, slot[keep], x2[tok[keep]])
        buf = buf.view(self.E, C, self.dim)
        if self.world > 1:
            from torch.distributed.nn.functional import all_to_all_single
            send = buf.reshape(self.world, self.local, C, self.dim).reshape(-1, self.dim).contiguous()
            recv = all_to_all_single(torch.empty_like(send), send, group=self.group)
            # rows from rank src for my local expert j: recv[src, j] -> [local, world * C, D]
            y = self.experts(recv.view(self.world, self.local, C, self.dim).transpose(0, 1).reshape(
                self.local, self.world * C, self.dim))
            back = y.view(self.local, self.world, C, self.dim).transpose(0, 1).reshape(-1, self.dim).contiguous()
            out_buf = all_to_all_single(torch.empty_like(back), back, group=self.group)
            out_buf = out_buf.view(self.world, self.local, C, self.dim).reshape(self.E * C, self.dim)
        else:
            out_buf = self.experts(buf).reshape(self.E * C, self.dim)
        gathered = out_buf.index_select(0, slot.clamp(max=self.E * C - 1)) * (keep.to(out_buf.dtype) *
                                                                                 w.reshape(-1).to(out_buf.dtype))[:, None]
        out = gathered.view(N, self.k, self.dim).sum(1)
        return out.view(shape)


def moe_dense_reference(mlp, h):
    """Every token through its top-k experts without capacity limits (test oracle; local experts only)."""
    x2 = h.reshape(-1, mlp.dim).float()
    w, idx = mlp.route(x2)
    out = torch.zeros_like(x2)
    for e in range(mlp.E):
        a, b = (x2 @ mlp.w_in[e].float().T).chunk(2, dim=-1)
        y = (F.silu(a) * b) @ mlp.w_out[e].float().T
        for k in range(mlp.k):
            m = idx[:, k] == e
            out[m] += w[m, k, None] * y[m]
    return out.view(h.shape)


def moe_denoiser(den, experts=8, top_k=2, expert_hidden=4096, every=2, capacity_factor=1.25, group=None,
                 transport="p2p"):
    """Replace the MLP of every `every`-th block (odd blocks for every=2) with an MoE MLP, in place."""
    for i, blk in enumerate(den.blocks):
        if i % every == every - 1:
            blk.mlp = MoEMLP(den.config.dim, expert_hidden, experts, top_k, capacity_factor, group, transport).to(
                den.patch_in.weight.device)
    return den


def moe_aux_loss(den):
    losses = [m.aux_loss for m in den.modules() if isinstance(m, MoEMLP) and m.aux_loss is not None]
    return torch.stack(losses).mean() if losses else None
