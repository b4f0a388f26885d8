"""Pipeline parallelism: stage partitioning, stage-local models and a 1F1B schedule over NCCL point-to-point.

Reference behaviour (train_pp.py:311-385, 446-454, 1329-1346, 1539-1551, 2219-2283): stage 0 holds the text
encoder and the stem (patch_in, time MLP, ada, micro-conditioning), every stage a contiguous range of blocks (stage 0
fewer, balancing the text encoder's cost), the last stage the head; activations (x, t6, text) flow forward and their
gradients backward; M micro-batches per step run in one-forward-one-backward order. Here:

* ``stage_ranges`` balances blocks the same way; ``StageModel`` materialises only the parameters a stage owns
  (the full model is built on the meta device first), with the full model's parameter names, so stage files merge
  into an ordinary checkpoint.
* ``OneFOneB`` is this framework's own scheduler: warm-up forwards (pp - s - 1), steady 1F1B with the send of one
  micro-batch's activations batched with the receive of another's gradient (``batch_isend_irecv``, so the pairs can
  not deadlock), cool-down backwards. Per stage boundary and micro-batch: x (bf16), t6, text (bf16), text lengths.
* The last stage needs the flow-matching target eps - x0 for every micro-batch; stage 0 (which has the data)
  sends all of them before the schedule starts.
* PP x DP: rank = replica * pp + stage; gradient reduction and sharded Muon run over the stage group (the same
  stage of every replica), the clipping norm over the pipe group.
"""
import math

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..models.dit import Denoiser, _flush
from ..models.text import build_text_encoder
from ..ops import reference as R


def stage_ranges(depth, pp, first_extra=0.0):
    """Contiguous [lo, hi) block ranges; stage 0 also does `first_extra` blocks' worth of other work."""
    bounds = np.linspace(0, depth + first_extra, pp + 1) - first_extra
    bounds = np.clip(bounds.round(), 0, depth).astype(int)
    bounds[0], bounds[-1] = 0, depth
    if not (np.diff(bounds)[1:] > 0).all():
        raise ValueError(f"{depth} blocks can not fill {pp} stages")
    return [(int(bounds[s]), int(bounds[s + 1])) for s in range(pp)]


def grid_layout(world, pp):
    """(stage, replica) of every rank and the process groups: pipes (one per replica) and stage groups."""
    assert world % pp == 0, "world size must be a multiple of the pipeline depth"
    dp = world // pp
    pipes = [[r * pp + s for s in range(pp)] for r in range(dp)]
    stages = [[r * pp + s for r in range(dp)] for s in range(pp)]
    return dp, pipes, stages


class StageModel(nn.Module):
    """The part of (text encoder, denoiser) one stage runs. Parameter names are the full model's
    (``te.*`` / ``den.*``) in ``full_named_parameters``."""

    def __init__(self, den_cfg, te_cfg, lo, hi, first, last, device, seed=0):
        super().__init__()
        self.den_cfg, self.lo, self.hi, self.first, self.last = den_cfg, lo, hi, first, last
        with torch.device("meta"):
            den = Denoiser(den_cfg)
        self.blocks = nn.ModuleList([den.blocks[i] for i in range(lo, hi)])
        if first:
            self.patch_in, self.time_mlp, self.ada = den.patch_in, den.time_mlp, den.ada
            self.cond_mlp = den.cond_mlp if den_cfg.micro_cond else None
        if last:
            self.norm, self.patch_out = den.norm, den.patch_out
        self.to_empty(device=device)
        torch.manual_seed(seed)
        with torch.no_grad():  # the unsplit model's init_stem / init_block / init_head, on the owned parts
            if first:
                Denoiser.init_stem(self)
            for b in self.blocks:
                Denoiser.init_block(b)
            if last:
                Denoiser.init_head(self)
        if first:
            self.te = build_text_encoder(te_cfg)
            self.te.init_weights()
            self.te.to(device)
        self._rope = {}

    # Denoiser.init_stem / init_cond / init_head read these attributes
    @property
    def config(self):
        return self.den_cfg

    def init_cond(self):
        if self.den_cfg.micro_cond:
            nn.init.normal_(self.cond_mlp[0].weight, std=0.02)
            nn.init.zeros_(self.cond_mlp[0].bias)
            nn.init.zeros_(self.cond_mlp[2].weight)
            nn.init.zeros_(self.cond_mlp[2].bias)

    @torch.no_grad()
    def load_full_state(self, te_sd, den_sd):
        """Copy this stage's tensors out of the unsplit model's state dicts."""
        for prefix, name, p in self.full_named_parameters():
            p.copy_((te_sd if prefix == "te" else den_sd)[name].to(p.device, p.dtype))

    def full_named_parameters(self):
        """(prefix, full name, param) with the unsplit model's names."""
        out = []
        for n, p in self.named_parameters():
            if n.startswith("te."):
                out.append(("te", n[3:], p))
            elif n.startswith("blocks."):
                i, rest = n[len("blocks."):].split(".", 1)
                out.append(("den", f"blocks.{self.lo + int(i)}.{rest}", p))
            else:
                out.append(("den", n, p))
        return out

    def rope(self, h, w, device):
        key = (h, w, str(device))
        if key not in self._rope:
            self._rope[key] = R.rope_2d_table(h, w, self.den_cfg.dim // self.den_cfg.heads, self.den_cfg.rope_ref,
                                              device)
        return self._rope[key]

    def stem(self, z_t, t, text_kw, cond=None):
        """Stage 0: (x, t6, text, text_len) from latents, t and the text-encoder inputs."""
        from ..ops import fused as Fz
        from ..train.flow import LMTextEncoder
        b, c, h, w = z_t.shape
        if isinstance(self.te, LMTextEncoder):
            if getattr(self, "te_checkpoint", False) and torch.is_grad_enabled():  # recomputed in the backward
                text, valid = torch.utils.checkpoint.checkpoint(
                    lambda st, v, nl: self.te(lm_states=st, valid=v, is_null=nl), text_kw["lm_states"],
                    text_kw["valid"], text_kw.get("is_null"), use_reentrant=False)
            else:
                text, valid = self.te(**text_kw)
        else:
            text, valid = self.te(text_kw["ids"])
        tok = z_t.flatten(2).transpose(1, 2)
        if z_t.is_cuda:
            tok = tok.to(torch.bfloat16).contiguous()
            text = text.to(torch.bfloat16)
        x = Fz.linear(tok, self.patch_in)
        t_emb = Fz.linear(R.timestep_embedding(t, 256), self.time_mlp[0])
        t_emb = Fz.linear(F.silu(t_emb), self.time_mlp[2])
        if self.den_cfg.micro_cond:
            cond = cond if cond is not None else R.default_micro_cond(self.den_cfg.micro_cond, 16 * h, b, t.device)
            cc = Fz.linear(R.micro_cond_embedding(cond), self.cond_mlp[0])
            t_emb = t_emb + Fz.linear(F.silu(cc), self.cond_mlp[2])
        t6 = Fz.linear(F.silu(t_emb), self.ada).view(b, 6, self.den_cfg.dim)
        return x, t6, text, R.valid_to_len(valid).to(torch.int32)

    def run(self, x, t6, text, text_len, side):
        cos, sin = self.rope(side, side, x.device)
        pending = None
        for blk in self.blocks:
            x, pending = blk(x, pending, t6, text, text_len, cos, sin)
        if self.last:
            from ..ops import fused as Fz
            if x.is_cuda:
                y, g = pending if pending is not None else (None, None)
                _, hn = Fz.adanorm(x, y, g, self.norm.weight)
            else:
                hn = R.rmsnorm(_flush(x, pending), self.norm.weight)
            return Fz.linear(hn, self.patch_out)  # token-major velocity [B, T, C]
        return _flush(x, pending)


class OneFOneB:
    """1F1B over one pipe. ``pipe`` = global ranks of this replica's stages (pipe[s] is stage s)."""

    def __init__(self, stage_model, pipe, stage, micro_shapes, device, group=None):
        self.m = stage_model
        self.pipe, self.s, self.pp = pipe, stage, len(pipe)
        self.shapes = micro_shapes  # dict: x, t6, text (shapes), dtypes
        self.device = device
        self.group = group

    # ---- communication -----------------------------------------------------------------------------------------
    def _empty_acts(self):
        sh = self.shapes
        return [torch.empty(sh["x"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["t6"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["text"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["x"][0], dtype=torch.int32, device=self.device)]

    def _run(self, ops):
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()

    def _recv_ops(self, bufs, peer):
        return [dist.P2POp(dist.irecv, b, self.pipe[peer], self.group) for b in bufs]

    def _send_ops(self, bufs, peer):
        return [dist.P2POp(dist.isend, b.contiguous(), self.pipe[peer], self.group) for b in bufs]

    # ---- one step --------------------------------------------------------------------------------------------
    def step(self, M, first_inputs=None, targets=None, side=None, loss_scale=1.0, before_last_backward=None):
        """first_inputs(i) -> (z_t, t, text_kw) on stage 0; targets: list of M token-major targets on the last
        stage. Returns the summed loss (last stage) or None."""
        s, pp = self.s, self.pp
        first, last = s == 0, s == pp - 1
        n_warm = min(pp - s - 1, M)
        n_steady = M - n_warm
        saved = {}
        losses = []

        def forward(i, acts):
            if first:
                z, t, kw = first_inputs(i)
                x, t6, text, tl = self.m.stem(z, t, {k: v for k, v in kw.items() if k != "cond"}, kw.get("cond"))
                ins = None
            else:
                x, t6, text, tl = acts
                for a in (x, t6, text):
                    a.requires_grad_(True)
                ins = (x, t6, text)
            out = self.m.run(x, t6, text, tl, side)
            if last:
                loss = F.mse_loss(out.float(), targets[i]) * loss_scale
                losses.append(loss.detach())
                saved[i] = (ins, loss, None)
                return None
            saved[i] = (ins, (out, t6, text), tl)
            return [out.detach(), t6.detach(), text.detach(), tl]

        def backward(i, grads):
            if i == M - 1 and before_last_backward is not None:
                before_last_backward()  # e.g. arm the gradient buckets: they reduce as this backward completes them
            ins, outs, _ = saved.pop(i)
            if last:
                outs.backward()
            else:
                torch.autograd.backward(list(outs), grads)
            if first:
                return None
            return [a.grad if a.grad is not None else torch.zeros_like(a) for a in ins]

        def recv_fwd():
            if first:
                return None
            bufs = self._empty_acts()
            self._run(self._recv_ops(bufs, s - 1))
            return bufs

        for i in range(n_warm):
            out = forward(i, recv_fwd())
            self._run(self._send_ops(out, s + 1))
        acts = recv_fwd() if n_steady > 0 else None
        for j in range(n_steady):
            i_f, i_b = n_warm + j, j
            out = forward(i_f, acts)
            if last:
                gr = None
            else:  # send activations of i_f, receive the gradient of i_b
                gr = [torch.empty_like(t) for t in out[:3]]
                self._run(self._send_ops(out, s + 1) + self._recv_ops(gr, s + 1))
            g_in = backward(i_b, gr)
            if j == n_steady - 1:
                acts = None
                if not first:
                    self._run(self._send_ops(g_in, s - 1))
            else:
                if first:
                    acts = None
                else:  # send the gradient of i_b, receive the activations of i_f + 1
                    nxt = self._empty_acts()
                    self._run(self._send_ops(g_in, s - 1) + self._recv_ops(nxt, s - 1))
                    acts = nxt
        for i in range(n_steady, M):
            gr = None
            if not last:
                gr = [torch.empty(self.shapes[k], dtype=self.shapes["dtype"], device=self.device)
                      for k in ("x", "t6", "text")]
                self._run(self._recv_ops(gr, s + 1))
            g_in = backward(i, gr)
            if not first:
                self._run(self._send_ops(g_in, s - 1))
        return torch.stack(losses).sum() if last else None


def send_targets(targets, pipe, group=None):
    """Stage 0 -> last stage: the M flow-matching targets (one batched transfer before the schedule)."""
    if len(pipe) == 1:
        return targets
    ops = [dist.P2POp(dist.isend, t.contiguous(), pipe[-1], group) for t in targets]
    for r in dist.batch_isend_irecv(ops):
        r.wait()
    return None


def recv_targets(M, shape, dtype, device, pipe, group=None):
    bufs = [torch.empty(shape, dtype=dtype, device=device) for _ in range(M)]
    ops = [dist.P2POp(dist.irecv, b, pipe[0], group) for b in bufs]
    for r in dist.batch_isend_irecv(ops):
        r.wait()
    return bufs


@torch.no_grad()
def pipe_grad_norm(params, group=None):
    """Global gradient norm of the pipe (every stage's squared norm summed over the pipe group)."""
    grads = [p.grad for p in params if p.grad is not None]
    sq = torch.stack(torch._foreach_norm(grads)).float().square().sum() if grads else torch.zeros((), device="cpu")
    if dist.is_initialized():
        dist.all_reduce(sq, group=group)
    return sq.sqrt()


@torch.no_grad()
def clip_with_norm(params, total_norm, max_norm):
    coef = (max_norm / (total_norm + 1e-6)).clamp(max=1.0)
    grads = [p.grad for p in params if p.grad is not None]
    torch._foreach_mul_(grads, coef.to(grads[0].device) if grads else coef)
