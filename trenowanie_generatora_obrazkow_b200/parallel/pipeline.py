"""Pipeline parallelism: stage partitioning, stage-local models and a 1F1B schedule over NCCL point-to-point.

Reference behaviour (train_pp.py:311-385, 446-454, 1329-1346, 1539-1551, 2219-2283): stage 0 holds the text
encoder and the stem (patch_in, time MLP, ada, micro-conditioning), every stage a contiguous range of blocks (stage 0
fewer, balancing the text encoder's cost), the last stage the head; activations (x, t6, text) flow forward and their
gradients backward; M micro-batches per step run in one-forward-one-backward order. Here:

* ``stage_ranges`` balances blocks the same way; ``StageModel`` materialises only the parameters a stage owns
  (the full model is built on the meta device first), with the full model's parameter names, so stage files merge
  into an ordinary checkpoint.
* ``OneFOneB`` is this framework's own scheduler: warm-up forwards (pp - s - 1), steady 1F1B, cool-down backwards.
  Per stage boundary and micro-batch: x (bf16), t6, text (bf16), text lengths forward; their gradients backward.
  Every adjacent stage pair has two process groups, one per direction (``direction_groups``), so a communicator
  stream only ever carries activations s -> s + 1 or gradients s + 1 -> s, in the same order on both ends: no
  send can wait behind a receive, and transfers are posted individually. A receive is posted one micro-batch
  before its data is used and the compute stream waits for it only right before that use; sends never hold the
  compute stream (their completion is awaited once, at the end of the step), so a stage runs on while its
  neighbour is still busy.
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
        self.act_checkpoint = False

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

    def stem(self, z_t, t, text_kw, cond=None, hw=None):
        """Stage 0: (x, t6, text, text_len) from latents, t and the text-encoder inputs. z_t is [B, C, H, W], or with
        ``hw`` = (H, W) already token-major [B, H * W, C] (the fused flow-matching input kernel's output)."""
        from ..ops import fused as Fz
        from ..train.flow import LMTextEncoder
        if hw is None:
            b, c, h, w = z_t.shape
        else:
            b, (h, w) = z_t.shape[0], hw
        if isinstance(self.te, LMTextEncoder):
            if getattr(self, "te_checkpoint", False) and torch.is_grad_enabled():  # recomputed in the backward
                text, valid = torch.utils.checkpoint.checkpoint(
                    lambda st, v, nl: self.te(lm_states=st, valid=v, is_null=nl), text_kw["lm_states"],
                    text_kw["valid"], text_kw.get("is_null"), use_reentrant=False)
            else:
                text, valid = self.te(**text_kw)
        else:
            text, valid = self.te(text_kw["ids"])
        tok = z_t.flatten(2).transpose(1, 2) if hw is None else z_t
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
        from ..ops import fused as Fz
        cos, sin = self.rope(side, side, x.device)
        pending = None
        for blk in self.blocks:  # act_checkpoint: False, "full" or "selective" (ops/fused.py run_block)
            x, pending = Fz.run_block(blk, (x, pending, t6, text, text_len, cos, sin), self.act_checkpoint)
        if self.last:
            from ..ops import fused as Fz
            if x.is_cuda:
                y, g = pending if pending is not None else (None, None)
                _, hn = Fz.adanorm(x, y, g, self.norm.weight)
            else:
                hn = R.rmsnorm(_flush(x, pending), self.norm.weight)
            return Fz.linear(hn, self.patch_out)  # token-major velocity [B, T, C]
        return _flush(x, pending)


def direction_groups(pipes, device=None):
    """{(rank_a, rank_b): group} for every adjacent stage pair of every pipe, one group per direction (a -> b). A
    collective over the default group: every rank calls it, in the same order.

    NCCL builds a group's communicator at its first operation, and that setup blocks the host until both members
    take part. Left to the schedule, stage s would block setting up its first gradient receive while stage s + 1,
    whose GPU already holds a posted receive from stage s, cannot finish the forward that precedes its first gradient
    send: a deadlock. So every group is set up here with a one-element all-reduce, the groups walked in one global
    order by every rank (each waits only for groups it belongs to, so the earliest unfinished group always has both
    members waiting on it)."""
    out = {}
    for pipe in pipes:
        for s in range(len(pipe) - 1):
            a, b = pipe[s], pipe[s + 1]
            out[(a, b)] = dist.new_group([a, b])  # activations a -> b
            out[(b, a)] = dist.new_group([a, b])  # gradients b -> a
    if dist.get_backend() == "nccl":
        me = dist.get_rank()
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        one = torch.zeros(1, device=dev)
        for key in sorted(out):
            if me in key:
                dist.all_reduce(one, group=out[key])
        torch.cuda.synchronize(dev)
    return out


class OneFOneB:
    """1F1B over one pipe. ``pipe`` = global ranks of this replica's stages (pipe[s] is stage s); ``links``: the
    result of ``direction_groups`` (required for more than one stage: a send and a receive between the same two
    ranks must never share a stream, or each could wait behind the other)."""

    def __init__(self, stage_model, pipe, stage, micro_shapes, device, links=None):
        self.m = stage_model
        self.pipe, self.s, self.pp = pipe, stage, len(pipe)
        self.shapes = micro_shapes  # dict: x, t6, text (shapes), dtypes
        self.device = device
        self.links = links or {}
        if self.pp > 1:
            for a, b in ((stage - 1, stage), (stage, stage - 1), (stage, stage + 1), (stage + 1, stage)):
                if 0 <= a < self.pp and 0 <= b < self.pp and (pipe[a], pipe[b]) not in self.links:
                    raise ValueError("OneFOneB needs direction_groups(...) links for its neighbours")
        self._sends = []   # (works, buffers) of sends whose completion is awaited at the end of the step
        self.early = False

    # ---- communication -----------------------------------------------------------------------------------------
    def _empty_acts(self):
        sh = self.shapes
        return [torch.empty(sh["x"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["t6"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["text"], dtype=sh["dtype"], device=self.device),
                torch.empty(sh["x"][0], dtype=torch.int32, device=self.device)]

    def _empty_grads(self):
        sh = self.shapes
        return [torch.empty(sh[k], dtype=sh["dtype"], device=self.device) for k in ("x", "t6", "text")]

    def _link(self, src, dst):
        return self.links[(self.pipe[src], self.pipe[dst])]

    def _post_recv(self, bufs, peer):
        """Post receives from stage `peer`; returns a handle for ``_wait``."""
        g = self._link(peer, self.s)
        ops = [dist.P2POp(dist.irecv, b, self.pipe[peer], g) for b in bufs]
        return bufs, dist.batch_isend_irecv(ops)

    @staticmethod
    def _wait(handle):
        """The compute stream waits for the posted receives (NCCL: a stream dependency, the host runs on)."""
        bufs, works = handle
        for w in works:
            w.wait()
        return bufs

    def _send(self, bufs, peer):
        g = self._link(self.s, peer)
        bufs = [b.contiguous() for b in bufs]
        works = dist.batch_isend_irecv([dist.P2POp(dist.isend, b, self.pipe[peer], g) for b in bufs])
        self._sends.append((works, bufs))  # kept alive; completion awaited at the end of the step

    def _finish_sends(self):
        for works, _ in self._sends:
            for w in works:
                w.wait()
        self._sends = []

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
        # receives posted a micro-batch ahead (off by default): with NCCL a receive posted before its peer reaches the
        # matching send leaves a kernel waiting on the GPU, and a host call that synchronises the device meanwhile
        # (the caching allocator freeing cached blocks under memory pressure) then waits for a peer that is itself
        # waiting on this rank. On B200 at 1024 px the 2-stage bench stalled that way; posting each receive right
        # before it is needed keeps every pending NCCL kernel one whose peer is already on its way to the match.
        early = self.early

        def forward(i, acts):
            if first:
                z, t, kw = first_inputs(i)
                x, t6, text, tl = self.m.stem(z, t, {k: v for k, v in kw.items() if k not in ("cond", "hw")},
                                              kw.get("cond"), kw.get("hw"))
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

        # posted receives: activations of forward i, gradients of backward i
        act_h, grad_h = {}, {}

        def post_act(i):
            if not first and i < M and i not in act_h:
                act_h[i] = self._post_recv(self._empty_acts(), s - 1)

        def post_grad(i):
            if not last and i < M and i not in grad_h:
                grad_h[i] = self._post_recv(self._empty_grads(), s + 1)

        def acts_of(i):
            if first:
                return None
            post_act(i)
            return self._wait(act_h.pop(i))

        def grads_of(i):
            if last:
                return None
            post_grad(i)
            return self._wait(grad_h.pop(i))

        for i in range(n_warm):
            a = acts_of(i)
            if early:
                post_act(i + 1)
            out = forward(i, a)
            self._send(out, s + 1)
        if early:
            post_grad(0)
        for j in range(n_steady):
            i_f, i_b = n_warm + j, j
            a = acts_of(i_f)
            if early:
                post_act(i_f + 1)
            out = forward(i_f, a)
            if not last:
                self._send(out, s + 1)
            g_in = backward(i_b, grads_of(i_b))
            if early:
                post_grad(i_b + 1)
            if not first:
                self._send(g_in, s - 1)
        for i in range(n_steady, M):
            g_in = backward(i, grads_of(i))
            if early:
                post_grad(i + 1)
            if not first:
                self._send(g_in, s - 1)
        self._finish_sends()
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
