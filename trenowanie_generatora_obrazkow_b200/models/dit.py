"""Flow-matching DiT denoiser (adaLN-single, 2D RoPE, QK-norm, text cross-attention, SwiGLU).

Behaviour follows the reference Denoiser (aurora/model.py:191-210, :315-405): patch_in on one token per latent
pixel, time MLP, shared ``ada`` projection to 6 x dim plus a per-block ``mod_table``, gated self-attention and MLP,
ungated and unmodulated cross-attention, final RMSNorm without modulation, patch_out. Parameter names and shapes are
the reference's, so ``state_dict`` of either framework loads into the other.

Execution is B200-first: each block is a chain of fused sm_100a kernels (ops/fused.py). The residual stream stays
bf16; the gated residual add of each branch is deferred into the next RMSNorm kernel (adanorm), so a block costs one
read/write pass of the residual stream per norm instead of separate add / norm / modulate passes.
"""
import math

import torch
import torch.nn as nn

from ..ops import fused as Fz
from ..ops import reference as R
from .config import DenoiserConfig


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        return R.rmsnorm(x, self.weight, self.eps)


class SwiGLU(nn.Module):
    def __init__(self, dim, hidden):
        super().__init__()
        self.in_proj = nn.Linear(dim, 2 * hidden, bias=False)
        self.out_proj = nn.Linear(hidden, dim, bias=False)

    def forward(self, h):
        return Fz.linear(Fz.up_swiglu(h, self.in_proj), self.out_proj)


class SelfAttention(nn.Module):
    def __init__(self, dim, heads):
        super().__init__()
        self.heads = heads
        self.head_dim = dim // heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.out = nn.Linear(dim, dim, bias=False)
        self.q_norm = RMSNorm(self.head_dim)
        self.k_norm = RMSNorm(self.head_dim)
        self.logit_mult = 1.0  # sampling only: multiplies the attention logits (resolution extrapolation)

    def forward(self, h, cos, sin):
        qkv = Fz.linear(h, self.qkv)
        o = Fz.self_attention_core(qkv, self.heads, self.heads, self.head_dim, self.q_norm.weight, self.k_norm.weight,
                                   cos, sin, None, self.logit_mult / math.sqrt(self.head_dim))
        return Fz.linear(o, self.out)


class CrossAttention(nn.Module):
    def __init__(self, dim, heads, text_dim):
        super().__init__()
        self.heads = heads
        self.head_dim = dim // heads
        self.q = nn.Linear(dim, dim, bias=False)
        self.kv = nn.Linear(text_dim, 2 * dim, bias=False)
        self.out = nn.Linear(dim, dim, bias=False)

    def forward(self, h, text, text_len):
        o = Fz.cross_attention_core(Fz.linear(h, self.q), Fz.linear(text, self.kv), self.heads, text_len)
        return Fz.linear(o, self.out)


class DenoiserBlock(nn.Module):
    """adaLN-single block: (t6 + mod_table) -> shift/scale/gate x 2 (reference aurora/model.py:191-210)."""

    def __init__(self, dim, heads, text_dim, mlp_hidden):
        super().__init__()
        self.norm1 = RMSNorm(dim)
        self.attn = SelfAttention(dim, heads)
        self.norm2 = RMSNorm(dim)
        self.cross = CrossAttention(dim, heads, text_dim)
        self.norm3 = RMSNorm(dim)
        self.mlp = SwiGLU(dim, mlp_hidden)
        self.mod_table = nn.Parameter(torch.zeros(6, dim))

    def forward(self, x, pending, t6, text, text_len, cos, sin):
        """x: residual stream [B, T, D] with `pending` = (branch, gate) not yet added (None for the first block).
        Returns (x, pending) with this block's gated MLP branch pending."""
        mod = (t6 + self.mod_table[None]).to(x.dtype)
        shift1, scale1, gate1, shift2, scale2, gate2 = mod.unbind(1)
        y, g = pending if pending is not None else (None, None)
        x, h = Fz.adanorm(x, y, g, self.norm1.weight, shift1, scale1)
        y = self.attn(h, cos, sin)
        x, h = Fz.adanorm(x, y, gate1, self.norm2.weight)
        y = self.cross(h, text, text_len)
        x, h = Fz.adanorm(x, y, None, self.norm3.weight, shift2, scale2)
        return x, (self.mlp(h), gate2)


def _flush(x, pending):
    if pending is None:
        return x
    y, g = pending
    return x + (y if g is None else g[:, None] * y)


class Denoiser(nn.Module):
    """Velocity predictor v(z_t, t, text) on (B, C, H, W) latents, one token per latent pixel."""

    def __init__(self, cfg: DenoiserConfig = DenoiserConfig()):
        super().__init__()
        self.config = cfg
        dim = cfg.dim
        self.patch_in = nn.Linear(cfg.latent_channels, dim, bias=False)
        self.time_mlp = nn.Sequential(nn.Linear(256, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.ada = nn.Linear(dim, 6 * dim)
        if cfg.micro_cond:
            self.cond_mlp = nn.Sequential(nn.Linear(8 * 256, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.blocks = nn.ModuleList([DenoiserBlock(dim, cfg.heads, cfg.text_dim, cfg.mlp_hidden)
                                     for _ in range(cfg.depth)])
        self.norm = RMSNorm(dim)
        self.patch_out = nn.Linear(dim, cfg.latent_channels, bias=False)
        self._rope_cache = {}
        self.checkpoint_blocks = False  # activation checkpointing: False, "full" / True or "selective"

    # ---------------------------------------------------------------------------------------------- RoPE tables
    def rope(self, h, w, device):
        """2D RoPE tables [h*w, head_dim] for an h x w latent grid (rope_ref: position interpolation)."""
        key = (h, w, str(device), self.config.rope_ref)
        ent = self._rope_cache.get(key)
        if ent is None:
            ent = R.rope_2d_table(h, w, self.config.dim // self.config.heads, self.config.rope_ref, device)
            self._rope_cache[key] = ent
        return ent

    # ---------------------------------------------------------------------------------------------- conditioning
    def time_embedding(self, t, cond=None, res=0):
        """Time embedding (+ micro-conditions (B, 8), default: a whole image at res px) -> [B, D]."""
        t_emb = Fz.linear(R.timestep_embedding(t, 256), self.time_mlp[0])
        t_emb = Fz.linear(torch.nn.functional.silu(t_emb), self.time_mlp[2])
        if self.config.micro_cond:
            if cond is None:
                cond = R.default_micro_cond(self.config.micro_cond, res, t.shape[0], t.device)
            c = Fz.linear(R.micro_cond_embedding(cond), self.cond_mlp[0])
            t_emb = t_emb + Fz.linear(torch.nn.functional.silu(c), self.cond_mlp[2])
        return t_emb

    def modulation(self, t, cond=None, res=0):
        b, dim = t.shape[0], self.config.dim
        t_emb = self.time_embedding(t, cond, res)
        return Fz.linear(torch.nn.functional.silu(t_emb), self.ada).view(b, 6, dim)

    # ---------------------------------------------------------------------------------------------- forward
    def embed(self, z_t):
        """(B, C, H, W) latents -> tokens [B, H*W, D] (row-major)."""
        b, c, h, w = z_t.shape
        tok = z_t.flatten(2).transpose(1, 2)
        if z_t.is_cuda:
            tok = tok.to(torch.bfloat16).contiguous()
        return Fz.linear(tok, self.patch_in)

    def head(self, x, pending, shape, tokens_out=False):
        b, c, h, w = shape
        if x.is_cuda:
            y, g = pending if pending is not None else (None, None)
            _, hn = Fz.adanorm(x, y, g, self.norm.weight)
        else:
            hn = self.norm(_flush(x, pending))
        out = Fz.linear(hn, self.patch_out)
        if tokens_out:
            return out
        return out.transpose(1, 2).reshape(b, c, h, w)

    def run_blocks(self, x, pending, t6, text, text_len, cos, sin, lo=0, hi=None, hidden_at=0):
        hidden = None
        hi = len(self.blocks) if hi is None else hi
        for i in range(lo, hi):
            # activation checkpointing: False, "full" (True) or "selective" (ops/fused.py run_block)
            x, pending = Fz.run_block(self.blocks[i], (x, pending, t6, text, text_len, cos, sin),
                                      self.checkpoint_blocks)
            if i + 1 == hidden_at:
                hidden = _flush(x, pending)
        return x, pending, hidden

    def forward(self, z_t, t, text, text_valid=None, hidden_at=0, cond=None, text_len=None, rope=None,
                tokens_out=False):
        """z_t (B, C, H, W); t (B,); text (B, L, text_dim); text_valid (B, L) bool or text_len (B,) int32.
        hidden_at > 0: also return the token states after that many blocks (REPA).
        rope: optional (cos, sin) [B, T, d] per-sample tables (RPE-2D random positions).
        tokens_out: return the velocity token-major (B, H*W, C) as computed (the sampler's fused update reads it)."""
        return self._forward(self.embed(z_t), z_t.shape, t, text, text_valid, hidden_at, cond, text_len, rope,
                             tokens_out)

    def forward_tokens(self, z_tok, hw, t, text, text_valid=None, hidden_at=0, cond=None, text_len=None, rope=None):
        """z_tok [B, H*W, C] token-major latents (bf16 on CUDA, as the fused flow-matching input kernel writes them):
        the patch-in GEMM reads them directly. Returns the token-major velocity [B, H*W, C] (and the hidden state
        with hidden_at)."""
        b, _, c = z_tok.shape
        return self._forward(Fz.linear(z_tok, self.patch_in), (b, c) + tuple(hw), t, text, text_valid, hidden_at,
                             cond, text_len, rope, True)

    def _forward(self, x, shape, t, text, text_valid, hidden_at, cond, text_len, rope, tokens_out):
        b, c, h, w = shape
        if text_len is None:
            text_len = R.valid_to_len(text_valid) if text_valid is not None else None
        if x.is_cuda:
            text = text.to(torch.bfloat16)
            if text_len is not None:
                text_len = text_len.to(device=x.device, dtype=torch.int32)
        t6 = self.modulation(t, cond, 16 * h)
        cos, sin = rope if rope is not None else self.rope(h, w, x.device)
        x, pending, hidden = self.run_blocks(x, None, t6, text, text_len, cos, sin, hidden_at=hidden_at)
        out = self.head(x, pending, shape, tokens_out)
        return out if not hidden_at else (out, hidden)

    # ---------------------------------------------------------------------------------------------- init
    @torch.no_grad()
    def init_weights(self):
        self.init_stem()
        for block in self.blocks:
            self.init_block(block)
        self.init_head()

    @torch.no_grad()
    def init_stem(self):
        """adaLN-Zero (single): ada and every mod_table start at zero, so all gates are 0 and each block starts as
        the identity; the gated output projections keep a normal init (one zero factor per gated product)."""
        nn.init.normal_(self.patch_in.weight, std=self.patch_in.in_features ** -0.5)
        for lin in (self.time_mlp[0], self.time_mlp[2]):
            nn.init.normal_(lin.weight, std=0.02)
            nn.init.zeros_(lin.bias)
        nn.init.zeros_(self.ada.weight)
        nn.init.zeros_(self.ada.bias)
        self.init_cond()

    @torch.no_grad()
    def init_cond(self):
        if self.config.micro_cond:
            nn.init.normal_(self.cond_mlp[0].weight, std=0.02)
            nn.init.zeros_(self.cond_mlp[0].bias)
            nn.init.zeros_(self.cond_mlp[2].weight)
            nn.init.zeros_(self.cond_mlp[2].bias)

    @staticmethod
    @torch.no_grad()
    def init_block(block):
        for lin in (block.attn.qkv, block.attn.out, block.cross.q, block.cross.kv, block.mlp.in_proj,
                    block.mlp.out_proj):
            nn.init.normal_(lin.weight, std=lin.in_features ** -0.5)
        for norm in (block.norm1, block.norm2, block.norm3, block.attn.q_norm, block.attn.k_norm):
            nn.init.ones_(norm.weight)
        nn.init.zeros_(block.mod_table)
        nn.init.zeros_(block.cross.out.weight)  # ungated cross-attention: a zero output still gets a gradient

    @torch.no_grad()
    def init_head(self):
        nn.init.ones_(self.norm.weight)
        nn.init.zeros_(self.patch_out.weight)

    @torch.no_grad()
    def grow(self, new_depth):
        """SANA-1.5-style depth growth (reference train_pp.py:1401-1426): keep the trained blocks and append new
        blocks whose attn.out, cross.out and mlp.out_proj start at zero (each new block starts as the identity)."""
        cfg = self.config
        old = len(self.blocks)
        assert new_depth >= old
        dev = self.patch_in.weight.device
        for _ in range(new_depth - old):
            blk = DenoiserBlock(cfg.dim, cfg.heads, cfg.text_dim, cfg.mlp_hidden).to(dev)
            self.init_block(blk)
            nn.init.zeros_(blk.attn.out.weight)
            nn.init.zeros_(blk.cross.out.weight)
            nn.init.zeros_(blk.mlp.out_proj.weight)
            self.blocks.append(blk)
        from dataclasses import replace
        self.config = replace(cfg, depth=new_depth)
