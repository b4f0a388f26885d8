"""Slayer-style GPT used as a frozen caption encoder (reference aurora/slayer.py:30-146: the SlayerLab GoLLeM
inference architecture with a ``hidden(idx, n_blocks)`` read-out).

Architecture: token embedding (tied output head), pre-norm blocks of causal multi-head attention (fused qkv with bias,
optional per-head q/k RMSNorm, interleaved-pair RoPE with base ``rope_theta``, optional value residual: block 0's
values are mixed into every later block with a learned scalar) and a SwiGLU (gate / up / down, no bias) or GELU MLP;
final norm. Module and parameter names match the reference so its ``model.safetensors`` loads strictly.

The LM is frozen inference: it runs once per caption batch outside the training step (or on a separate LM rank), so
it uses PyTorch matmuls. Two attention paths: padded rows with causal SDPA (``hidden``), and captions packed back
to back without padding (``hidden_packed``, reference aurora/slayer.py:326-432 for its HF LM): positions restart per
caption and the sm_100a varlen causal attention kernel keeps attention inside each caption, so the matmuls see only
real tokens. For real tokens both paths give the same states (up to bf16 rounding).
"""
import json
import os
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GPTConfig:
    vocab: int = 50304
    n_layer: int = 12
    n_embd: int = 768
    n_head: int = 12
    block: int = 1024
    norm: str = "rmsnorm"
    norm_eps: float = 1e-6
    pos: str = "rope"
    rope_theta: float = 100000.0
    ffn: str = "swiglu"
    ffn_mult: float = 8 / 3
    value_residual: bool = True
    qk_norm: bool = True

    @classmethod
    def from_dict(cls, d):
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


class RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        r = torch.rsqrt(x.float().square().mean(-1, keepdim=True) + self.eps)
        return x * r.to(x.dtype) * self.weight


def _norm(d, cfg):
    return RMSNorm(d, cfg.norm_eps) if cfg.norm == "rmsnorm" else nn.LayerNorm(d)


def rope_pairs(x, theta):
    """Rotate (even, odd) channel pairs of x [B, H, T, D] by position-dependent angles (base theta)."""
    T, D = x.shape[-2], x.shape[-1]
    inv = theta ** (-torch.arange(0, D, 2, device=x.device, dtype=torch.float32) / D)
    ang = torch.arange(T, device=x.device, dtype=torch.float32)[:, None] * inv[None]
    c, s = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
    a, b = x[..., 0::2], x[..., 1::2]
    return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)


def rope_pairs_at(x, pos, theta):
    """rope_pairs for packed tokens: x [T, H, D] at per-token positions pos [T]."""
    D = x.shape[-1]
    inv = theta ** (-torch.arange(0, D, 2, device=x.device, dtype=torch.float32) / D)
    ang = pos.to(torch.float32)[:, None] * inv[None]
    c, s = ang.cos().to(x.dtype)[:, None], ang.sin().to(x.dtype)[:, None]
    a, b = x[..., 0::2], x[..., 1::2]
    return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)


class SwiGLU(nn.Module):
    def __init__(self, d, hidden):
        super().__init__()
        self.gate = nn.Linear(d, hidden, bias=False)
        self.up = nn.Linear(d, hidden, bias=False)
        self.down = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class Block(nn.Module):
    def __init__(self, cfg, first):
        super().__init__()
        d = cfg.n_embd
        self.cfg, self.first, self.nh = cfg, first, cfg.n_head
        self.ln1, self.ln2 = _norm(d, cfg), _norm(d, cfg)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.mlp = SwiGLU(d, int(round(cfg.ffn_mult * d))) if cfg.ffn == "swiglu" else \
            nn.Sequential(nn.Linear(d, 4 * d), nn.GELU(), nn.Linear(4 * d, d))
        if cfg.value_residual and not first:
            self.vr_lambda = nn.Parameter(torch.zeros(1))
        if cfg.qk_norm:
            self.q_norm = RMSNorm(d // cfg.n_head, cfg.norm_eps)
            self.k_norm = RMSNorm(d // cfg.n_head, cfg.norm_eps)

    def forward(self, x, v_first=None):
        B, T, D = x.shape
        heads = lambda t: t.view(B, T, self.nh, D // self.nh).transpose(1, 2)
        q, k, v = (heads(t) for t in self.qkv(self.ln1(x)).split(D, dim=-1))
        if self.cfg.qk_norm:
            q, k = self.q_norm(q), self.k_norm(k)
        if self.cfg.pos == "rope":
            q, k = rope_pairs(q, self.cfg.rope_theta), rope_pairs(k, self.cfg.rope_theta)
        if self.cfg.value_residual:
            if self.first:
                v_first = v
            else:
                v = v + self.vr_lambda * v_first
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, D)
        x = x + self.proj(y)
        return x + self.mlp(self.ln2(x)), v_first

    def forward_packed(self, x, pos, cu, max_len, v_first=None):
        """x [T, D] of captions packed back to back (offsets cu, positions pos restarting per caption)."""
        from ..ops.fused import varlen_attention
        T, D = x.shape
        q, k, v = (t.view(T, self.nh, D // self.nh) for t in self.qkv(self.ln1(x)).split(D, dim=-1))
        if self.cfg.qk_norm:
            q, k = self.q_norm(q), self.k_norm(k)
        if self.cfg.pos == "rope":
            q, k = rope_pairs_at(q, pos, self.cfg.rope_theta), rope_pairs_at(k, pos, self.cfg.rope_theta)
        if self.cfg.value_residual:
            if self.first:
                v_first = v
            else:
                v = v + self.vr_lambda * v_first
        y = varlen_attention(q, k, v, cu, max_len, causal=True).to(x.dtype).reshape(T, D)
        x = x + self.proj(y)
        return x + self.mlp(self.ln2(x)), v_first


class GPT(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        self.tok = nn.Embedding(cfg.vocab, cfg.n_embd)
        if cfg.pos != "rope":
            self.pos = nn.Embedding(cfg.block, cfg.n_embd)
        self.blocks = nn.ModuleList([Block(cfg, i == 0) for i in range(cfg.n_layer)])
        self.lnf = _norm(cfg.n_embd, cfg)
        self.head = nn.Linear(cfg.n_embd, cfg.vocab, bias=False)
        self.head.weight = self.tok.weight

    def hidden(self, idx, n_blocks):
        """Residual stream after the first n_blocks blocks (no final norm, no head)."""
        x = self.tok(idx)
        if self.cfg.pos != "rope":
            x = x + self.pos(torch.arange(idx.shape[1], device=idx.device))[None]
        v_first = None
        for blk in self.blocks[:n_blocks]:
            x, v_first = blk(x, v_first)
        return x

    def forward(self, idx):
        return self.head(self.lnf(self.hidden(idx, len(self.blocks))))

    @torch.no_grad()
    def run_slice(self, x, lo, hi):
        """Blocks [lo, hi) for a pipeline's LM layer split. lo == 0: x are ids. Otherwise x is the previous
        slice's carry: the residual stream and block 0's values side by side (B, T, 2 n_embd), since the value
        residual of every later block reads them. Returns the carry, or the residual stream when hi is the end."""
        v_first = None
        if lo == 0:
            x = self.tok(x.long())
            if self.cfg.pos != "rope":
                x = x + self.pos(torch.arange(x.shape[1], device=x.device))[None]
        else:
            D = self.cfg.n_embd
            B, T = x.shape[:2]
            x, vf = x[..., :D], x[..., D:]
            if self.cfg.value_residual:
                v_first = vf.reshape(B, T, self.cfg.n_head, D // self.cfg.n_head).transpose(1, 2)
        for blk in self.blocks[lo:hi]:
            x, v_first = blk(x, v_first)
        if hi >= len(self.blocks):
            return x
        B, T, D = x.shape
        vf = v_first.transpose(1, 2).reshape(B, T, D) if v_first is not None else torch.zeros_like(x)
        return torch.cat([x, vf.to(x.dtype)], dim=-1)

    @torch.no_grad()
    def hidden_packed(self, seqs, n_blocks):
        """Residual stream after n_blocks blocks for captions given as 1-D id tensors, run as one packed sequence
        -> (sum of lengths, n_embd), captions back to back."""
        dev = self.tok.weight.device
        lens = [len(q) for q in seqs]
        ids = torch.cat(list(seqs)).to(dev, non_blocking=True).long()
        pos = torch.cat([torch.arange(n) for n in lens]).to(dev, non_blocking=True)
        cu = torch.tensor([0] + lens).cumsum(0).to(dev, dtype=torch.int32)
        x = self.tok(ids)
        if self.cfg.pos != "rope":
            x = x + self.pos(pos)
        v_first = None
        for blk in self.blocks[:n_blocks]:
            x, v_first = blk.forward_packed(x, pos, cu, max(lens), v_first)
        return x


def load_gpt(path):
    """(GPT, tokenizer.json path) from a local directory with config.json + model.safetensors (+ tokenizer.json)."""
    from safetensors.torch import load_model
    with open(os.path.join(path, "config.json")) as f:
        cfg = GPTConfig.from_dict(json.load(f))
    model = GPT(cfg)
    load_model(model, os.path.join(path, "model.safetensors"), strict=True)
    return model.requires_grad_(False).eval(), os.path.join(path, "tokenizer.json")
