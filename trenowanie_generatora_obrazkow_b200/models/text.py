"""Text encoders: the from-scratch GQA ``TextEncoder`` with a tied MLM head, and the ``LMTextEncoder`` refiner that
turns frozen-LM hidden states into denoiser text tokens.

Reference: TextAttention / TextBlock / TextEncoder aurora/model.py:113-145, :279-312; LMTextEncoder
aurora/slayer.py:152-235 (frozen LM kept outside the parameters, learned ``null`` vector for the CFG null prompt,
in_norm -> in_proj -> bidirectional TextBlocks -> norm -> out_proj). Parameter names match the reference.

Here the frozen LM is not part of the module: ``LMTextEncoder.forward`` takes its states (``lm_states``), computed
by whatever LM backend the caller runs (a frozen-LM server rank, a layer-split LM, or synthetic N(0, 1) states of the
LM's width in the benchmarks). Token ids are still accepted to derive the padding mask and null rows.
"""
import numpy as np
import torch
import torch.nn as nn

from ..ops import fused as Fz
from ..ops import reference as R
from .config import LMEncoderConfig, TextEncoderConfig

LM_PAD, LM_NULL = 65535, 65534
PAD_ID, BOS_ID, EOS_ID, NULL_ID, MASK_ID = 0, 2, 3, 4, 5


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


class TextAttention(nn.Module):
    def __init__(self, dim, heads, kv_heads, head_dim):
        super().__init__()
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.qkv = nn.Linear(dim, (heads + 2 * kv_heads) * head_dim, bias=False)
        self.out = nn.Linear(heads * head_dim, dim, bias=False)

    def forward(self, h, lens, cos, sin):
        o = Fz.self_attention_core(Fz.linear(h, self.qkv), self.heads, self.kv_heads, self.head_dim, None, None, cos,
                                   sin, lens)
        return Fz.linear(o, self.out)


class SwiGLU(nn.Module):
    def __init__(self, dim, hidden):
        super().__init__()
        self.in_proj = nn.Linear(dim, 2 * hidden, bias=False)
        self.out_proj = nn.Linear(hidden, dim, bias=False)

    def forward(self, h):
        return Fz.linear(Fz.swiglu(Fz.linear(h, self.in_proj)), self.out_proj)


class TextBlock(nn.Module):
    """Pre-norm block with ungated residuals."""

    def __init__(self, dim, heads, kv_heads, head_dim, mlp_hidden):
        super().__init__()
        self.norm1 = RMSNorm(dim)
        self.attn = TextAttention(dim, heads, kv_heads, head_dim)
        self.norm2 = RMSNorm(dim)
        self.mlp = SwiGLU(dim, mlp_hidden)

    def forward(self, x, pending, lens, cos, sin):
        x, h = Fz.adanorm(x, pending, None, self.norm1.weight)
        y = self.attn(h, lens, cos, sin)
        x, h = Fz.adanorm(x, y, None, self.norm2.weight)
        return x, self.mlp(h)


def _run_blocks(blocks, x, lens, cos, sin, final_norm, checkpoint=False):
    pending = None
    for blk in blocks:  # checkpoint: False, "full" (True) or "selective" (ops/fused.py run_block)
        x, pending = Fz.run_block(blk, (x, pending, lens, cos, sin), checkpoint)
    _, h = Fz.adanorm(x, pending, None, final_norm.weight)
    return h


class TextEncoder(nn.Module):
    """From-scratch text encoder: GQA transformer with 1D RoPE, SwiGLU, RMSNorm (reference aurora/model.py:279-312)."""

    def __init__(self, cfg: TextEncoderConfig = TextEncoderConfig()):
        super().__init__()
        self.config = cfg
        self.token_embedding = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.blocks = nn.ModuleList([TextBlock(cfg.dim, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.mlp_hidden)
                                     for _ in range(cfg.depth)])
        self.norm = RMSNorm(cfg.dim)
        self._rope = {}

    def null_ids(self):
        row = np.full(self.config.max_tokens, PAD_ID, dtype=np.int64)
        row[:3] = (BOS_ID, NULL_ID, EOS_ID)
        return row

    def rope(self, T, device):
        key = (T, str(device))
        if key not in self._rope:
            self._rope[key] = R.rope_1d_table(T, self.config.head_dim, device)
        return self._rope[key]

    def forward(self, ids):
        valid = ids.ne(self.config.pad_id)
        lens = R.valid_to_len(valid)
        h = self.token_embedding(ids)
        if h.is_cuda:
            h = h.to(torch.bfloat16)
        cos, sin = self.rope(ids.shape[1], ids.device)
        return _run_blocks(self.blocks, h, lens, cos, sin, self.norm), valid

    @torch.no_grad()
    def init_weights(self):
        nn.init.normal_(self.token_embedding.weight, std=0.02)
        for block in self.blocks:
            for lin in (block.attn.qkv, block.mlp.in_proj):
                nn.init.normal_(lin.weight, std=lin.in_features ** -0.5)
            nn.init.zeros_(block.attn.out.weight)
            nn.init.zeros_(block.mlp.out_proj.weight)


class LMTextEncoder(nn.Module):
    """Frozen-LM states -> trainable refiner -> denoiser text tokens (reference aurora/slayer.py:152-235)."""

    def __init__(self, cfg: LMEncoderConfig):
        super().__init__()
        self.config = cfg
        self.in_norm = RMSNorm(cfg.lm_dim)
        self.null = nn.Parameter(torch.zeros(1, 1, cfg.lm_dim))  # learned CFG null prompt
        self.in_proj = nn.Linear(cfg.lm_dim, cfg.dim, bias=False) if cfg.dim != cfg.lm_dim else nn.Identity()
        self.blocks = nn.ModuleList([TextBlock(cfg.dim, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.mlp_hidden)
                                     for _ in range(cfg.depth)])
        self.norm = RMSNorm(cfg.dim)
        out = getattr(cfg, "out_dim", 0)
        self.out_proj = nn.Linear(cfg.dim, out, bias=False) if out and out != cfg.dim else nn.Identity()
        self.checkpoint_blocks = False
        self._rope = {}

    def null_ids(self):
        row = np.full(self.config.max_tokens, LM_PAD, dtype=np.int64)
        row[0] = LM_NULL
        return row

    def rope(self, T, device):
        key = (T, str(device))
        if key not in self._rope:
            self._rope[key] = R.rope_1d_table(T, self.config.head_dim, device)
        return self._rope[key]

    @torch.no_grad()
    def init_weights(self):
        for block in self.blocks:
            for lin in (block.attn.qkv, block.mlp.in_proj):
                nn.init.normal_(lin.weight, std=lin.in_features ** -0.5)
            nn.init.zeros_(block.attn.out.weight)
            nn.init.zeros_(block.mlp.out_proj.weight)
        for lin in (self.in_proj, self.out_proj):
            if isinstance(lin, nn.Linear):
                nn.init.normal_(lin.weight, std=lin.in_features ** -0.5)

    def forward(self, ids=None, lm_states=None, valid=None, is_null=None):
        """ids (B, L) LM token rows (LM_PAD right padding, LM_NULL first for the null prompt) or, without ids,
        `valid` (B, L) bool and `is_null` (B,) bool. lm_states (B, L, lm_dim) frozen-LM states.
        Returns (text tokens (B, L, dim or out_dim), valid (B, L))."""
        assert lm_states is not None, "frozen-LM states must be passed in (the LM runs outside the refiner)"
        if ids is not None:
            valid = ids.ne(LM_PAD)
            is_null = ids[:, 0].eq(LM_NULL)
        B, L, _ = lm_states.shape
        if valid is None:
            valid = torch.ones(B, L, dtype=torch.bool, device=lm_states.device)
        lens = R.valid_to_len(valid)
        h = lm_states.to(torch.bfloat16) if lm_states.is_cuda else lm_states.float()
        _, h = Fz.adanorm(h.contiguous(), None, None, self.in_norm.weight)
        if is_null is not None:
            h = torch.where(is_null.to(h.device)[:, None, None], self.null.to(h.dtype).expand_as(h), h)
        if isinstance(self.in_proj, nn.Linear):
            h = Fz.linear(h, self.in_proj)
        cos, sin = self.rope(L, h.device)
        h = _run_blocks(self.blocks, h, lens, cos, sin, self.norm, self.checkpoint_blocks)
        if isinstance(self.out_proj, nn.Linear):
            h = Fz.linear(h, self.out_proj)
        return h, valid


def build_text_encoder(cfg):
    return LMTextEncoder(cfg) if isinstance(cfg, LMEncoderConfig) else TextEncoder(cfg)
