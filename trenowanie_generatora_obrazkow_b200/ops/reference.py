"""fp32 PyTorch oracles of every op the kernels implement (CPU path and numerics reference of the GPU tests).

The math is the reference's (aurora/model.py): RMSNorm :27-34, interleaved-pair RoPE :37-50 and :98-99, 2D RoPE
:53-72, RPE-2D coordinates :75-80, micro-conditioning :83-95, SwiGLU :102-110, attention :113-188, time embedding
:213-218. Layout differs: activations are [batch, token, head, head_dim] and RoPE tables are [token, head_dim]
(or [batch, token, head_dim] for per-sample coordinates).
"""
import math

import torch
import torch.nn.functional as F

EPS = 1e-6


def rmsnorm(x, w, eps=EPS):
    """x * rsqrt(mean(x^2) + eps) * w, the statistic in fp32 and the scale cast back to x's dtype."""
    return x * torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps).to(x.dtype) * w


def rotate_pairs(x):
    """(x0, x1, x2, x3, ...) -> (-x1, x0, -x3, x2, ...)."""
    ev, od = x[..., 0::2], x[..., 1::2]
    return torch.stack((-od, ev), dim=-1).flatten(-2)


def apply_rope(x, cos, sin):
    """x [B, T, H, d]; cos / sin [T, d] or [B, T, d] (already duplicated per pair)."""
    if cos.dim() == 2:
        cos, sin = cos[None, :, None], sin[None, :, None]
    else:
        cos, sin = cos[:, :, None], sin[:, :, None]
    return x * cos.to(x.dtype) + rotate_pairs(x) * sin.to(x.dtype)


def _dup(a):
    return a.repeat_interleave(2, dim=-1)


def rope_1d_table(n, d, device=None):
    """1D RoPE for positions 0..n-1: inv_freq = 10000^(-2i/d) -> cos, sin [n, d]."""
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))
    ang = torch.arange(n, dtype=torch.float32, device=device)[:, None] * inv
    return _dup(ang.cos()), _dup(ang.sin())


def rope_2d_from_coords(rows, cols, d):
    """(B, h) row and (B, w) column positions -> cos, sin [B, h*w, d]: the first half of the head dim rotates with
    the row, the second half with the column; tokens are row-major."""
    b, h, w = rows.shape[0], rows.shape[1], cols.shape[1]
    inv = 1.0 / (10000 ** (torch.arange(0, d // 2, 2, dtype=torch.float32, device=rows.device) / (d // 2)))
    ar = (rows.float()[:, :, None] * inv)[:, :, None].expand(b, h, w, -1)
    ac = (cols.float()[:, :, None] * inv)[:, None].expand(b, h, w, -1)
    ang = torch.cat([ar, ac], dim=-1).reshape(b, h * w, -1)
    return _dup(ang.cos()), _dup(ang.sin())


def grid_coords(side, ref=0, device=None):
    """Positions of `side` tokens along one axis; ref > 0 spreads them over a ref-token field
    ((i + 0.5) * ref / side - 0.5, position interpolation)."""
    c = torch.arange(side, dtype=torch.float32, device=device)
    if ref and ref != side:
        c = (c + 0.5) * (ref / side) - 0.5
    return c


def rope_2d_table(h, w, d, ref=0, device=None):
    """2D RoPE of an h x w grid -> cos, sin [h*w, d]."""
    cos, sin = rope_2d_from_coords(grid_coords(h, ref, device)[None], grid_coords(w, ref, device)[None], d)
    return cos[0], sin[0]


def random_rope_coords(b, side, field, device=None, generator=None):
    """RPE-2D (arXiv:2503.18719): per sample and axis `side` sorted distinct integer positions of 0..field-1."""
    def axis():
        r = torch.rand(b, field, device=device, generator=generator)
        return r.topk(side, dim=1).indices.sort(dim=1).values
    return axis(), axis()


def timestep_embedding(t, dim=256):
    """t * 1000 -> [sin, cos] with freqs exp(-ln(1e4) i / (half - 1))."""
    t = t.float() * 1000.0
    half = dim // 2
    freqs = torch.exp(-math.log(10000) * torch.arange(half, device=t.device).float() / max(half - 1, 1))
    ang = t[:, None] * freqs[None]
    return torch.cat([ang.sin(), ang.cos()], dim=-1)


def micro_cond_embedding(cond, dim=256):
    """(B, 8) micro-conditions in pixels -> (B, 8 * dim) sinusoids with freqs exp(-ln(1e4) i / half)."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000) * torch.arange(half, device=cond.device).float() / half)
    ang = cond.float()[:, :, None] * freqs
    return torch.cat([ang.sin(), ang.cos()], dim=-1).flatten(1)


def default_micro_cond(base, res, b, device=None):
    """Micro-conditions of a whole uncropped image: [orig_h, orig_w, top, left, bottom, right, tgt_h, tgt_w]."""
    o = max(base, res)
    return torch.tensor([o, o, 0, 0, o, o, res, res], dtype=torch.float32, device=device).expand(b, 8)


def attention(q, k, v, kv_len=None, scale=None):
    """q [B, Tq, Hq, d], k / v [B, Tk, Hkv, d] (Hq % Hkv == 0), keys >= kv_len[b] masked -> [B, Tq, Hq, d]."""
    B, Tq, Hq, d = q.shape
    Hkv = k.shape[2]
    rep = Hq // Hkv
    qh = q.transpose(1, 2)
    kh = k.transpose(1, 2).repeat_interleave(rep, dim=1)
    vh = v.transpose(1, 2).repeat_interleave(rep, dim=1)
    mask = None
    if kv_len is not None:
        mask = (torch.arange(k.shape[1], device=q.device)[None] < kv_len.to(q.device)[:, None])[:, None, None, :]
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, scale=scale)
    return o.transpose(1, 2)


def varlen_attention(q, k, v, cu_seqlens, causal=True, scale=None):
    """Packed sequences: q [T, Hq, d], k / v [T, Hkv, d], cu_seqlens [n + 1] token offsets; attention stays inside
    each sequence (causal: key <= query position) -> [T, Hq, d]."""
    out = torch.empty_like(q)
    cu = [int(c) for c in cu_seqlens.tolist()]
    for a, b in zip(cu[:-1], cu[1:]):
        if b <= a:
            continue
        qh, kh, vh = (x[a:b].transpose(0, 1) for x in (q, k, v))
        rep = qh.shape[0] // kh.shape[0]
        kh, vh = kh.repeat_interleave(rep, 0), vh.repeat_interleave(rep, 0)
        out[a:b] = F.scaled_dot_product_attention(qh, kh, vh, is_causal=causal, scale=scale).transpose(0, 1)
    return out


def swiglu(ab):
    a, b = ab.chunk(2, dim=-1)
    return F.silu(a) * b


def valid_to_len(valid):
    """Boolean key mask [B, L] (a prefix per row, captions are right-padded) -> int32 lengths [B]."""
    return valid.sum(dim=1).to(torch.int32)
