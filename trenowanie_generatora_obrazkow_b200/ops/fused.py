"""Differentiable fused ops used by the models.

CUDA tensors run the sm_100a kernels (csrc/); CPU tensors run the fp32 oracles of ``reference.py`` under ordinary
autograd. Each CUDA op is a ``torch.autograd.Function`` whose backward is a hand-written kernel too:

* ``linear``        tcgen05 GEMM forward / dgrad; the weight gradient is accumulated in fp32 straight into
                    ``weight.grad`` by the GEMM epilogue (the grad never exists in bf16). Weights are read from a
                    bf16 shadow copy refreshed whenever the fp32 master changes (``bf16_weight``).
* ``adanorm``       residual update + RMSNorm + adaLN modulation (DenoiserBlock, reference aurora/model.py:204-210);
                    the norm weight's gradient is accumulated in place into ``weight.grad`` (fp32) like the linear
                    weights', so ``torch.autograd.grad`` does not return it: read ``weight.grad``.
* ``self_attention_core``  per-head q/k RMSNorm + RoPE + flash attention, reading q/k/v from the fused qkv rows (the
                    q / k norm weights' gradients likewise go to their ``.grad``).
* ``cross_attention_core`` flash attention against text keys/values with a key-length mask.
* ``swiglu``        silu(a) * b.
* ``varlen_attention`` packed variable-length (causal) attention for the frozen caption LM (inference only).
"""
import torch

from . import reference as R
from ._ext import err_buf, ext
from .gemm import gemm

# ----------------------------------------------------------------------------------------------------------------
# bf16 shadow weights and gradient-ready callbacks
# ----------------------------------------------------------------------------------------------------------------
_GRAD_HOOKS = []


def bf16_weight(p):
    """bf16 copy of a floating parameter, kept on the parameter object and recomputed when the parameter changed in
    place (its version counter moved) or moved to another device."""
    if p.dtype == torch.bfloat16:
        return p.detach()
    ent = getattr(p, "_tgo_bf16", None)
    ver = p._version
    if ent is None or ent[0] != ver or ent[1].device != p.device or ent[1].shape != p.shape:
        w = p.detach().to(torch.bfloat16)
        p._tgo_bf16 = (ver, w)
        return w
    return ent[1]


def swiglu_weight(p):
    """bf16 copy of a (2H, D) gate | up weight with the gate and up rows interleaved in blocks of 128 (the layout of
    the fused up projection + SwiGLU GEMM), cached like bf16_weight."""
    ent = getattr(p, "_tgo_swiglu", None)
    ver = p._version
    if ent is None or ent[0] != ver or ent[1].device != p.device:
        H = p.shape[0] // 2
        w = p.detach().to(torch.bfloat16)
        w = torch.stack([w[:H].view(H // 128, 128, -1), w[H:].view(H // 128, 128, -1)], 1).reshape(2 * H, -1)
        p._tgo_swiglu = (ver, w.contiguous())
        return p._tgo_swiglu[1]
    return ent[1]


def up_swiglu(x, layer):
    """silu(x Wg^T) * (x Wu^T) for an nn.Linear of (2H, D) gate | up rows. On CUDA without autograd (sampling) and
    H % 128 == 0: one GEMM whose epilogue applies the SwiGLU (the (M, 2H) product never reaches memory)."""
    w = layer.weight
    H = w.shape[0] // 2
    if x.is_cuda and not (torch.is_grad_enabled() and (x.requires_grad or w.requires_grad)) and H % 128 == 0:
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        out = torch.empty(x2.shape[0], H, device=x.device, dtype=torch.bfloat16)
        ext().gemm_swiglu(x2, swiglu_weight(w), out, err_buf(x.device))
        return out.view(*x.shape[:-1], H)
    return swiglu(linear(x, layer))


def set_bf16_weight(p, w):
    """Register an externally produced bf16 copy of p (e.g. written by a fused optimizer kernel)."""
    p._tgo_bf16 = (p._version, w)


def add_grad_ready_hook(fn):
    """fn(param) is called right after a weight gradient was accumulated into ``param.grad`` by a fused op."""
    _GRAD_HOOKS.append(fn)
    return fn


def remove_grad_ready_hook(fn):
    if fn in _GRAD_HOOKS:
        _GRAD_HOOKS.remove(fn)


def _grad_buffer(p):
    if p.grad is None:
        p.grad = torch.zeros_like(p, dtype=torch.float32)
    return p.grad


def _notify(p):
    for fn in _GRAD_HOOKS:
        fn(p)


def _weight_grad_target(w):
    """Where a fused backward accumulates (+=) the gradient of a small fp32 weight (norm weights): the parameter's
    own gradient buffer, so no zero-filled temporary and no autograd accumulation kernel run per use; the autograd
    function then returns None for it and calls ``_weight_grad_done``. Falls back to a temporary (returned
    through autograd) when the buffer cannot take the sum in place."""
    if w.requires_grad and w.is_leaf and w.dtype == torch.float32 and (w.grad is None or (
            w.grad.dtype == torch.float32 and w.grad.is_contiguous())):
        return _grad_buffer(w), True
    return torch.zeros_like(w, dtype=torch.float32), False


def _weight_grad_done(w, direct, g):
    """(autograd's gradient for w): None when it was accumulated in place (and the ready hooks ran)."""
    if direct:
        _notify(w)
        return None
    return g if w.requires_grad else None


# ----------------------------------------------------------------------------------------------------------------
# selective activation checkpointing
# ----------------------------------------------------------------------------------------------------------------
# Keep what the backward needs from the GEMMs and attention, rebuild the elementwise results (reference
# train_pp.py:271-287, whose policy saves matmul / attention outputs and recomputes the rest). Here the elementwise
# results that autograd functions save are tagged with a recipe: the adanorm output (saved by the next linear), the
# normalised + rotated q and k (saved by attention) and the SwiGLU output (saved by the down projection). Under
# ``selective_recompute()`` a saved-tensor hook stores a tagged tensor as its recipe, which the backward runs again
# from tensors that are saved anyway (the residual stream, q/k/v, the up projection's output); everything else is
# saved as usual, so no GEMM or attention is recomputed.
_SAC_ACTIVE = [0]


class _Recipe:
    """Rebuilds one or more tensors at most once (q and k share one kernel launch)."""
    __slots__ = ("fn", "outs")

    def __init__(self, fn):
        self.fn, self.outs = fn, None

    def get(self, i):
        if self.outs is None:
            self.outs = self.fn()
        return self.outs[i]


class _Rebuild:
    __slots__ = ("recipe", "index", "shape")

    def __init__(self, recipe, index, shape):
        self.recipe, self.index, self.shape = recipe, index, shape


def _tag(t, recipe, index=0):
    if _SAC_ACTIVE[0]:
        t._tgo_recipe = (recipe, index, None)
    return t


def _tag_view(view, base):
    """A view of a tagged tensor (same storage and start) is rebuilt the same way, then reshaped."""
    r = getattr(base, "_tgo_recipe", None)
    if r is not None and view is not base and view.data_ptr() == base.data_ptr():
        view._tgo_recipe = (r[0], r[1], tuple(view.shape))


def _pack(t):
    r = getattr(t, "_tgo_recipe", None)
    return t if r is None else _Rebuild(*r)


def _unpack(x):
    if not isinstance(x, _Rebuild):
        return x
    out = x.recipe.get(x.index)
    return out if x.shape is None else out.reshape(x.shape)


class selective_recompute:
    """Context of a block's forward under selective activation checkpointing (see above)."""

    def __enter__(self):
        self._hooks = torch.autograd.graph.saved_tensors_hooks(_pack, _unpack)
        self._hooks.__enter__()
        _SAC_ACTIVE[0] += 1
        return self

    def __exit__(self, *exc):
        _SAC_ACTIVE[0] -= 1
        return self._hooks.__exit__(*exc)


def run_block(block, args, mode):
    """block(*args) with activation checkpointing: mode None / False (none), "full" / True (recompute the whole
    block in the backward) or "selective" (recompute only its elementwise results)."""
    if not mode or not torch.is_grad_enabled():
        return block(*args)
    if mode == "selective":
        with selective_recompute():
            return block(*args)
    return torch.utils.checkpoint.checkpoint(block, *args, use_reentrant=False)


# ----------------------------------------------------------------------------------------------------------------
# linear
# ----------------------------------------------------------------------------------------------------------------
class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, w16):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        _tag_view(x2, x)
        y = gemm(x2, w16)
        ctx.save_for_backward(x2, w16)
        ctx.weight = weight
        ctx.in_shape = x.shape
        ctx.in_dtype = x.dtype
        return y.view(*x.shape[:-1], w16.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w16 = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.dtype != torch.bfloat16:
            dy2 = dy2.to(torch.bfloat16)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, w16, b_mn=True).view(ctx.in_shape)
            if ctx.in_dtype != torch.bfloat16:
                dx = dx.to(ctx.in_dtype)
        weight = ctx.weight
        if weight.requires_grad:
            g = _grad_buffer(weight)
            gemm(dy2, x2, out=g, a_mn=True, b_mn=True, accumulate=True)
            _notify(weight)
        return dx, None, None


def linear(x, layer_or_weight, bias=None):
    """y = x @ W^T (+ b). Accepts an ``nn.Linear`` (its weight and bias) or a weight tensor."""
    if isinstance(layer_or_weight, torch.nn.Linear):
        weight, bias = layer_or_weight.weight, layer_or_weight.bias
    else:
        weight = layer_or_weight
    if not x.is_cuda:
        return torch.nn.functional.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))
    y = _LinearFn.apply(x, weight, bf16_weight(weight))
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y


# ----------------------------------------------------------------------------------------------------------------
# adanorm
# ----------------------------------------------------------------------------------------------------------------
def _opt(t):
    return t if t is not None else None


class _AdaNormFn(torch.autograd.Function):
    """(x, y, gate, w, shift, scale) -> (x_new, h); x_new = x + gate * y (or x + y); only used with y given."""

    @staticmethod
    def forward(ctx, x, y, gate, w, shift, scale, eps):
        B, T, D = x.shape
        x_new, h, rstd = ext().adanorm_fwd(x, y, gate, w, shift, scale, T, eps)
        ctx.save_for_backward(x_new, rstd, w, scale, y, gate)
        ctx.T = T
        ctx.has_mod = shift is not None
        ctx.w_param = w
        return x_new, h

    @staticmethod
    def backward(ctx, dx_new, dh):
        x_new, rstd, w, scale, y, gate = ctx.saved_tensors
        if dh is None:
            dh = torch.zeros_like(x_new)
        dw, direct = _weight_grad_target(ctx.w_param)
        dxe = dx_new.contiguous() if dx_new is not None else None
        dx, dy, dshift, dscale, dgate = ext().adanorm_bwd(dh.contiguous(), dxe, x_new, rstd, w, dw, scale, y, gate,
                                                          ctx.T)
        if dy is None:
            dy = dx  # ungated residual: d(branch) == d(x_new)
        return dx, dy, dgate, _weight_grad_done(ctx.w_param, direct, dw), dshift, dscale, None


class _NormModFn(torch.autograd.Function):
    """x -> h = rmsnorm(x) * w * (1 + scale) + shift (no residual update)."""

    @staticmethod
    def forward(ctx, x, w, shift, scale, eps):
        B, T, D = x.shape
        _, h, rstd = ext().adanorm_fwd(x, None, None, w, shift, scale, T, eps)
        ctx.save_for_backward(x, rstd, w, scale)
        ctx.T = T
        ctx.w_param = w
        return h

    @staticmethod
    def backward(ctx, dh):
        x, rstd, w, scale = ctx.saved_tensors
        dw, direct = _weight_grad_target(ctx.w_param)
        dx, _, dshift, dscale, _ = ext().adanorm_bwd(dh.contiguous(), None, x, rstd, w, dw, scale, None, None, ctx.T)
        return dx, _weight_grad_done(ctx.w_param, direct, dw), dshift, dscale, None


def adanorm(x, y, gate, w, shift=None, scale=None, eps=R.EPS):
    """x_new = x + gate * y (y None: x_new = x; gate None: x + y); h = rmsnorm(x_new) * w * (1 + scale) + shift.

    x, y: [B, T, D]; gate, shift, scale: [B, D] (per-sample rows, may be strided views); w: [D] fp32.
    Returns (x_new, h).
    """
    if not x.is_cuda:
        xn = x if y is None else (x + (y if gate is None else gate[:, None] * y))
        h = R.rmsnorm(xn, w, eps)
        if scale is not None:
            h = h * (1 + scale[:, None]) + shift[:, None]
        return xn, h
    x = x.contiguous()
    if y is None:
        h = _NormModFn.apply(x, w, shift, scale, eps)
        x_new = x
    else:
        x_new, h = _AdaNormFn.apply(x, y.contiguous(), gate, w, shift, scale, eps)
    if _SAC_ACTIVE[0]:  # h = rmsnorm(x_new) w (1 + scale) + shift, rebuilt from the residual stream
        T, xd = x.shape[1], x_new.detach()
        sd = None if shift is None else shift.detach()
        cd = None if scale is None else scale.detach()
        _tag(h, _Recipe(lambda: (ext().adanorm_fwd(xd, None, None, w.detach(), sd, cd, T, eps)[1],)))
    return x_new, h


# ----------------------------------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------------------------------
def _rope_arg(cos):
    if cos is None:
        return None
    return cos.contiguous().float()


class _SelfAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, q_w, k_w, cos, sin, kv_len, hq, hkv, hd, scale, eps):
        B, T, C = qkv.shape
        q2 = qkv.view(B * T, C)
        q, k, rq, rk = ext().qknorm_rope_fwd(q2, hq, hkv, hd, q_w, k_w, cos, sin, T, eps)
        q4 = q.view(B, T, hq, hd)
        k4 = k.view(B, T, hkv, hd)
        v4 = qkv[:, :, (hq + hkv) * hd:(hq + 2 * hkv) * hd].unflatten(-1, (hkv, hd))
        o, lse = ext().attention_fwd(q4, k4, v4, kv_len, scale, None, err_buf(q4.device))
        if _SAC_ACTIVE[0]:  # normalised + rotated q, k: one kernel rebuilds both from qkv
            q2d = q2.detach()
            rec = _Recipe(lambda: ext().qknorm_rope_fwd(q2d, hq, hkv, hd, q_w, k_w, cos, sin, T, eps)[:2])
            _tag(q, rec, 0)
            _tag(k, rec, 1)
        ctx.save_for_backward(qkv, q, k, o, lse, rq, rk, q_w, k_w, cos, sin, kv_len)
        ctx.dims = (hq, hkv, hd, scale)
        ctx.q_param, ctx.k_param = q_w, k_w
        return o.view(B, T, hq * hd)

    @staticmethod
    def backward(ctx, do):
        qkv, q, k, o, lse, rq, rk, q_w, k_w, cos, sin, kv_len = ctx.saved_tensors
        hq, hkv, hd, scale = ctx.dims
        B, T, C = qkv.shape
        do = do.contiguous().view(B, T, hq, hd)
        dqkv = torch.empty_like(qkv)
        # fp32 dq: the attention backward hands over its accumulator and the q/k-norm backward reads it, so no
        # separate fp32 -> bf16 pass runs in between
        dq = torch.empty(q.shape, device=q.device, dtype=torch.float32)
        dk = torch.empty_like(k)
        dv4 = dqkv[:, :, (hq + hkv) * hd:(hq + 2 * hkv) * hd].unflatten(-1, (hkv, hd))
        q4, k4 = q.view(B, T, hq, hd), k.view(B, T, hkv, hd)
        v4 = qkv[:, :, (hq + hkv) * hd:(hq + 2 * hkv) * hd].unflatten(-1, (hkv, hd))
        ext().attention_bwd(q4, k4, v4, o, lse, do, kv_len, scale, dq.view(B, T, hq, hd), dk.view(B, T, hkv, hd), dv4,
                            err_buf(q.device))
        dwq, dq_direct = _weight_grad_target(ctx.q_param) if q_w is not None else (None, False)
        dwk, dk_direct = _weight_grad_target(ctx.k_param) if k_w is not None else (None, False)
        ext().qknorm_rope_bwd(qkv.view(B * T, C), hq, hkv, hd, q_w, k_w, cos, sin, T, rq, rk, dq, dk,
                              dqkv.view(B * T, C), dwq, dwk)
        if q_w is not None:
            dwq = _weight_grad_done(ctx.q_param, dq_direct, dwq)
        if k_w is not None:
            dwk = _weight_grad_done(ctx.k_param, dk_direct, dwk)
        return dqkv, dwq, dwk, None, None, None, None, None, None, None, None


def self_attention_core(qkv, heads, kv_heads, head_dim, q_w=None, k_w=None, cos=None, sin=None, kv_len=None,
                        scale=None, eps=R.EPS):
    """qkv [B, T, (heads + 2 kv_heads) * head_dim] -> attention output [B, T, heads * head_dim].

    q / k get a per-head RMSNorm when q_w / k_w are given, then RoPE when cos / sin are given ([T, d] or
    [B, T, d]); keys at positions >= kv_len[b] are masked.
    """
    scale = head_dim ** -0.5 if scale is None else scale
    B, T, _ = qkv.shape
    if not qkv.is_cuda:
        q, k, v = qkv.split([heads * head_dim, kv_heads * head_dim, kv_heads * head_dim], dim=-1)
        q = q.view(B, T, heads, head_dim)
        k = k.view(B, T, kv_heads, head_dim)
        v = v.view(B, T, kv_heads, head_dim)
        if q_w is not None:
            q, k = R.rmsnorm(q, q_w, eps), R.rmsnorm(k, k_w, eps)
        if cos is not None:
            q, k = R.apply_rope(q, cos, sin), R.apply_rope(k, cos, sin)
        return R.attention(q, k, v, kv_len, scale).reshape(B, T, heads * head_dim)
    return _SelfAttnFn.apply(qkv.contiguous(), q_w, k_w, _rope_arg(cos), _rope_arg(sin), kv_len, heads, kv_heads,
                             head_dim, float(scale), eps)


class _CrossAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, kv, kv_len, heads, head_dim, scale):
        B, T, D = q.shape
        L = kv.shape[1]
        q4 = q.view(B, T, heads, head_dim)
        k4 = kv[:, :, :D].unflatten(-1, (heads, head_dim))
        v4 = kv[:, :, D:].unflatten(-1, (heads, head_dim))
        o, lse = ext().attention_fwd(q4, k4, v4, kv_len, scale, None, err_buf(q4.device))
        ctx.save_for_backward(q, kv, o, lse, kv_len)
        ctx.dims = (heads, head_dim, scale)
        return o.view(B, T, D)

    @staticmethod
    def backward(ctx, do):
        q, kv, o, lse, kv_len = ctx.saved_tensors
        heads, head_dim, scale = ctx.dims
        B, T, D = q.shape
        do = do.contiguous().view(B, T, heads, head_dim)
        dq = torch.empty_like(q)
        dkv = torch.empty_like(kv)
        q4 = q.view(B, T, heads, head_dim)
        k4 = kv[:, :, :D].unflatten(-1, (heads, head_dim))
        v4 = kv[:, :, D:].unflatten(-1, (heads, head_dim))
        ext().attention_bwd(q4, k4, v4, o, lse, do, kv_len, scale, dq.view(B, T, heads, head_dim),
                            dkv[:, :, :D].unflatten(-1, (heads, head_dim)),
                            dkv[:, :, D:].unflatten(-1, (heads, head_dim)), err_buf(q.device))
        return dq, dkv, None, None, None, None


def cross_attention_core(q, kv, heads, kv_len=None, scale=None):
    """q [B, T, D] (heads of D / heads), kv [B, L, 2D] = [k | v] -> [B, T, D]; keys >= kv_len[b] masked."""
    B, T, D = q.shape
    hd = D // heads
    scale = hd ** -0.5 if scale is None else scale
    if not q.is_cuda:
        k, v = kv.chunk(2, dim=-1)
        L = kv.shape[1]
        return R.attention(q.view(B, T, heads, hd), k.reshape(B, L, heads, hd), v.reshape(B, L, heads, hd), kv_len,
                           scale).reshape(B, T, D)
    return _CrossAttnFn.apply(q.contiguous(), kv.contiguous(), kv_len, heads, hd, float(scale))


@torch.no_grad()
def varlen_attention(q, k, v, cu_seqlens, max_len=None, causal=True, scale=None):
    """Captions packed back to back without padding (reference aurora/slayer.py:326-342, varlen flash attention):
    q [T, Hq, d], k / v [T, Hkv, d], cu_seqlens int32 [n + 1]; attention stays inside each sequence."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    if not q.is_cuda:
        return R.varlen_attention(q, k, v, cu_seqlens, causal, scale)
    if max_len is None:
        max_len = int((cu_seqlens[1:] - cu_seqlens[:-1]).max())
    cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
    o, _ = ext().attention_varlen_fwd(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), cu,
                                      int(max_len), float(scale), bool(causal), err_buf(q.device))
    return o


# ----------------------------------------------------------------------------------------------------------------
# swiglu
# ----------------------------------------------------------------------------------------------------------------
class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ab):
        ab = ab.contiguous()
        ctx.save_for_backward(ab)
        return ext().swiglu_fwd(ab)

    @staticmethod
    def backward(ctx, dg):
        (ab,) = ctx.saved_tensors
        return ext().swiglu_bwd(ab, dg.contiguous())


def fm_inputs(x0, eps, t):
    """Flow-matching input and target, token-major [B, H*W, C]: z_t = (1 - t) x0 + t eps (bf16 on CUDA, the
    patch-in GEMM's input) and eps - x0 (fp32), from fp32 [B, C, H, W] latents; one kernel on CUDA."""
    if x0.is_cuda:
        z_tok, target = ext().fm_inputs(x0.float().contiguous(), eps.float().contiguous(), t.float().contiguous())
        return z_tok, target
    tt = t.view(-1, 1, 1, 1)
    tok = lambda a: a.flatten(2).transpose(1, 2)
    return tok((1 - tt) * x0 + tt * eps), tok(eps - x0)


def swiglu(ab):
    if not ab.is_cuda:
        return R.swiglu(ab)
    ab = ab.contiguous()
    g = _SwiGLUFn.apply(ab)
    if _SAC_ACTIVE[0]:  # rebuilt from the up projection's output (saved by the SwiGLU backward)
        _tag(g, _Recipe(lambda: (ext().swiglu_fwd(ab.detach()),)))
    return g
