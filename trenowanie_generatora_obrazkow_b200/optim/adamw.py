"""AdamW whose CUDA step is one multi-tensor launch with the gradient-clip coefficient, the bf16 shadow refresh and
the EMA update fused in (csrc/optim.cu), and the on-device global gradient norm that feeds it.

State layout, hyper-parameters and math are torch.optim.AdamW's (amsgrad off, not maximised), so optimizer state
dicts load either way; CPU parameters use torch's implementation (tests). Reference usage being replaced:
``torch.optim.AdamW(fused=True)`` + ``clip_grad_norm_`` + ``torch._foreach_lerp_`` for the EMA (reference
train.py:338, 942, 966).
"""
import math

import torch

BLOCKS = 148 * 4


class DeviceTables:
    """Small host tables mirrored on the device, re-uploaded only when their contents change."""

    def __init__(self):
        self._t = {}

    def get(self, key, rows, dtype, device, width):
        t = self._t.get(key)
        if t is None or t[0] != rows:
            dev = torch.tensor(rows if rows else [[0] * width], dtype=dtype).reshape(-1, width)
            dev = dev[: len(rows)].to(device)
            t = (rows, dev)
            self._t[key] = t
        return t[1]


def shadow_ptr(p):
    """Address of p's bf16 shadow when one is cached and current (0 otherwise: it will be rebuilt on use)."""
    ent = getattr(p, "_tgo_bf16", None)
    if ent is None or ent[0] != p._version or ent[1].device != p.device or ent[1].shape != p.shape:
        return 0
    return ent[1].data_ptr()


def after_raw_update(params):
    """Parameters were changed by raw-pointer kernels that also refreshed their bf16 shadows: drop the other
    derived copies (the interleaved SwiGLU weight) so they are rebuilt from the new values."""
    for p in params:
        if getattr(p, "_tgo_swiglu", None) is not None:
            p._tgo_swiglu = None


class GradNorm:
    """Global L2 norm of a list of fp32 gradients and the clip coefficient min(1, clip / (norm + 1e-6)), computed
    on the device in one launch (no host synchronisation, gradients left unscaled)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.acc = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.gnorm = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.coef = torch.ones(1, dtype=torch.float32, device=self.device)
        self.tables = DeviceTables()

    def __call__(self, grads, clip, extra_sumsq=None):
        from ..ops._ext import ext
        rows = [(g.data_ptr(), g.numel()) for g in grads]
        segs = self.tables.get("g", rows, torch.int64, self.device, 2)
        ext().grad_norm(segs, self.acc, self.counter, extra_sumsq, float(clip), self.gnorm, self.coef, BLOCKS)
        return self.gnorm.reshape(()), self.coef


class FusedAdamW(torch.optim.AdamW):
    """torch.optim.AdamW with a fused CUDA step (module docstring). ``step(coef=..., ema=..., ema_rate=...)``:
    coef scales the gradients first (device scalar or float); ema is an optim.groups.EMA whose tensors for these
    parameters are updated in the same launch with e += ema_rate (p - e) (and marked done for this step)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, fused=False,
                         foreach=False)
        self.tables = DeviceTables()

    def _device_ok(self):
        return all(p.is_cuda and p.dtype == torch.float32 and (p.grad is None or (
            p.grad.dtype == torch.float32 and p.grad.is_contiguous())) for g in self.param_groups for p in g["params"])

    @torch.no_grad()
    def step(self, closure=None, coef=None, ema=None, ema_rate=0.0):
        if closure is not None:
            with torch.enable_grad():
                closure()
        if not self._device_ok():
            if coef is not None:
                grads = [p.grad for g in self.param_groups for p in g["params"] if p.grad is not None]
                if grads:
                    torch._foreach_mul_(grads, coef.to(grads[0].device) if torch.is_tensor(coef) else float(coef))
            super().step()
            if ema is not None:  # EMA of these parameters, unfused
                for g in self.param_groups:
                    for p in g["params"]:
                        e = ema.lookup(p)
                        if e is not None:
                            e.lerp_(p.detach().float(), ema_rate)
                            ema.mark_fused(p)
            return
        from ..ops._ext import ext
        rows, hyper, dev = [], [], None
        for gi, g in enumerate(self.param_groups):
            if g.get("amsgrad") or g.get("maximize"):
                raise ValueError("FusedAdamW: amsgrad / maximize are not supported")
            b1, b2 = g["betas"]
            step_n = None
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["step"] = torch.zeros((), dtype=torch.float32)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                step_n = float(st["step"])
                e = ema.lookup(p) if ema is not None else None
                if e is not None:
                    ema.mark_fused(p)
                rows.append((p.data_ptr(), p.grad.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(),
                             shadow_ptr(p), 0 if e is None else e.data_ptr(), p.numel(), gi))
                dev = p.device
            if step_n is None:
                hyper.append((1.0, 0.0, 1.0, 1.0, b1, b2))
                continue
            bc1 = 1 - b1 ** step_n
            bc2 = 1 - b2 ** step_n
            hyper.append((1 - g["lr"] * g["weight_decay"], g["lr"] / bc1, 1 / math.sqrt(bc2), g["eps"], b1, b2))
        if not rows:
            return
        segs = self.tables.get("segs", rows, torch.int64, dev, 8)
        hyp = torch.tensor(hyper, dtype=torch.float32).pin_memory().to(dev, non_blocking=True)
        c = None
        if coef is not None:
            c = coef.reshape(1).float() if torch.is_tensor(coef) else torch.full((1,), float(coef), device=dev)
        ext().adamw(segs, hyp, c, float(ema_rate), BLOCKS)
        after_raw_update([p for g in self.param_groups for p in g["params"]])
