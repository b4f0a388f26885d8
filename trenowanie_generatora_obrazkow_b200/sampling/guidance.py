"""Guidance variants of the Euler flow-matching sampler, for side-by-side evaluation grids (reference
tests/guidance_grid.py):

  cfg       v = v_u + w (v_c - v_u)                                   (the default sampler)
  cfgzero   CFG-Zero* (Fan et al. 2025, arXiv:2503.18886): per sample s* = <v_c, v_u> / |v_u|^2,
            v = s* v_u + w (v_c - s* v_u), and the first step is skipped (zero-init)
  ag        autoguidance (Karras et al. 2024, arXiv:2406.02507): a weaker model with the same prompt replaces the
            unconditional branch, v = v_bad + w (v_c - v_bad); it brings its own text encoding
Options: shift (time grid t = s u / (1 + (s - 1) u)) and off (no guidance while t <= off: the conditional velocity
alone on the last, lowest-noise steps).
"""
import torch

from .euler import time_grid


@torch.no_grad()
def guided_latents(den, text, text_len, null_text, null_len, noise, steps=50, w=3.0, method="cfg", shift=1.0,
                   off=-1.0, guide=None):
    """noise (B, C, h, w); text / text_len of the prompts, null_text / null_len of the null prompt (cfg, cfgzero);
    guide = (bad denoiser, its text, its text_len) for method "ag". Returns fp32 latents."""
    B = noise.shape[0]
    z = noise.float().clone()
    ts = time_grid(steps, shift, z.device).tolist()
    tl = text_len.reshape(-1).to(torch.int32)
    nul = null_text.expand(B, -1, -1)
    nl = null_len.reshape(-1).expand(B).to(torch.int32)

    def vel(model, zz, t, tx, tlen):
        return model(zz, torch.full((zz.shape[0],), t, device=zz.device), tx, text_len=tlen).float()

    for k in range(steps):
        t0, t1 = ts[k], ts[k + 1]
        if t0 <= off:
            v = vel(den, z, t0, text, tl)
        elif method == "ag":
            bad, btext, blen = guide
            vc = vel(den, z, t0, text, tl)
            vb = vel(bad, z, t0, btext, blen.reshape(-1).to(torch.int32))
            v = vb + w * (vc - vb)
        else:
            vu, vc = vel(den, torch.cat([z, z]), t0, torch.cat([nul, text]), torch.cat([nl, tl])).chunk(2)
            if method == "cfgzero":
                if k == 0:
                    continue  # zero-init: no update on the first step
                s = ((vc * vu).flatten(1).sum(1) / (vu.flatten(1).square().sum(1) + 1e-8)).view(-1, 1, 1, 1)
                vu = s * vu
            elif method != "cfg":
                raise ValueError(f"unknown guidance method {method!r}")
            v = vu + w * (vc - vu)
        z = z + (t1 - t0) * v
    return z


def parse_method(spec):
    """'cfg:3', 'cfgzero:3', 'ag:<guide>:2', optionally '|shift=S|off=T' -> dict(method, w, guide, shift, off)."""
    head, *opts = spec.split("|")
    parts = head.split(":")
    kind = parts[0]
    out = dict(method=kind, w=float(parts[-1]) if len(parts) > 1 else 3.0, guide=parts[1] if kind == "ag" else None,
               shift=1.0, off=-1.0)
    for o in opts:
        k, v = o.split("=")
        out[k] = float(v)
    return out
