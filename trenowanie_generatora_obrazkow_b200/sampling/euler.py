"""Euler sampler with classifier-free guidance.

Reference: aurora/fid.py:13-39 and the diffusers pipeline aurora/hf_pipeline.py:748-760, 816-827:
  u = linspace(1, 0, steps + 1); t_k = s u / (1 + (s - 1) u)     (time shift s)
  each step runs the denoiser once on [null; cond] and updates z += (t_{k+1} - t_k) (v_u + w (v_c - v_u)) in fp32;
  noise for prompts i .. i + batch is drawn from a generator seeded seed * 1_000_003 + noise_offset + i.
On CUDA the guidance combine, the Euler update and the token-major -> latent-layout transpose are one kernel
(csrc/elementwise.cu), and the text encoder runs once per prompt batch.
"""
import torch

from ..models.text import LMTextEncoder
from ..ops import reference as R
from ..ops._ext import ext


def time_grid(steps, shift=1.0, device=None):
    u = torch.linspace(1.0, 0.0, steps + 1, device=device)
    return shift * u / (1 + (shift - 1) * u)


def prompt_noise(n, channels, side, seed, offset=0, device=None):
    """Noise of prompts offset .. offset + n (one generator per call, as the reference's per-batch seeding)."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + offset)
    return torch.randn(n, channels, side, side, device=device, generator=g)


@torch.no_grad()
def sample_latents(den, text, text_len, null_text, null_len, steps=50, cfg=3.0, seed=0, shift=1.0, latent_size=None,
                   noise=None, cond=None):
    """text (B, L, D) / text_len (B,) of the prompts; null_text (1 or B, L, D) / null_len of the null prompt.
    Returns normalised latents (B, C, h, w) fp32."""
    c = den.config
    B = text.shape[0]
    side = latent_size or c.latent_size
    device = text.device
    if noise is None:
        noise = prompt_noise(B, c.latent_channels, side, seed, 0, device)
    z = noise.float().contiguous()
    ts = time_grid(steps, shift, device).tolist()
    tx = torch.cat([null_text.expand(B, -1, -1), text])
    tl = torch.cat([null_len.reshape(-1).expand(B), text_len.reshape(-1)]).to(device=device, dtype=torch.int32)
    cond2 = None if cond is None else torch.cat([cond, cond])
    for k in range(steps):
        t0, t1 = ts[k], ts[k + 1]
        tt = torch.full((2 * B,), t0, device=device)
        zz = torch.cat([z, z])
        if z.is_cuda:
            v = den(zz, tt, tx, text_len=tl, cond=cond2, tokens_out=True)
            ext().euler_cfg(v.contiguous(), z, t1 - t0, cfg)
        else:
            v = den(zz, tt, tx, text_len=tl, cond=cond2).float()
            v_u, v_c = v.chunk(2)
            z = z + (t1 - t0) * (v_u + cfg * (v_c - v_u))
    return z


@torch.no_grad()
def encode_prompts(te, ids=None, lm_states=None, valid=None):
    """Text encoder outputs for prompts and for the null prompt: (text, lens, null_text, null_len)."""
    if isinstance(te, LMTextEncoder):
        B, L, _ = lm_states.shape
        if valid is None:
            valid = torch.ones(B, L, dtype=torch.bool, device=lm_states.device)
        text, v = te(lm_states=lm_states, valid=valid, is_null=torch.zeros(B, dtype=torch.bool, device=valid.device))
        nvalid = torch.zeros(1, L, dtype=torch.bool, device=valid.device)
        nvalid[0, 0] = True
        null, nv = te(lm_states=torch.zeros_like(lm_states[:1]), valid=nvalid,
                      is_null=torch.ones(1, dtype=torch.bool, device=valid.device))
    else:
        text, v = te(ids)
        null_row = torch.as_tensor(te.null_ids(), device=ids.device)[None, : ids.shape[1]]
        null, nv = te(null_row)
    return text, R.valid_to_len(v), null, R.valid_to_len(nv)


@torch.no_grad()
def sample(te, den, steps=50, cfg=3.0, seed=0, shift=1.0, latent_size=None, batch=64, ids=None, lm_states=None,
           valid=None, noise_offset=0):
    """Latents for a list of prompts (token ids for a TextEncoder, LM states for an LMTextEncoder), `batch` at a
    time, noise fixed by (seed, prompt index)."""
    n = (ids if ids is not None else lm_states).shape[0]
    side = latent_size or den.config.latent_size
    out = []
    for i in range(0, n, batch):
        sl = slice(i, i + batch)
        text, lens, null, nlen = encode_prompts(te, None if ids is None else ids[sl],
                                                None if lm_states is None else lm_states[sl],
                                                None if valid is None else valid[sl])
        dev = text.device
        noise = prompt_noise(text.shape[0], den.config.latent_channels, side, seed, noise_offset + i, dev)
        out.append(sample_latents(den, text, lens, null, nlen, steps, cfg, seed, shift, side, noise))
    return torch.cat(out)
