"""REPA representation alignment (Yu et al. 2024, arXiv:2410.06940; iREPA arXiv:2512.10794), reference
aurora/repa.py:17-94 and train.py:695-702, :890-923.

The denoiser's hidden state after block ``repa_layer`` (one token per latent pixel) is projected and aligned with
frozen vision-encoder patch features of the same image: loss = -cos(proj(h), target), added with ``repa_weight`` for
the first ``repa_frac`` of every micro-batch, every ``repa_every``-th step, until ``repa_until`` of training.

* ``make_projector``: REPA's 3-layer SiLU MLP (dim -> 2048 -> 2048 -> target), or iREPA's 3x3 conv over the token
  grid (``conv=True``).
* ``REPATarget``: FLUX.2 decoder -> image -> timm encoder patch tokens (DINOv2-B/14-reg by default); needs diffusers,
  timm and local weights, none of which this offline image has, so it raises a clear error here.
* ``LatentTarget``: an offline stand-in with the same interface: a fixed (seeded) random 3x3 conv of the latents
  followed by GELU, giving a (B, tokens, dim) target that depends on spatial structure. It exercises the whole REPA
  path (projector, hidden-state tap, loss, schedule, checkpointing) without the pretrained encoder; alignment
  numbers from it mean nothing for image quality.
``spatial_norm`` (iREPA): targets normalised per image and channel over the tokens.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F


class ConvProjector(nn.Module):
    def __init__(self, dim, target_dim):
        super().__init__()
        self.conv = nn.Conv2d(dim, target_dim, 3, padding=1)

    def forward(self, h):  # (N, side * side, dim) -> (N, side * side, target_dim)
        n, t, d = h.shape
        side = int(round(t ** 0.5))
        x = h.transpose(1, 2).reshape(n, d, side, side)
        return self.conv(x.to(self.conv.weight.dtype)).flatten(2).transpose(1, 2)


def make_projector(dim, target_dim, hidden=2048, conv=False):
    if conv:
        return ConvProjector(dim, target_dim)
    return nn.Sequential(nn.Linear(dim, hidden), nn.SiLU(), nn.Linear(hidden, hidden), nn.SiLU(),
                         nn.Linear(hidden, target_dim))


def _spatial_norm(f):
    return (f - f.mean(1, keepdim=True)) / (f.std(1, keepdim=True) + 1e-6)


class LatentTarget:
    def __init__(self, channels, dim=768, spatial_norm=False, seed=0, device=None):
        g = torch.Generator().manual_seed(seed + 577)
        self.w = (torch.randn(dim, channels, 3, 3, generator=g) / (channels * 9) ** 0.5).to(device)
        self.dim, self.spatial_norm = dim, spatial_norm

    @torch.no_grad()
    def __call__(self, x0):
        f = F.gelu(F.conv2d(x0.float(), self.w.to(x0.device), padding=1)).flatten(2).transpose(1, 2)
        return _spatial_norm(f) if self.spatial_norm else f


class REPATarget:
    def __init__(self, vae_dir, encoder="vit_base_patch14_reg4_dinov2.lvd142m", device="cuda", spatial_norm=False,
                 grid=16):
        try:
            import timm
            from diffusers import AutoencoderKLFlux2  # noqa: F401
        except ImportError as e:
            raise RuntimeError("REPATarget needs timm, diffusers and local FLUX.2 VAE / encoder weights (not in this "
                               "image); --repa-target latent runs the offline stand-in") from e
        from ..sampling.vae import LatentDecoder
        self.decoder = LatentDecoder(vae_dir, device)
        self.enc = timm.create_model(encoder, pretrained=True, dynamic_img_size=True).to(device).eval()
        self.enc.requires_grad_(False)
        cfg = self.enc.pretrained_cfg
        self.img_mean = torch.tensor(cfg["mean"], device=device).view(1, 3, 1, 1)
        self.img_std = torch.tensor(cfg["std"], device=device).view(1, 3, 1, 1)
        self.prefix = getattr(self.enc, "num_prefix_tokens", 0)
        self.dim = self.enc.num_features
        patch = self.enc.patch_embed.patch_size
        self.size = (patch[0] * grid, patch[1] * grid)
        self.spatial_norm, self.device = spatial_norm, device

    @torch.no_grad()
    def __call__(self, x0):
        img = torch.from_numpy(self.decoder.decode(x0)).to(self.device).permute(0, 3, 1, 2).float() / 127.5 - 1
        img = F.interpolate(img, size=self.size, mode="bicubic", antialias=True, align_corners=False)
        img = ((img + 1) / 2 - self.img_mean) / self.img_std
        with torch.autocast("cuda", dtype=torch.bfloat16):
            f = self.enc.forward_features(img)[:, self.prefix:].float()
        return _spatial_norm(f) if self.spatial_norm else f


def repa_active(step, steps, until=0.4, every=1):
    """The reference's schedule: on every ``every``-th step (offset every // 2) before ``until`` of training."""
    return step < int(until * steps) and step % every == every // 2
