"""FLUX.2 latent <-> image conversion around a diffusers VAE (gated: needs diffusers and local VAE weights).

Latent layout (reference aurora/vae_encode.py:8-38, aurora/repa.py:17-50): the VAE's 32-channel latents at H/8
are packed 2 x 2 into 128 channels at H/16 with channel = c * 4 + dh * 2 + dw, and normalised with the VAE's batch
norm statistics (z - mean) / sqrt(var + eps). Encoding takes the posterior mode.
"""
import torch


def pack_2x2(z):
    """(B, C, 2h, 2w) -> (B, 4C, h, w), channel = c * 4 + dh * 2 + dw."""
    b, c, h2, w2 = z.shape
    return z.view(b, c, h2 // 2, 2, w2 // 2, 2).permute(0, 1, 3, 5, 2, 4).reshape(b, c * 4, h2 // 2, w2 // 2)


def unpack_2x2(z):
    """Inverse of pack_2x2: (B, 4C, h, w) -> (B, C, 2h, 2w)."""
    b, c4, h, w = z.shape
    return z.reshape(b, c4 // 4, 2, 2, h, w).permute(0, 1, 4, 2, 5, 3).reshape(b, c4 // 4, 2 * h, 2 * w)


class _VAE:
    def __init__(self, path, device):
        try:
            from diffusers import AutoencoderKLFlux2
        except ImportError as e:
            raise RuntimeError("decoding / encoding latents needs diffusers (not installed here)") from e
        vae = AutoencoderKLFlux2.from_pretrained(path, torch_dtype=torch.bfloat16)
        eps = float(getattr(vae.config, "batch_norm_eps", 1e-4))
        self.mean = vae.bn.running_mean.float().view(1, -1, 1, 1).to(device)
        self.std = torch.sqrt(vae.bn.running_var.float() + eps).view(1, -1, 1, 1).to(device)
        self.vae = vae.to(device).eval().requires_grad_(False)


class LatentDecoder(_VAE):
    @torch.no_grad()
    def decode(self, z, chunk=8):
        """Normalised packed latents -> uint8 images (B, H, W, 3) as numpy."""
        out = []
        for i in range(0, len(z), chunk):
            x = unpack_2x2(z[i:i + chunk].float() * self.std + self.mean)
            img = self.vae.decode(x.to(torch.bfloat16)).sample.float().clamp(-1, 1)
            out.append(((img + 1) * 127.5).round().to(torch.uint8).permute(0, 2, 3, 1).cpu())
        return torch.cat(out).numpy()


class LatentEncoder(_VAE):
    @torch.no_grad()
    def __call__(self, img, chunk=8):
        """uint8 (B, 3, H, W) -> normalised packed latents (B, 128, H/16, W/16) fp32."""
        out = []
        for i in range(0, len(img), chunk):
            x = (img[i:i + chunk].float() / 127.5 - 1).to(torch.bfloat16)
            z = pack_2x2(self.vae.encode(x).latent_dist.mode().float())
            out.append((z - self.mean) / self.std)
        return torch.cat(out)


class PatchEncoder:
    """Stand-in image encoder with the FLUX.2 latent shape, for runs without the VAE weights (service-rank and
    loader plumbing, tests): every 16 x 16 RGB patch goes through a fixed, seeded linear map to ``channels``
    values, so (B, 3, H, W) uint8 -> (B, channels, H / 16, W / 16) float32, roughly unit variance."""

    def __init__(self, channels=128, patch=16, seed=0, device=None):
        g = torch.Generator().manual_seed(seed + 7)
        n = 3 * patch * patch
        self.patch = patch
        self.proj = (torch.randn(channels, n, generator=g) / n ** 0.5).to(device)

    @torch.no_grad()
    def __call__(self, img):
        x = img.float() / 127.5 - 1
        B, _, H, W = x.shape
        cols = torch.nn.functional.unfold(x, self.patch, stride=self.patch)  # (B, 3 p p, h w)
        z = self.proj.to(x.device) @ cols
        return (z * 3.0).view(B, -1, H // self.patch, W // self.patch)
