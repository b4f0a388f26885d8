"""Lower-resolution latents next to the 256 px ones (reference prepare_lowres.py:22-180): every <shard>.lat.npy
(N, 128, 16, 16) normalised FLUX.2 latents becomes <shard>.lat<size>.npy (N, 128, size/16, size/16) float16 for each
--sizes, the layout train.py --crop-res / --multi-res and ShardStore read.

  torchrun --nproc_per_node 8 prepare_lowres.py --data data/aurora --vae FLUX.2-dev-vae --sizes 128 64 32
  python prepare_lowres.py --data data/aurora --latent-pool --sizes 128 64      # no VAE at hand

Methods:
  --vae DIR       decode the 256 px latents with the FLUX.2 decoder, downscale the images (bicubic, antialiased),
                  encode them again (posterior mode), pack 2 x 2 and normalise: what the reference does (needs
                  diffusers and the VAE weights, neither of which this offline image has).
  --latent-pool   area-average the latent grid instead (a cheap approximation, not what the VAE would produce).
Shards are split over the ranks (RANK / WORLD_SIZE, no collectives); finished outputs are skipped, so an interrupted
run resumes; files are written to a temporary name and renamed; the next shard is read and the last one written by
an I/O thread while the current one converts. --bench N times N batches of the first shard and writes nothing.
"""
import argparse
import glob
import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch
import torch.nn.functional as F


class VaeResizer:
    def __init__(self, vae_dir, device):
        from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentDecoder, LatentEncoder
        self.dec, self.enc, self.device = LatentDecoder(vae_dir, device), LatentEncoder(vae_dir, device), device

    @torch.no_grad()
    def __call__(self, lat, sizes):
        z = torch.from_numpy(np.ascontiguousarray(lat)).to(self.device).float()
        img = torch.from_numpy(self.dec.decode(z)).to(self.device).permute(0, 3, 1, 2).float()  # uint8 -> float
        out = {}
        for s in sizes:
            small = F.interpolate(img, size=(s, s), mode="bicubic", antialias=True, align_corners=False)
            out[s] = self.enc(small.clamp(0, 255).round().to(torch.uint8)).half().cpu().numpy()
        return out


class LatentPool:
    def __init__(self, device):
        self.device = device

    @torch.no_grad()
    def __call__(self, lat, sizes):
        z = torch.from_numpy(np.ascontiguousarray(lat)).to(self.device).float()
        return {s: F.adaptive_avg_pool2d(z, s // 16).half().cpu().numpy() for s in sizes}


def outputs(path, sizes, out_dir):
    name = os.path.basename(path)[: -len(".lat.npy")]
    return {s: (os.path.join(out_dir, f"{s}px", f"{name}.lat{s}.npy") if out_dir
                else f"{path[: -len('.lat.npy')]}.lat{s}.npy") for s in sizes}


def convert_shard(conv, lat, sizes, batch):
    res = {s: np.empty((len(lat), 128, s // 16, s // 16), dtype=np.float16) for s in sizes}
    for i in range(0, len(lat), batch):
        chunk = lat[i:i + batch]
        n = len(chunk)
        if n < batch:  # one batch shape for every call
            chunk = np.concatenate([chunk, np.repeat(chunk[-1:], batch - n, axis=0)])
        for s, z in conv(chunk, sizes).items():
            res[s][i:i + n] = z[:n]
    return res


def save(outs, res):
    for s, o in outs.items():
        np.save(o + ".tmp.npy", res[s])
        os.replace(o + ".tmp.npy", o)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--data", required=True)
    p.add_argument("--vae", default="")
    p.add_argument("--latent-pool", action="store_true")
    p.add_argument("--out-dir", default="", help="write <out-dir>/<size>px/<shard>.lat<size>.npy instead")
    p.add_argument("--sizes", type=int, nargs="+", default=[128, 64, 32])
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--bench", type=int, default=0)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = p.parse_args(argv)
    assert all(s % 16 == 0 and s < 256 for s in a.sizes), "sizes must be multiples of 16, below 256"
    assert bool(a.vae) != a.latent_pool, "pick one method: --vae DIR or --latent-pool"
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    device = torch.device(a.device if a.device != "cuda" else f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    conv = VaeResizer(a.vae, device) if a.vae else LatentPool(device)
    shards = sorted(glob.glob(os.path.join(a.data, "*.lat.npy")))[rank::world]
    if a.bench:
        lat = np.load(shards[0], mmap_mode="r")
        n = a.batch * (a.bench + 2)
        lat = np.concatenate([lat] * (-(-n // len(lat))))[:n]
        convert_shard(conv, lat[: 2 * a.batch], a.sizes, a.batch)  # warm-up
        t0 = time.perf_counter()
        convert_shard(conv, lat[2 * a.batch:], a.sizes, a.batch)
        dt = time.perf_counter() - t0
        print(f"rank {rank}: {a.batch * a.bench / dt:.1f} img/s (batch {a.batch}, sizes {a.sizes})", flush=True)
        return
    todo = [s for s in shards if not all(os.path.exists(o) for o in outputs(s, a.sizes, a.out_dir).values())]
    print(f"rank {rank}: {len(todo)} of {len(shards)} shards to convert", flush=True)
    io = ThreadPoolExecutor(2)
    nxt = io.submit(np.load, todo[0]) if todo else None
    writes, done, t0 = [], 0, time.time()
    for k, path in enumerate(todo):
        outs = outputs(path, a.sizes, a.out_dir)
        for o in outs.values():
            os.makedirs(os.path.dirname(o) or ".", exist_ok=True)
        lat = nxt.result()
        nxt = io.submit(np.load, todo[k + 1]) if k + 1 < len(todo) else None
        writes.append(io.submit(save, outs, convert_shard(conv, lat, a.sizes, a.batch)))
        done += len(lat)
        el = time.time() - t0
        print(f"rank {rank}: [{k + 1}/{len(todo)}] {os.path.basename(path)} ({len(lat)} images), "
              f"{done / max(el, 1e-9):.0f} img/s", flush=True)
    for w in writes:
        w.result()
    io.shutdown()


if __name__ == "__main__":
    main()
