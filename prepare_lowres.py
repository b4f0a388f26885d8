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

VAE options (reference prepare_lowres.py:96-125):
  --decoder DIR       decode with another AutoencoderKLFlux2's decoder (e.g. the small one, cheaper; its differences
                      mostly vanish after the downscale); the encoder and the latent statistics stay --vae's.
  --channels-last     NHWC activations for the VAE convolutions.
  --cudnn-benchmark   let cuDNN time and pick its convolution algorithms.
  --cpu-threads N     torch CPU threads per rank (torchrun sets 1; 0 leaves the setting alone).
  --compile [MODE]    capture the decoder and the encoder into CUDA graphs, one per batch shape (the last batch of a
                      shard is padded, so there is one shape); this project replays graphs where the reference
                      uses torch.compile, and MODE is accepted for the same command line but has no effect.
"""
import argparse
import glob
import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch
import torch.nn.functional as F


class GraphedCall:
    """fn(x) replayed from a CUDA graph captured per input shape / dtype (warm-up on a side stream, then capture);
    the input is copied into the graph's static buffer and the returned tensor is the graph's static output, so
    it is consumed before the next call. Off CUDA it calls fn directly."""

    def __init__(self, fn):
        self.fn, self.graphs = fn, {}

    def __call__(self, x):
        if x.device.type != "cuda":
            return self.fn(x)
        key = (tuple(x.shape), x.dtype)
        if key not in self.graphs:
            static = x.clone()
            side = torch.cuda.Stream(x.device)
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.fn(static)
            torch.cuda.current_stream(x.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self.fn(static)
            self.graphs[key] = (g, static, out)
        g, static, out = self.graphs[key]
        static.copy_(x)
        g.replay()
        return out


class VaeResizer:
    """decode (``dec``) -> bicubic antialiased downscale -> encode (``enc``), both sampling/vae.py objects. A
    separate ``decoder_dir`` decodes with another VAE's decoder but the encoder's latent statistics."""

    def __init__(self, vae_dir, device, decoder_dir="", channels_last=False, graphs=False, dec=None, enc=None):
        from trenowanie_generatora_obrazkow_b200.sampling.vae import LatentDecoder, LatentEncoder
        self.enc = enc if enc is not None else LatentEncoder(vae_dir, device)
        self.dec = dec if dec is not None else LatentDecoder(decoder_dir or vae_dir, device)
        self.dec.mean, self.dec.std = self.enc.mean, self.enc.std  # one latent normalisation: the encoder's
        self.device = device
        if channels_last:
            for m in (self.dec, self.enc):
                m.vae.to(memory_format=torch.channels_last)
        if graphs:
            self.dec.vae.decode = GraphedCall(self.dec.vae.decode)
            self.enc.vae.encode = GraphedCall(self.enc.vae.encode)

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
    p.add_argument("--decoder", default="", help="another AutoencoderKLFlux2 whose decoder makes the 256 px images")
    p.add_argument("--channels-last", action="store_true", help="NHWC activations for the VAE")
    p.add_argument("--cudnn-benchmark", action="store_true", help="let cuDNN pick its fastest conv algorithms")
    p.add_argument("--cpu-threads", type=int, default=0, help="torch CPU threads per rank (0: leave torch's setting; "
                   "torchrun sets 1, and 3 x 8 ranks suits a 24-core host)")
    p.add_argument("--compile", nargs="?", const="default", default="",
                   help="replay the VAE decoder / encoder from CUDA graphs (MODE has no effect)")
    a = p.parse_args(argv)
    assert all(s % 16 == 0 and s < 256 for s in a.sizes), "sizes must be multiples of 16, below 256"
    assert bool(a.vae) != a.latent_pool, "pick one method: --vae DIR or --latent-pool"
    assert not (a.latent_pool and (a.decoder or a.channels_last or a.compile)), "VAE options need --vae"
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    if a.cpu_threads > 0:
        torch.set_num_threads(a.cpu_threads)
    torch.backends.cudnn.benchmark = a.cudnn_benchmark
    device = torch.device(a.device if a.device != "cuda" else f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    conv = (VaeResizer(a.vae, device, a.decoder, a.channels_last, bool(a.compile)) if a.vae
            else LatentPool(device))
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
