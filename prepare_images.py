"""Encoded images packed for random access by row (reference prepare_images.py:31-150): <name>.img.bin holds the
encoded files back to back, unchanged, and <name>.img.off.npy (int64 [N + 1]) their byte offsets, written last so a
shard exists only once complete. data/shards.py memory-maps both (ShardStore img_root / img_res) and decodes rows
with PIL when training encodes latents in the loader.

  python prepare_images.py dir --src photos/ --out data/x --name shard-00000 [--per-shard 10000]
  python prepare_images.py parquet --parquet-dir data/monet --column image      # next to every parquet
  python prepare_images.py monet --parquet-dir data/monet_z_image               # prepare_monet.py's thumbnails
  python prepare_images.py flux-reason --src raw/FLUX-Reason-6M --out data/flux_reason_1024 --data data/aurora \
      --fraction 0.5 --workers 16 --tmp /scratch

``dir`` packs the JPEG / PNG / WEBP files of a directory (sorted by name) into shards of --per-shard images;
``parquet`` packs an image column (bytes, or {"bytes": ...} structs) of every parquet file; ``monet`` is ``parquet``
with the thumbnail column of prepare_monet.py's output. ``flux-reason`` packs the dataset's <subset>/<shard>.parquet
files into <out>/<shard>.img.*, shard names and row order those of the latent shards, so their captions and tokens
apply as they are: the held-out shards always, --fraction of the training shards (the same evenly spaced choice as
training), each shard in its own short-lived worker process (--workers at once; memory the parquet reader keeps goes
back to the OS when the worker exits), optionally staged through --tmp (a copy there, packed, then deleted, e.g. off
network storage), with --data the image count of every shard checked against its caption offsets (.off.npy), and
--max-shards for a test. The reference downloads each parquet from the Hub; offline, --src is a local copy of the
dataset folder.
"""
import argparse
import glob
import os
import shutil
import tempfile
import time
from multiprocessing import get_context

import numpy as np


class PackWriter:
    """Streaming writer: images are appended as they come, so a shard is never held in memory whole."""

    def __init__(self, out_base):
        self.base, self.sizes = out_base, []
        self.f = open(out_base + ".img.bin.tmp", "wb")

    def add(self, blobs):
        for b in blobs:
            self.f.write(b)
            self.sizes.append(len(b))

    def close(self):
        self.f.close()
        os.replace(self.base + ".img.bin.tmp", self.base + ".img.bin")
        off = np.zeros(len(self.sizes) + 1, dtype=np.int64)
        np.cumsum(self.sizes, out=off[1:])
        with open(self.base + ".img.off.npy.tmp", "wb") as f:
            np.save(f, off)
        os.replace(self.base + ".img.off.npy.tmp", self.base + ".img.off.npy")  # last: shard complete
        return len(self.sizes), int(off[-1])


def read_packed(base, i):
    """Bytes of image i of a packed shard."""
    off = np.load(base + ".img.off.npy", mmap_mode="r")
    with open(base + ".img.bin", "rb") as f:
        f.seek(int(off[i]))
        return f.read(int(off[i + 1] - off[i]))


def cmd_dir(a):
    exts = (".jpg", ".jpeg", ".png", ".webp")
    files = sorted(f for f in glob.glob(os.path.join(a.src, "**", "*"), recursive=True) if f.lower().endswith(exts))
    os.makedirs(a.out, exist_ok=True)
    for s in range(0, len(files), a.per_shard):
        name = f"{a.name}-{s // a.per_shard:05d}" if len(files) > a.per_shard else a.name
        w = PackWriter(os.path.join(a.out, name))
        for path in files[s:s + a.per_shard]:
            with open(path, "rb") as f:
                w.add([f.read()])
        n, nbytes = w.close()
        print(f"{name}: {n} images, {nbytes / 1e6:.1f} MB", flush=True)


def cmd_parquet(a):
    import pyarrow.parquet as pq
    files = sorted(f for f in glob.glob(os.path.join(a.parquet_dir, "**", "*.parquet"), recursive=True)
                   if os.path.basename(f).count(".") == 1)
    for path in files:
        base = path[: -len(".parquet")]
        if os.path.exists(base + ".img.off.npy") and not a.force:
            continue
        w = PackWriter(base)
        pf = pq.ParquetFile(path)
        for g in range(pf.num_row_groups):
            col = pf.read_row_group(g, columns=[a.column])[a.column].to_pylist()
            w.add(image_bytes(col))
        n, nbytes = w.close()
        print(f"{os.path.relpath(path, a.parquet_dir)}: {n} images, {nbytes / 1e6:.1f} MB", flush=True)


def image_bytes(col):
    return [x["bytes"] if isinstance(x, dict) else x for x in col]


def flux_reason_one(job):
    """Pack one FLUX-Reason parquet; returns (name, images, bytes, skipped). Runs in its own worker process."""
    import pyarrow.parquet as pq
    path, out, data, tmp_root, column = job
    name = os.path.basename(path)[: -len(".parquet")]
    base = os.path.join(out, name)
    if os.path.exists(base + ".img.off.npy"):
        return name, 0, 0, True
    tmp = tempfile.mkdtemp(dir=tmp_root) if tmp_root else None
    try:
        local = shutil.copy(path, tmp) if tmp else path
        pf = pq.ParquetFile(local, memory_map=True)
        w = PackWriter(base)
        for g in range(pf.metadata.num_row_groups):
            w.add(image_bytes(pf.read_row_group(g, columns=[column])[column].to_pylist()))
        ref = os.path.join(data, f"{name}.off.npy") if data else ""
        if ref and os.path.exists(ref):
            n_cap = len(np.load(ref)) - 1
            if n_cap != len(w.sizes):
                w.f.close()
                os.remove(base + ".img.bin.tmp")
                raise ValueError(f"{name}: {len(w.sizes)} images, {n_cap} caption rows in {data}")
        n, size = w.close()
    finally:
        if tmp:
            shutil.rmtree(tmp, ignore_errors=True)
    return name, n, size, False


def flux_reason_jobs(a):
    from trenowanie_generatora_obrazkow_b200.data.shards import select_fraction, split_shards
    files = sorted(glob.glob(os.path.join(a.src, "*", "*.parquet")) + glob.glob(os.path.join(a.src, "*.parquet")))
    by_name = {os.path.basename(f)[: -len(".parquet")]: f for f in files}
    train, val = split_shards(sorted(by_name))  # the held-out shards of latent training
    names = select_fraction(train, a.fraction) + val
    if a.max_shards:
        names = names[: a.max_shards]
    return [(by_name[n], a.out, a.data, a.tmp, a.column) for n in names], len(by_name), len(val)


def cmd_flux_reason(a):
    jobs, total, n_val = flux_reason_jobs(a)
    os.makedirs(a.out, exist_ok=True)
    if a.tmp:
        os.makedirs(a.tmp, exist_ok=True)
    print(f"{total} parquets, {len(jobs)} selected ({n_val} held-out) -> {a.out}", flush=True)
    t0, done, imgs, gb = time.time(), 0, 0, 0.0
    with get_context("spawn").Pool(max(1, a.workers), maxtasksperchild=1) as pool:
        for name, n, size, skipped in pool.imap_unordered(flux_reason_one, jobs):
            done += 1
            imgs += n
            gb += size / 1e9
            el = time.time() - t0
            print(f"[{done}/{len(jobs)}] {name}: {'skip' if skipped else f'{n} images, {size / 1e9:.2f} GB'} | "
                  f"{imgs:,} images, {gb:.1f} GB, eta {(len(jobs) - done) * el / done / 3600:.1f} h", flush=True)
    return imgs


def cmd_monet(a):
    a.column, a.force = "thumbnail", False
    cmd_parquet(a)


def main(argv=None):
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("dir")
    s.add_argument("--src", required=True)
    s.add_argument("--out", required=True)
    s.add_argument("--name", default="images")
    s.add_argument("--per-shard", type=int, default=10000)
    s = sub.add_parser("parquet")
    s.add_argument("--parquet-dir", required=True)
    s.add_argument("--column", default="image")
    s.add_argument("--force", action="store_true")
    s = sub.add_parser("monet")
    s.add_argument("--parquet-dir", required=True)
    s = sub.add_parser("flux-reason")
    s.add_argument("--src", required=True, help="local copy of the dataset folder (<subset>/<shard>.parquet)")
    s.add_argument("--out", required=True)
    s.add_argument("--data", default="", help="latent shards to check the image counts against (their .off.npy)")
    s.add_argument("--fraction", type=float, default=1.0, help="of the training shards (held-out ones always)")
    s.add_argument("--workers", type=int, default=16, help="parquets packed at once (one process each)")
    s.add_argument("--tmp", default="", help="stage each parquet through a copy here (deleted after packing)")
    s.add_argument("--max-shards", type=int, default=0, help="only the first N selected shards (a test)")
    s.add_argument("--column", default="image")
    a = p.parse_args(argv)
    return {"dir": cmd_dir, "parquet": cmd_parquet, "monet": cmd_monet, "flux-reason": cmd_flux_reason}[a.cmd](a)


if __name__ == "__main__":
    main()
