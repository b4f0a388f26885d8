"""Encoded images packed for random access by row (reference prepare_images.py:31-150): <name>.img.bin holds the
encoded files back to back, unchanged, and <name>.img.off.npy (int64 [N + 1]) their byte offsets, written last so a
shard exists only once complete. data/shards.py memory-maps both (ShardStore img_root / img_res) and decodes rows
with PIL when training encodes latents in the loader.

  python prepare_images.py dir --src photos/ --out data/x --name shard-00000 [--per-shard 10000]
  python prepare_images.py parquet --parquet-dir data/monet --column image      # next to every parquet

``dir`` packs the JPEG / PNG / WEBP files of a directory (sorted by name) into shards of --per-shard images;
``parquet`` packs an image column (bytes, or {"bytes": ...} structs) of every parquet file. Downloading source
datasets from the Hub is not available offline.
"""
import argparse
import glob
import os

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
            w.add([x["bytes"] if isinstance(x, dict) else x for x in col])
        n, nbytes = w.close()
        print(f"{os.path.relpath(path, a.parquet_dir)}: {n} images, {nbytes / 1e6:.1f} MB", flush=True)


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
    a = p.parse_args(argv)
    {"dir": cmd_dir, "parquet": cmd_parquet}[a.cmd](a)


if __name__ == "__main__":
    main()
