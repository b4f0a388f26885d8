"""Translated captions as a dataset folder (reference export_captions_pl.py, export_monet_captions_pl.py): the
translations written by translate_captions.py are collected into data/train-<n>.parquet files (one row per image:
shard, row index, the source captions and their translations, or `__key__` and the two caption columns for the
parquet mode) plus a README.md dataset card. Publishing it to the Hugging Face Hub needs network access, which this
machine does not have: upload the folder from elsewhere.

  python export_captions.py --data data/aurora --out exports/aurora_captions_pl --shards-per-file 50
  python export_captions.py --parquet-dir data/monet_z_image --source z-image --out exports/monet_pl

--shards-per-file N cuts the files at shard boundaries (N training shards per parquet, shard mode) instead of every
--per-file rows. --repo names the Hub repository the card's loading snippet uses; --source names the MONET synthetic
source the parquets came from (card text only).
"""
import argparse
import glob
import json
import os

CARD = """---
license: {license}
language: [{src}, {tgt}]
task_categories: [text-to-image]
---
# {name}

Captions of {origin} translated from `{src}` to `{tgt}` by translate_captions.py ({rows} rows in {files} files).
Quoted text (what is written in the images) was kept verbatim.
{usage}"""

USAGE = """
```python
from datasets import load_dataset
ds = load_dataset("{repo}", split="train")
```
"""


def _chunks(rows, per_file, shards_per_file=0):
    """Row groups of the output files: every ``per_file`` rows, or (shards_per_file > 0) ``shards_per_file`` whole
    shards per file."""
    if not shards_per_file:
        return [rows[i:i + per_file] for i in range(0, len(rows), per_file)]
    order = list(dict.fromkeys(r["shard"] for r in rows))
    group = {s: i // shards_per_file for i, s in enumerate(order)}
    out = [[] for _ in range(-(-len(order) // shards_per_file))]
    for r in rows:
        out[group[r["shard"]]].append(r)
    return out


def _write(rows, out, per_file, shards_per_file=0):
    import pyarrow as pa
    import pyarrow.parquet as pq
    os.makedirs(os.path.join(out, "data"), exist_ok=True)
    n_files = 0
    for part in _chunks(rows, per_file, shards_per_file):
        cols = {k: [r[k] for r in part] for k in part[0]}
        path = os.path.join(out, "data", f"train-{n_files:05d}.parquet")
        pq.write_table(pa.table(cols), path + ".tmp", compression="zstd")
        os.replace(path + ".tmp", path)
        n_files += 1
    return n_files


def collect_caps(data, suffix):
    rows = []
    for path in sorted(glob.glob(os.path.join(data, f"*.caps_{suffix}.json"))):
        shard = os.path.basename(path)[: -len(f".caps_{suffix}.json")]
        src = json.load(open(os.path.join(data, shard + ".caps.json")))
        dst = json.load(open(path))
        for i, (a, b) in enumerate(zip(src, dst)):
            rows.append(dict(shard=shard, index=i, captions=a, **{f"captions_{suffix}": b}))
    return rows


def collect_parquets(root, column, suffix):
    import pyarrow.parquet as pq
    rows = []
    for path in sorted(glob.glob(os.path.join(root, "**", f"*.{suffix}.parquet"), recursive=True)):
        src = pq.read_table(path[: -len(f".{suffix}.parquet")] + ".parquet", columns=["__key__", column]).to_pylist()
        dst = pq.read_table(path).to_pylist()
        for s, d in zip(src, dst):
            assert s["__key__"] == d["__key__"], f"{path}: row order differs from its source"
            rows.append({"__key__": s["__key__"], column: s[column], f"{column}_{suffix}": d[f"{column}_{suffix}"]})
    return rows


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--data", default="")
    p.add_argument("--parquet-dir", default="")
    p.add_argument("--column", default="caption_short")
    p.add_argument("--suffix", default="pl")
    p.add_argument("--out", required=True)
    p.add_argument("--per-file", type=int, default=100_000)
    p.add_argument("--name", default="")
    p.add_argument("--license", default="apache-2.0")
    p.add_argument("--shards-per-file", type=int, default=0, help="shard mode: this many shards per parquet file")
    p.add_argument("--repo", default="", help="Hub repository named in the card's loading snippet (card only)")
    p.add_argument("--source", default="", help="the MONET synthetic source of the parquets (card only)")
    a = p.parse_args(argv)
    assert bool(a.data) != bool(a.parquet_dir), "give --data or --parquet-dir"
    assert not (a.shards_per_file and a.parquet_dir), "--shards-per-file applies to --data (shard) mode"
    rows = collect_caps(a.data, a.suffix) if a.data else collect_parquets(a.parquet_dir, a.column, a.suffix)
    assert rows, "no translated captions found"
    files = _write(rows, a.out, a.per_file, a.shards_per_file)
    origin = os.path.basename(os.path.normpath(a.data or a.parquet_dir))
    if a.source:
        origin = f"the MONET `{a.source}` synthetic images ({origin})"
    name = a.name or (a.repo.split("/")[-1] if a.repo else f"{origin} captions ({a.suffix})")
    with open(os.path.join(a.out, "README.md"), "w") as f:
        f.write(CARD.format(license=a.license, src="en", tgt=a.suffix, name=name, origin=origin, rows=len(rows),
                            files=files, usage=USAGE.format(repo=a.repo) if a.repo else ""))
    print(f"{len(rows)} rows in {files} files -> {a.out}")
    return len(rows)


if __name__ == "__main__":
    main()
