"""Translated captions as a dataset folder (reference export_captions_pl.py, export_monet_captions_pl.py): the
translations written by translate_captions.py are collected into data/train-<n>.parquet files (one row per image:
shard, row index, the source captions and their translations, or `__key__` and the two caption columns for the
parquet mode) plus a README.md dataset card. Publishing it to the Hugging Face Hub needs network access, which this
machine does not have: upload the folder from elsewhere.

  python export_captions.py --data data/aurora --out exports/aurora_captions_pl
  python export_captions.py --parquet-dir data/monet_z_image --column caption_short --out exports/monet_pl
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
"""


def _write(rows, out, per_file):
    import pyarrow as pa
    import pyarrow.parquet as pq
    os.makedirs(os.path.join(out, "data"), exist_ok=True)
    n_files = 0
    for i in range(0, len(rows), per_file):
        part = rows[i:i + per_file]
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
    a = p.parse_args(argv)
    assert bool(a.data) != bool(a.parquet_dir), "give --data or --parquet-dir"
    rows = collect_caps(a.data, a.suffix) if a.data else collect_parquets(a.parquet_dir, a.column, a.suffix)
    assert rows, "no translated captions found"
    files = _write(rows, a.out, a.per_file)
    origin = os.path.basename(os.path.normpath(a.data or a.parquet_dir))
    with open(os.path.join(a.out, "README.md"), "w") as f:
        f.write(CARD.format(license=a.license, src="en", tgt=a.suffix, name=a.name or f"{origin} captions ({a.suffix})",
                            origin=origin, rows=len(rows), files=files))
    print(f"{len(rows)} rows in {files} files -> {a.out}")
    return len(rows)


if __name__ == "__main__":
    main()
