"""MONET synthetic thumbnails + captions slimmed for training (reference prepare_monet.py): every parquet under --src
is rewritten to --out (same relative path) without the embedding_* columns (and any other --drop prefixes), with a
`caption_short` column: the shortest non-empty VLM caption of the row, by word count (the one to translate).

  python prepare_monet.py --src raw/monet/v1.2.0/synthetic --source z-image --out data/monet_z_image --workers 8

The reference reads the parquets straight from the Hugging Face Hub; there is no network here, so --src is a local
copy of the dataset folder (with --source, the folder holding one directory per synthetic source, as on the Hub:
z-image, flux-klein, flux-schnell). --max-files takes only the first N parquets (a test). Files already written
are skipped (resume); each is written to a temporary name, zstd compressed, and renamed.
"""
import argparse
import glob
import os
from concurrent.futures import ThreadPoolExecutor, as_completed

import pyarrow as pa
import pyarrow.parquet as pq

CAPTIONS = ["caption_florence-2-large", "caption_internvl-3-8b", "caption_sharegpt4v-7b",
            "caption_gemini-2.5-flash-lite"]


def shortest_caption(table, columns=CAPTIONS):
    cols = [table[c].to_pylist() for c in columns if c in table.column_names]
    out = []
    for caps in zip(*cols) if cols else [() for _ in range(table.num_rows)]:
        clean = [" ".join(c.split()) for c in caps if isinstance(c, str) and c.strip()]
        out.append(min(clean, key=lambda c: len(c.split())) if clean else None)
    return pa.array(out, pa.string())


def slim_one(src, dst, drop=("embedding_",)):
    if os.path.exists(dst):
        return dst, 0, True
    pf = pq.ParquetFile(src)
    keep = [n for n in pf.schema_arrow.names if not n.startswith(tuple(drop))]
    t = pf.read(columns=keep)
    t = t.append_column("caption_short", shortest_caption(t))
    os.makedirs(os.path.dirname(dst) or ".", exist_ok=True)
    pq.write_table(t, dst + ".tmp", compression="zstd")
    os.replace(dst + ".tmp", dst)
    return dst, t.num_rows, False


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--src", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--workers", type=int, default=8)
    p.add_argument("--drop", nargs="*", default=["embedding_"], help="column name prefixes to leave out")
    p.add_argument("--source", default="", choices=["", "z-image", "flux-klein", "flux-schnell"],
                   help="the synthetic source directory under --src (empty: --src is one source's folder)")
    p.add_argument("--max-files", type=int, default=0, help="only the first N parquets (a test)")
    a = p.parse_args(argv)
    src = os.path.join(a.src, a.source) if a.source else a.src
    if not os.path.isdir(src):
        p.error(f"no such source folder: {src}")
    files = sorted(glob.glob(os.path.join(src, "**", "*.parquet"), recursive=True))
    if a.max_files:
        files = files[:a.max_files]
    print(f"{a.source or src}: {len(files)} parquet files -> {a.out}", flush=True)
    jobs = [(f, os.path.join(a.out, os.path.relpath(f, src))) for f in files]
    rows = skipped = 0
    with ThreadPoolExecutor(a.workers) as ex:
        futs = [ex.submit(slim_one, s, d, tuple(a.drop)) for s, d in jobs]
        for i, f in enumerate(as_completed(futs)):
            dst, n, skip = f.result()
            rows += n
            skipped += skip
            print(f"[{i + 1}/{len(futs)}] {dst}: {'done before' if skip else f'{n} rows'}", flush=True)
    print(f"{len(files)} files ({skipped} skipped), {rows} rows written")


if __name__ == "__main__":
    main()
