"""Raw latent shards -> the memory-mapped shard layout read by data/shards.py (reference prepare_data.py:83-410).

  python prepare_data.py inspect data/raw/some-shard.npz
  python prepare_data.py convert --src data/raw --out data/x [--fraction 0.1] [--workers 6] [--delete-raw]
  python prepare_data.py tokenize --data data/x --tokenizer path/tokenizer.json
  python prepare_data.py tokenize --data data/x --encoder slayer149 --tokenizer path/tokenizer.json [--lang pl]
  python prepare_data.py tokenize-parquet --parquet-dir data/monet --encoder poziomka --tokenizer tok.json
  python prepare_data.py tokenize-hf --src captions_pl/ --out data/x --encoder poziomka --tokenizer tok.json

convert: every <name>.npz with ``lat`` (N, 128, 16, 16) and ``caps`` becomes <name>.lat.npy (float16) and
<name>.caps.json (the caption entries flattened to lists of strings), written through .tmp files with the .lat.npy
renamed last; manifest.json lists the full source so --fraction picks the same training shards as the training
side. tokenize: <name>.tok.npy ([BOS] ids [EOS] PAD, width 64) + <name>.off.npy (written last), or for a frozen-LM
encoder <name>.tok_<encoder>[_<lang>].npy ([LM BOS] ids PAD=65535). Downloading from the Hub is not available
offline: point --src / --tokenizer at local files.
"""
import argparse
import glob
import json
import os
from concurrent.futures import ProcessPoolExecutor, as_completed

import numpy as np

from trenowanie_generatora_obrazkow_b200.data.shards import select_fraction, split_shards

MAX_TOKENS = 64
PAD_ID, BOS_ID, EOS_ID = 0, 2, 3
# frozen-LM encoders: row width and the LM's BOS id (reference prepare_data.py:171-176)
ENCODERS = {"slayer149": dict(width=96, bos=12285, pad=65535),
            "poziomka": dict(width=256, bos=1, pad=65535)}


def _atomic(path, write):
    tmp = path + ".tmp"
    write(tmp)
    os.replace(tmp, path)


def save_npy(path, arr):
    _atomic(path, lambda tmp: np.save(open(tmp, "wb"), arr))


def save_json(path, obj, **kw):
    def write(tmp):
        with open(tmp, "w") as f:
            json.dump(obj, f, **kw)
    _atomic(path, write)


def flatten_captions(c):
    """One raw ``caps`` entry (str, bytes, JSON text, list, tuple, dict, array, None) -> list of non-empty strings."""
    if isinstance(c, np.ndarray):
        c = c.tolist()
    if isinstance(c, bytes):
        c = c.decode("utf-8", "replace")
    if c is None:
        return []
    if isinstance(c, str):
        s = c.strip()
        if s.startswith(("[", "{")):
            try:
                return flatten_captions(json.loads(s))
            except json.JSONDecodeError:
                pass
        return [s] if s else []
    if isinstance(c, dict):
        return flatten_captions(list(c.values()))
    if isinstance(c, (list, tuple)):
        return [s for x in c for s in flatten_captions(x)]
    return []


def cmd_inspect(a):
    d = np.load(a.file, allow_pickle=True)
    for k in d.files:
        print(f"{k}: shape={d[k].shape} dtype={d[k].dtype}")
    lat = d["lat"][:256].astype(np.float32)
    print(f"lat[:256] mean={lat.mean():.4f} std={lat.std():.4f} (normalised latents: ~0 / ~1)")
    for i in range(min(2, len(d["caps"]))):
        print(f"caps[{i}] {type(d['caps'][i]).__name__}: {repr(d['caps'][i])[:400]} -> {flatten_captions(d['caps'][i])}")


def convert_one(src, out, delete_raw):
    name = os.path.basename(src)[: -len(".npz")]
    d = np.load(src, allow_pickle=True)
    lat = np.ascontiguousarray(d["lat"], dtype=np.float16)
    assert lat.ndim == 4 and lat.shape[1] == 128, lat.shape
    caps = [flatten_captions(c) for c in d["caps"]]
    assert len(caps) == len(lat), (len(caps), len(lat))
    save_json(os.path.join(out, name + ".caps.json"), caps, ensure_ascii=False)
    save_npy(os.path.join(out, name + ".lat.npy"), lat)  # last: the shard is complete
    if delete_raw:
        os.remove(src)
    return name, len(lat), sum(map(len, caps))


def pick_fraction(names, fraction):
    if fraction >= 1:
        return sorted(names)
    train, val = split_shards(sorted(names))
    return sorted(select_fraction(train, fraction) + val)


def cmd_convert(a):
    if a.download:
        raise SystemExit("--download needs the Hugging Face Hub (no network here): download the .npz files "
                         "elsewhere and pass --src")
    os.makedirs(a.out, exist_ok=True)
    files = sorted(glob.glob(os.path.join(a.src, "**", "*.npz"), recursive=True))
    if a.include:
        files = [f for f in files if a.include in f]
    if a.limit:
        files = files[: a.limit]
    by_name = {os.path.basename(f)[: -len(".npz")]: f for f in files}
    save_json(os.path.join(a.out, "manifest.json"), {"shards": sorted(by_name)}, indent=0)
    keep = pick_fraction(list(by_name), a.fraction)
    todo = [n for n in keep if not os.path.exists(os.path.join(a.out, n + ".lat.npy"))]
    print(f"{len(keep)} shards selected, {len(keep) - len(todo)} already converted, {len(todo)} to do")
    with ProcessPoolExecutor(a.workers) as ex:
        futs = [ex.submit(convert_one, by_name[n], a.out, a.delete_raw) for n in todo]
        for i, f in enumerate(as_completed(futs)):
            name, n, c = f.result()
            print(f"[{i + 1}/{len(futs)}] {name}: {n} images, {c} captions", flush=True)


def encode_rows(texts, tokenizer_path, encoder=""):
    from tokenizers import Tokenizer
    tok = Tokenizer.from_file(tokenizer_path)
    lead = "" if encoder else " "  # the from-scratch tokenizer expects a leading space
    enc = tok.encode_batch([lead + " ".join(t.split()) for t in texts], add_special_tokens=False)
    if not encoder:  # [BOS] ids [EOS] PAD
        rows = np.full((len(texts), MAX_TOKENS), PAD_ID, dtype=np.uint16)
        for j, e in enumerate(enc):
            ids = e.ids[: MAX_TOKENS - 2]
            rows[j, 0], rows[j, 1:1 + len(ids)], rows[j, 1 + len(ids)] = BOS_ID, ids, EOS_ID
        return rows
    cfg = ENCODERS[encoder]
    rows = np.full((len(texts), cfg["width"]), cfg["pad"], dtype=np.uint16)
    for j, e in enumerate(enc):
        ids = e.ids[: cfg["width"] - 1]
        rows[j, 0], rows[j, 1:1 + len(ids)] = cfg["bos"], ids
    return rows


def tokenize_one(name, data, tokenizer, encoder="", lang=""):
    with open(os.path.join(data, name + ".caps.json")) as f:
        caps = json.load(f)
    if lang:
        with open(os.path.join(data, f"{name}.caps_{lang}.json")) as f:
            trans = json.load(f)
        assert len(trans) == len(caps), name
    flat, off = [], np.zeros(len(caps) + 1, dtype=np.int64)
    for i, cs in enumerate(caps):
        for k, c in enumerate(cs):
            if c.split():
                t = trans[i][k] if lang and k < len(trans[i]) and str(trans[i][k]).strip() else c
                flat.append(t)
        off[i + 1] = len(flat)
    rows = encode_rows(flat, tokenizer, encoder)
    out = name + (f".tok_{encoder}{'_' + lang if lang else ''}.npy" if encoder else ".tok.npy")
    save_npy(os.path.join(data, out), rows)
    if lang:  # the captions must line up with the English rows
        assert np.array_equal(np.load(os.path.join(data, name + ".off.npy")), off), f"{name}: rows do not line up"
    else:
        save_npy(os.path.join(data, name + ".off.npy"), off)  # last: the shard is tokenised
    return name, len(caps), len(flat)


def cmd_tokenize(a):
    assert not a.lang or a.encoder, "--lang needs --encoder"
    names = sorted(os.path.basename(p)[: -len(".caps.json")] for p in glob.glob(os.path.join(a.data, "*.caps.json")))
    suffix = f".tok_{a.encoder}{'_' + a.lang if a.lang else ''}.npy" if a.encoder else ".off.npy"
    todo = [n for n in names if a.force or not os.path.exists(os.path.join(a.data, n + suffix))]
    if a.lang:
        todo = [n for n in todo if os.path.exists(os.path.join(a.data, f"{n}.caps_{a.lang}.json"))]
    print(f"{len(names)} shards, {len(todo)} to tokenise")
    with ProcessPoolExecutor(a.workers) as ex:
        futs = [ex.submit(tokenize_one, n, a.data, a.tokenizer, a.encoder, a.lang) for n in todo]
        for i, f in enumerate(as_completed(futs)):
            name, n, c = f.result()
            print(f"[{i + 1}/{len(futs)}] {name}: {n} images, {c} captions", flush=True)


def tokenize_caption_table(path, out, tokenizer, encoder, caps_only=False):
    """One parquet of translated captions (columns shard, row, captions_en, captions_pl, pl_flagged: one row per
    image that has captions) -> for every shard named in it, in the layout ``tokenize`` writes: <shard>.caps.json
    (per image its English captions), and unless caps_only <shard>.off.npy, .tok_<encoder>.npy (English) and
    .tok_<encoder>_pl.npy (Polish; a flagged or empty translation falls back to its English caption). The image
    count of a shard comes from its .img.off.npy when present, else from the largest row. Returns
    [(shard, images, captions, English fallbacks)]."""
    import pyarrow.parquet as pq
    table = pq.read_table(path).to_pylist()
    shards = {}
    for r in table:
        shards.setdefault(r["shard"], {})[int(r["row"])] = r
    width, bos, pad = ENCODERS[encoder]["width"], ENCODERS[encoder]["bos"], ENCODERS[encoder]["pad"]
    tok = None
    if not caps_only:
        from tokenizers import Tokenizer
        tok = Tokenizer.from_file(tokenizer)
    done = []
    for shard in sorted(shards):
        rows = shards[shard]
        img_off = os.path.join(out, shard + ".img.off.npy")
        n = len(np.load(img_off)) - 1 if os.path.exists(img_off) else max(rows) + 1
        if max(rows) >= n:
            raise ValueError(f"{shard}: a caption for image {max(rows)} but the shard has {n} images")
        caps, en, pl, fallback = [], [], [], 0
        off = np.zeros(n + 1, dtype=np.int64)
        for i in range(n):
            mine = []
            r = rows.get(i)
            if r is not None:
                flags = r.get("pl_flagged") or [False] * len(r["captions_en"])
                for e, t, bad in zip(r["captions_en"], r.get("captions_pl") or [None] * len(r["captions_en"]), flags):
                    e = " ".join((e or "").split())
                    if not e:
                        continue
                    use_en = bool(bad) or not (t and str(t).strip())
                    mine.append(e)
                    en.append(e)
                    pl.append(e if use_en else " ".join(str(t).split()))
                    fallback += use_en
            caps.append(mine)
            off[i + 1] = len(en)
        save_json(os.path.join(out, shard + ".caps.json"), caps, ensure_ascii=False)
        if not caps_only:
            for texts, suffix in ((en, f".tok_{encoder}.npy"), (pl, f".tok_{encoder}_pl.npy")):
                rows_np = np.full((len(texts), width), pad, dtype=np.uint16)
                for j, e in enumerate(tok.encode_batch(texts, add_special_tokens=False) if texts else []):
                    ids = e.ids[: width - 1]
                    rows_np[j, 0], rows_np[j, 1:1 + len(ids)] = bos, ids
                save_npy(os.path.join(out, shard + suffix), rows_np)
            save_npy(os.path.join(out, shard + ".off.npy"), off)  # last: the shard is tokenised
        done.append((shard, n, len(en), fallback))
    return done


def cmd_tokenize_hf(a):
    if a.download:
        raise SystemExit("tokenize-hf --download needs the Hugging Face Hub (no network here): download the caption "
                         "parquets elsewhere and pass --src")
    if not a.caps_only and not a.tokenizer:
        raise SystemExit("tokenize-hf: --tokenizer (the encoder's tokenizer.json) is needed unless --caps-only")
    files = sorted(glob.glob(os.path.join(a.src, "**", "*.parquet"), recursive=True))
    os.makedirs(a.out, exist_ok=True)
    print(f"{len(files)} caption parquets -> {a.out}", flush=True)
    with ProcessPoolExecutor(a.workers) as ex:
        futs = [ex.submit(tokenize_caption_table, f, a.out, a.tokenizer, a.encoder, a.caps_only) for f in files]
        for i, fut in enumerate(as_completed(futs)):
            got = fut.result()
            print(f"[{i + 1}/{len(futs)}] {len(got)} shards, {sum(g[1] for g in got):,} images, "
                  f"{sum(g[2] for g in got):,} captions, {sum(g[3] for g in got):,} Polish -> English", flush=True)


def cmd_tokenize_parquet(a):
    import pyarrow.parquet as pq
    files = sorted(f for f in glob.glob(os.path.join(a.parquet_dir, "**", "*.parquet"), recursive=True)
                   if os.path.basename(f).count(".") == 1)
    for path in files:
        base = path[: -len(".parquet")]
        texts = [c or "" for c in pq.read_table(path, columns=[a.column])[a.column].to_pylist()]
        if a.lang:
            tr = pq.read_table(f"{base}.{a.lang}.parquet")[f"{a.column}_{a.lang}"].to_pylist()
            texts = [t if t else e for e, t in zip(texts, tr)]
        rows = encode_rows(texts, a.tokenizer, a.encoder)
        save_npy(f"{base}.tok_{a.encoder}{'_' + a.lang if a.lang else ''}.npy", rows)
        if not a.lang:
            save_npy(f"{base}.off.npy", np.arange(len(texts) + 1, dtype=np.int64))
        print(f"{os.path.relpath(path, a.parquet_dir)}: {len(texts)} images", flush=True)


def main(argv=None):
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("inspect")
    s.add_argument("file")
    s = sub.add_parser("convert")
    s.add_argument("--out", default="data/aurora")
    s.add_argument("--src", required=True)
    s.add_argument("--download", action="store_true")
    s.add_argument("--include", default="", help="only shards whose path contains this string")
    s.add_argument("--limit", type=int, default=0, help="only the first N shards (tests)")
    s.add_argument("--fraction", type=float, default=0.1)
    s.add_argument("--delete-raw", action="store_true")
    s.add_argument("--workers", type=int, default=4)
    s = sub.add_parser("tokenize")
    s.add_argument("--data", default="data/aurora")
    s.add_argument("--tokenizer", required=True)
    s.add_argument("--encoder", choices=[""] + sorted(ENCODERS), default="")
    s.add_argument("--lang", default="")
    s.add_argument("--workers", type=int, default=8)
    s.add_argument("--force", action="store_true")
    s = sub.add_parser("tokenize-hf", help="translated-caption parquets (shard, row, captions_en, captions_pl, "
                       "pl_flagged) -> captions + English and Polish token rows per shard")
    s.add_argument("--out", required=True)
    s.add_argument("--src", default="", help="local directory of the caption parquets (no Hub download offline)")
    s.add_argument("--download", action="store_true")
    s.add_argument("--caps-only", action="store_true",
                   help="only <shard>.caps.json (English captions for OPD), when the token rows already exist")
    s.add_argument("--encoder", choices=sorted(ENCODERS), default="poziomka")
    s.add_argument("--tokenizer", default="", help="the encoder's tokenizer.json")
    s.add_argument("--workers", type=int, default=8)
    s = sub.add_parser("tokenize-parquet")
    s.add_argument("--parquet-dir", required=True)
    s.add_argument("--tokenizer", required=True)
    s.add_argument("--encoder", choices=sorted(ENCODERS), default="poziomka")
    s.add_argument("--column", default="caption_short")
    s.add_argument("--lang", default="")
    a = p.parse_args(argv)
    {"inspect": cmd_inspect, "convert": cmd_convert, "tokenize": cmd_tokenize,
     "tokenize-parquet": cmd_tokenize_parquet, "tokenize-hf": cmd_tokenize_hf}[a.cmd](a)


if __name__ == "__main__":
    main()
