"""Prepared-shard data layer: a catalog of what a data directory holds, a flat sample table, a memory-mapped reader
with vectorised caption / crop draws, and the deterministic per-rank micro-batch stream.

On-disk format (shared with the reference's prepare_data.py / aurora/data.py:1-9 so prepared data serves both
frameworks), one set of files per shard <name>:
  <name>.lat.npy           float16 [N, 128, h, w]  normalised, 2x2-packed FLUX.2 latents (.lat<res>.npy: other grids)
  <name>.tok.npy           uint16  [C, 64]         from-scratch tokenizer captions ([BOS] ids [EOS] PAD)
  <name>.off.npy           int64   [N + 1]         captions of image i are rows off[i]:off[i+1]
  <name>.tok_<enc>[_<lang>].npy uint16 [C, L]      the same caption rows for a frozen-LM tokenizer (PAD 65535)
  <name>.caps[_<lang>].json                         caption strings, flattened in the same row order
  <name>.img.bin + <name>.img.off.npy               encoded images (prepare_images.py)
  manifest.json                                     the full shard list of the source dataset

Design:
  * ``ShardCatalog`` reads a directory listing once; shard selection (hold-out, fractions) works on names only.
  * ``SampleTable`` flattens every shard's offsets once into per-sample (shard, row, first caption, caption count)
    columns, so a batch's lookups are array gathers instead of a search per sample.
  * ``MapCache`` opens memory maps lazily and keeps at most ``max_open`` of them (least recently used is closed), so
    a run over thousands of shards needs a bounded number of file descriptors in every loader worker. The maps share
    the node's page cache across ranks and workers.
  * ``ShardStore.fetch`` draws every random choice of a batch as one vector (caption row, translated-caption switch,
    crop source and window) and then gathers rows shard by shard.
  * ``TrainStream`` yields micro-batch m of a rank from a plan keyed by (epoch, global micro-batch index); the epoch
    permutation is cached; workers take micro-batches round-robin, so resuming at m reproduces the sequence.
Stream semantics kept from the reference (aurora/data.py:271-334): one seeded global permutation per epoch, global
batch k = perm[k G:(k+1) G] with rank r taking its contiguous slice, round-robin loader workers.
"""
import io
import itertools
import json
import os
import re
from collections import OrderedDict

import numpy as np
import torch
from torch.utils.data import IterableDataset, get_worker_info

MAX_TOKENS = 64
PAD_ID, BOS_ID, EOS_ID, NULL_ID, MASK_ID = 0, 2, 3, 4, 5

_SHARD_SUFFIX = re.compile(r"-\d+-of-\d+$")


def null_ids(max_tokens=MAX_TOKENS):
    """Caption row of the empty (CFG-dropped) prompt: [BOS] [NULL] [EOS] then padding."""
    row = np.zeros(max_tokens, dtype=np.int64)
    row[0], row[1], row[2] = BOS_ID, NULL_ID, EOS_ID
    row[3:] = PAD_ID
    return row


def tok_kind(suffix=""):
    """File kind of a tokenisation: ``tok`` (from-scratch tokenizer) or ``tok_<suffix>`` (a frozen LM's)."""
    return "tok_" + suffix if suffix else "tok"


# ------------------------------------------------------------------------------------------------------------------
# shard catalog and selection
# ------------------------------------------------------------------------------------------------------------------
def subset_name(shard):
    """Subset a shard belongs to: its name without the ``-NNNNN-of-NNNNN`` part."""
    return _SHARD_SUFFIX.sub("", shard)


def subsets(names):
    """{subset: sorted shard names}."""
    out = {}
    for n in sorted(names):
        out.setdefault(subset_name(n), []).append(n)
    return out


def evenly_spaced(count, k):
    """k positions spread evenly over range(count), first and last included (duplicates dropped)."""
    if k <= 1:
        return [0]
    step = (count - 1) / (k - 1)
    return sorted({int(round(i * step)) for i in range(k)})


class ShardCatalog:
    """What a data directory holds, from one listing. ``ready`` = shards with captions and latents (or, with
    img_root, with packed images there)."""

    def __init__(self, root, img_root=""):
        self.root, self.img_root = root, img_root
        self.files = set(os.listdir(root)) if os.path.isdir(root) else set()
        img_files = set(os.listdir(img_root)) if img_root and os.path.isdir(img_root) else set()
        with_captions = {f[: -len(".off.npy")] for f in self.files
                         if f.endswith(".off.npy") and not f.endswith(".img.off.npy")}
        if img_root:
            self.ready = sorted(n for n in with_captions if n + ".img.off.npy" in img_files)
        else:
            self.ready = sorted(n for n in with_captions if n + ".lat.npy" in self.files)

    def has(self, name, kind):
        return f"{name}.{kind}.npy" in self.files

    def full(self):
        """Every shard of the source dataset (manifest.json of prepare_data.py), else the ready ones."""
        if "manifest.json" in self.files:
            with open(os.path.join(self.root, "manifest.json")) as f:
                return list(json.load(f)["shards"])
        return list(self.ready)


def list_shards(root, img_root=""):
    return ShardCatalog(root, img_root).ready


def full_shard_list(root, img_root=""):
    return ShardCatalog(root, img_root).full()


def split_shards(names, val_names=None):
    """(train, val) in the order of `names`. Default hold-out: the last shard of each subset that has several."""
    if val_names is None:
        val_names = [group[-1] for group in subsets(names).values() if len(group) > 1]
    held = frozenset(val_names)
    return [n for n in names if n not in held], [n for n in names if n in held]


def select_fraction(train_names, fraction):
    """Evenly spaced shards of every subset, so the subset mix is that of the full data (the same choice for
    prepare_data.py's download and for training)."""
    if fraction >= 1:
        return list(train_names)
    picked = []
    for group in subsets(train_names).values():
        picked += [group[i] for i in evenly_spaced(len(group), max(1, round(fraction * len(group))))]
    return sorted(picked)


def select_shards(root, fraction, tok_suffix="", alt_suffix="", img_root=""):
    """(train, val) names for a fraction of the full dataset; val does not depend on the fraction. Exits with a hint
    when a selected shard is not prepared."""
    cat = ShardCatalog(root, img_root)
    kinds = [tok_kind(tok_suffix)] + ([tok_kind(alt_suffix)] if alt_suffix else [])
    usable = {n for n in cat.ready if all(cat.has(n, k) for k in kinds)}
    train, val = split_shards(cat.full())
    train = select_fraction(train, fraction)
    missing = sorted(n for n in set(train) | set(val) if n not in usable)
    if missing:
        raise SystemExit(f"{len(missing)} shards selected by fraction {fraction} are not prepared in {root} "
                         f"(e.g. {missing[0]}); prepare them first (prepare_data.py convert / tokenize"
                         + (f" --encoder {tok_suffix}" if tok_suffix else "") + ")")
    if not train:
        raise SystemExit(f"no prepared training shards in {root}")
    return train, val


# ------------------------------------------------------------------------------------------------------------------
# sample table, memory maps, image decode
# ------------------------------------------------------------------------------------------------------------------
class SampleTable:
    """Per-sample columns over shards in order: shard, row within the shard, first caption row, caption count."""

    def __init__(self, offsets):
        counts = np.array([len(o) - 1 for o in offsets], dtype=np.int64)
        self.sizes = counts
        self.starts = np.zeros(len(counts) + 1, dtype=np.int64)
        np.cumsum(counts, out=self.starts[1:])
        n = int(self.starts[-1])
        self.shard = np.repeat(np.arange(len(counts), dtype=np.int32), counts)
        self.row = (np.arange(n, dtype=np.int64) - self.starts[:-1][self.shard]).astype(np.int32) if n else \
            np.zeros(0, np.int32)
        self.cap_first = np.concatenate([o[:-1] for o in offsets]).astype(np.int64) if n else np.zeros(0, np.int64)
        self.cap_count = np.concatenate([np.diff(o) for o in offsets]).astype(np.int32) if n else \
            np.zeros(0, np.int32)

    def __len__(self):
        return int(self.starts[-1])


class MapCache:
    """Lazily opened read-only memory maps, at most `max_open` held (the least recently used one is dropped; its
    file handle closes once no array refers to it)."""

    def __init__(self, max_open=1024):
        self.max_open = max_open
        self._maps = OrderedDict()

    def get(self, path, raw_bytes=False):
        m = self._maps.get(path)
        if m is None:
            m = np.memmap(path, dtype=np.uint8, mode="r") if raw_bytes else np.load(path, mmap_mode="r")
            self._maps[path] = m
            while len(self._maps) > self.max_open:
                self._maps.popitem(last=False)
        else:
            self._maps.move_to_end(path)
        return m

    def __getstate__(self):  # loader workers start with no open maps
        return {"max_open": self.max_open, "_maps": OrderedDict()}


def decode_image(data, res):
    """Encoded square image -> (3, res, res) uint8 RGB. A JPEG is decoded at the smallest DCT scale that still covers
    res (PIL draft mode), then resized with PIL's antialiased bicubic filter (prepare_lowres.py's downscale)."""
    from PIL import Image
    with Image.open(io.BytesIO(memoryview(data).tobytes())) as im:
        im.draft("RGB", (res, res))
        rgb = im.convert("RGB")
    if rgb.size != (res, res):
        rgb = rgb.resize((res, res), resample=Image.BICUBIC, reducing_gap=None)
    return np.ascontiguousarray(np.asarray(rgb).transpose(2, 0, 1))


# ------------------------------------------------------------------------------------------------------------------
# store
# ------------------------------------------------------------------------------------------------------------------
class ShardStore:
    """Random access to (latents or images, one caption row per image[, picked caption rows][, micro-conditions]).

    tok_suffix: which tokenisation to read; alt_suffix / alt_prob: with probability alt_prob a sample's caption row
    comes from the translated file instead (same row). lat_kind: latent grid file kind (``lat``, ``lat128``, ...);
    lat_root: folder of the latents / images if not `root`. crops [(lat_kind, root)] / crop_prob: with probability
    crop_prob a sample is a random window (the size of the training grid) of one of these larger grids of the same
    image, with its micro-conditions set to the window (RPE-2D resize-and-crop). cond_base > 0: also return (B, 8)
    micro-conditions in pixels of a cond_base-px original. img_res > 0: decoded uint8 images instead of latents.
    """

    def __init__(self, root, names, tok_suffix="", null_row=None, alt_suffix="", alt_prob=0.0, lat_kind="lat",
                 lat_root="", crops=(), crop_prob=0.0, cond_base=0, img_res=0, max_open=1024):
        if crops and not cond_base:
            raise ValueError("latent crops need micro-conditions (cond_base > 0)")
        if img_res and crops:
            raise ValueError("latent crops and decoded images do not mix")
        self.root, self.names = root, list(names)
        self.lat_root = lat_root or root
        self.lat_kind, self.img_res, self.cond_base = lat_kind, img_res, cond_base
        self.crops, self.crop_prob = [(k, r or root) for k, r in crops], crop_prob
        self.tok = tok_kind(tok_suffix)
        self.alt = tok_kind(alt_suffix) if alt_suffix and alt_prob > 0 else None
        self.alt_prob = alt_prob
        self.null_row = null_ids() if null_row is None else np.asarray(null_row, dtype=np.int64)
        self.table = SampleTable([np.load(self._path(root, n, "off")) for n in self.names])
        self.maps = MapCache(max_open)

    # compatibility views of the table
    @property
    def sizes(self):
        return self.table.sizes

    @property
    def starts(self):
        return self.table.starts

    def __len__(self):
        return len(self.table)

    @staticmethod
    def _path(root, name, kind):
        return os.path.join(root, f"{name}.{kind}.npy")

    def _latents(self, s):
        return self.maps.get(self._path(self.lat_root, self.names[s], self.lat_kind))

    def _tokens(self, s, kind):
        return self.maps.get(self._path(self.root, self.names[s], kind))

    def _images(self, s):
        base = os.path.join(self.lat_root, self.names[s])
        return self.maps.get(base + ".img.bin", raw_bytes=True), self.maps.get(base + ".img.off.npy")

    def _draw(self, n, rng, side):
        """Every random choice of a batch: caption row offsets, translated-caption switch, crop source / window."""
        plan = {"alt": np.zeros(n, bool), "crop": np.zeros(n, bool)}
        if rng is None:
            plan["cap_u"] = np.zeros(n)
            return plan
        plan["cap_u"] = rng.random(n)
        if self.alt:
            plan["alt"] = rng.random(n) < self.alt_prob
        if self.crops and side:
            plan["crop"] = rng.random(n) < self.crop_prob
            plan["crop_src"] = rng.integers(len(self.crops), size=n)
            plan["crop_u"] = rng.random((n, 2))
        return plan

    def fetch(self, indices, rng, rows=False, res=0, captions_only=False):
        """Latents (or images at res) + one caption per image (random with rng, else the first). rows: also
        [shard, caption row] per image (-1 when the image has no caption). captions_only: no latents (empty
        [B, 0] array), captions drawn with the same random choices."""
        if captions_only and self.crops:
            raise ValueError("caption-only reads cannot reproduce crop draws")
        idx = np.asarray(indices, dtype=np.int64)
        n = len(idx)
        t = self.table
        shard, row = t.shard[idx], t.row[idx].astype(np.int64)
        res = res or self.img_res
        if captions_only:
            lat = np.empty((n, 0), dtype=np.float16)
        elif res:
            lat = np.empty((n, 3, res, res), dtype=np.uint8)
        else:
            lat = np.empty((n,) + self._latents(int(shard[0]) if n else 0).shape[1:], dtype=np.float16)
        side = 0 if (captions_only or res) else lat.shape[-1]
        plan = self._draw(n, rng, side)

        # caption rows (vectorised): first + floor(u * count); no caption -> the null row
        count = t.cap_count[idx].astype(np.int64)
        cap = t.cap_first[idx] + np.minimum((plan["cap_u"] * count).astype(np.int64), np.maximum(count - 1, 0))
        has_cap = count > 0
        width = self._tokens(int(shard[0]) if n else 0, self.tok).shape[1]
        ids = np.empty((n, width), dtype=np.int64)
        if not has_cap.all():
            ids[~has_cap] = self.null_row
        picked = np.where(has_cap[:, None], np.stack([shard.astype(np.int64), cap], 1), -1)

        cond = None
        if self.cond_base:
            grid = lat.shape[-1]
            cb = float(self.cond_base)
            cond = np.empty((n, 8), np.float32)
            cond[:] = (cb, cb, 0.0, 0.0, cb, cb, 16.0 * grid, 16.0 * grid)

        for s in np.unique(shard):
            at = np.nonzero(shard == s)[0]
            s = int(s)
            with_cap = at[has_cap[at]]
            if len(with_cap):
                use_alt = plan["alt"][with_cap]
                for kind, sel in ((self.tok, with_cap[~use_alt]), (self.alt, with_cap[use_alt])):
                    if len(sel):
                        ids[sel] = self._tokens(s, kind)[cap[sel]]
            if captions_only:
                continue
            if res:
                blob, off = self._images(s)
                for j in at:
                    lat[j] = decode_image(blob[off[row[j]]:off[row[j] + 1]], res)
                continue
            whole = at[~plan["crop"][at]]
            if len(whole):
                lat[whole] = self._latents(s)[row[whole]]
            for j in at[plan["crop"][at]]:
                kind, croot = self.crops[int(plan["crop_src"][j])]
                src = self.maps.get(self._path(croot, self.names[s], kind))
                big = src.shape[-1]
                r0, c0 = (plan["crop_u"][j] * (big - side + 1)).astype(np.int64)
                lat[j] = src[row[j], :, r0:r0 + side, c0:c0 + side]
                px = self.cond_base / big  # original pixels per source token
                cond[j, 2:6] = (r0 * px, c0 * px, (r0 + side) * px, (c0 + side) * px)
        out = (lat, ids, picked) if rows else (lat, ids)
        return out + (cond,) if self.cond_base else out


class ConcatStore:
    """Several stores (same layout, no micro-conditions) as one index space, in their natural proportions."""

    def __init__(self, stores):
        self.stores = list(stores)
        lens = [len(s) for s in self.stores]
        self.owner = np.repeat(np.arange(len(lens), dtype=np.int32), lens)
        self.local = np.concatenate([np.arange(k, dtype=np.int64) for k in lens]) if lens else np.zeros(0, np.int64)

    def __len__(self):
        return len(self.owner)

    def fetch(self, indices, rng, rows=False, res=0):
        idx = np.asarray(indices, dtype=np.int64)
        parts = {}
        for k in np.unique(self.owner[idx]):
            at = np.nonzero(self.owner[idx] == k)[0]
            got = self.stores[int(k)].fetch(self.local[idx[at]], rng, res=res)
            if len(got) != 2:
                raise ValueError("ConcatStore: stores with micro-conditions are not supported")
            parts[int(k)] = (at, got)
        first = next(iter(parts.values()))[1]
        lat = np.empty((len(idx),) + first[0].shape[1:], dtype=first[0].dtype)
        ids = np.empty((len(idx), first[1].shape[1]), dtype=first[1].dtype)
        for at, (l, i) in parts.values():
            if i.shape[1] != ids.shape[1]:
                raise ValueError("ConcatStore: caption widths differ between stores")
            lat[at], ids[at] = l, i
        return (lat, ids, np.full((len(idx), 2), -1, dtype=np.int64)) if rows else (lat, ids)


class CaptionText:
    """Caption strings by (shard, caption row), from the .caps[_<lang>].json files the token rows were made from; the
    `keep` most recently used shards stay parsed."""

    def __init__(self, root, names, lang="", keep=8):
        self.root, self.names, self.keep = root, list(names), keep
        self.suffix = f"caps_{lang}" if lang else "caps"
        self._parsed = OrderedDict()

    def shard_captions(self, s):
        caps = self._parsed.get(s)
        if caps is None:
            with open(os.path.join(self.root, f"{self.names[s]}.{self.suffix}.json")) as f:
                caps = list(itertools.chain.from_iterable(json.load(f)))
            self._parsed[s] = caps
            if len(self._parsed) > self.keep:
                self._parsed.popitem(last=False)
        else:
            self._parsed.move_to_end(s)
        return caps

    def __call__(self, rows):
        return [self.shard_captions(int(s))[int(c)] if s >= 0 else "" for s, c in rows]


# ------------------------------------------------------------------------------------------------------------------
# stream
# ------------------------------------------------------------------------------------------------------------------
class TrainStream(IterableDataset):
    """Deterministic, resumable per-rank micro-batches (module docstring). sort_pad: order each micro-batch's rows by
    caption length (stable); rows: also yield the picked caption rows; res_groups [(res, n)]: split the micro-batch
    at random into groups decoded at their own resolutions (images as a tuple, captions concatenated in group order);
    captions_only: caption rows without latents."""

    def __init__(self, store, micro_batch, rank, world, seed, start_micro=0, sort_pad=None, rows=False,
                 res_groups=None, captions_only=False):
        if res_groups and sum(n for _, n in res_groups) != micro_batch:
            raise ValueError("res_groups must add up to the micro-batch")
        self.store, self.mb, self.rank, self.world = store, micro_batch, rank, world
        self.seed, self.start, self.sort_pad, self.rows = seed, start_micro, sort_pad, rows
        self.res_groups, self.captions_only = res_groups, captions_only
        self.per_epoch = max(1, len(store) // (micro_batch * world))
        self._perm_key, self._perm = None, None

    def _permutation(self, epoch):
        if self._perm_key != epoch:
            self._perm = np.random.default_rng((self.seed, epoch, 0x70)).permutation(len(self.store))
            self._perm_key = epoch
        return self._perm

    def _rng(self, m, stream):
        return np.random.default_rng((self.seed, m * self.world + self.rank, stream))

    def indices(self, m):
        """Global sample indices of this rank's micro-batch m (sorted: shard-local reads)."""
        epoch, k = divmod(m, self.per_epoch)
        first = (k * self.world + self.rank) * self.mb
        return np.sort(self._permutation(epoch)[first:first + self.mb])

    def _length_order(self, ids):
        if self.sort_pad is None:
            return None
        return np.argsort((ids != self.sort_pad).sum(1), kind="stable")

    def batch(self, m):
        """Micro-batch m of this rank, as the stream yields it."""
        idx = self.indices(m)
        if self.res_groups:
            return self._mixed(idx, m)
        kw = {"captions_only": True} if self.captions_only else {}
        lat, ids, picked, *cond = self.store.fetch(idx, self._rng(m, 1), rows=True, **kw)
        order = self._length_order(ids)
        if order is not None:
            lat, ids, picked, cond = lat[order], ids[order], picked[order], [c[order] for c in cond]
        out = (lat, ids, picked) if self.rows else (lat, ids)
        return tuple(torch.from_numpy(np.ascontiguousarray(x)) for x in out + tuple(cond))

    def _mixed(self, idx, m):
        rng = self._rng(m, 1)
        shuffled = idx[self._rng(m, 2).permutation(len(idx))]
        bounds = np.cumsum([0] + [n for _, n in self.res_groups])
        lats, ids, picked = [], [], []
        for (res, _), a, b in zip(self.res_groups, bounds[:-1], bounds[1:]):
            lat, ids_g, picked_g = self.store.fetch(np.sort(shuffled[a:b]), rng, rows=True, res=res)
            order = self._length_order(ids_g)
            if order is not None:
                lat, ids_g, picked_g = lat[order], ids_g[order], picked_g[order]
            lats.append(torch.from_numpy(np.ascontiguousarray(lat)))
            ids.append(ids_g), picked.append(picked_g)
        out = (tuple(lats), torch.from_numpy(np.concatenate(ids)))
        return out + (torch.from_numpy(np.concatenate(picked)),) if self.rows else out

    def __iter__(self):
        info = get_worker_info()
        worker, workers = (info.id, info.num_workers) if info is not None else (0, 1)
        for m in itertools.count(self.start + worker, workers):
            yield self.batch(m)


# ------------------------------------------------------------------------------------------------------------------
# validation
# ------------------------------------------------------------------------------------------------------------------
def _val_counts(sizes, n):
    """Images taken from each held-out shard: up to ceil(n / shards) from each, in order, n in total at most."""
    per = -(-n // max(1, len(sizes)))
    counts = np.minimum(np.asarray(sizes, dtype=np.int64), per)
    total = np.cumsum(counts)
    return np.clip(counts - np.maximum(total - n, 0), 0, None)


def val_groups(root, names, n):
    """[(shard, count)]: how load_val's n images split over the held-out shards."""
    sizes = [len(np.load(os.path.join(root, f"{name}.off.npy"))) - 1 for name in names]
    return [(name, int(k)) for name, k in zip(names, _val_counts(sizes, n))]


def load_val(root, names, n, tok_suffix="", null_row=None, lat_kind="lat", lat_root="", img_res=0, encode=None,
             chunk=64):
    """The first images of the held-out shards (val_groups' split), first caption each. encode: applied to every
    `chunk` of images as they are read (e.g. the VAE encoder), so only its outputs are kept."""
    store = ShardStore(root, names, tok_suffix, null_row, lat_kind=lat_kind, lat_root=lat_root, img_res=img_res)
    counts = _val_counts(store.sizes, n)
    idx = np.concatenate([store.starts[s] + np.arange(k) for s, k in enumerate(counts)]).astype(np.int64)
    if encode is None:
        lat, ids = store.fetch(idx, None)
        return torch.from_numpy(lat), torch.from_numpy(ids)
    lats, ids = [], []
    for lo in range(0, len(idx), chunk):
        lat, ids_c = store.fetch(idx[lo:lo + chunk], None)
        lats.append(encode(torch.from_numpy(lat)))
        ids.append(torch.from_numpy(ids_c))
    return torch.cat(lats), torch.cat(ids)


def load_val_cached(cache_dir, key_parts, load):
    """``load()`` (e.g. load_val with a VAE encoder) cached in ``cache_dir`` under the SHA-1 of ``key_parts`` (shard
    names, sample count, resolution, encoder identity ...), so a validation set that has to be encoded is encoded
    once per configuration (reference aurora/data.py:337-364). Written to a temporary name and renamed."""
    import hashlib
    key = hashlib.sha1(json.dumps(key_parts, sort_keys=True, default=str).encode()).hexdigest()[:16]
    path = os.path.join(cache_dir, f"val_{key}.pt")
    if os.path.exists(path):
        return torch.load(path, weights_only=True)
    val = load()
    os.makedirs(cache_dir, exist_ok=True)
    torch.save(tuple(val), path + ".tmp")
    os.replace(path + ".tmp", path)
    return val


def write_synthetic_shards(root, n_shards=2, per_shard=16, side=16, caps_per_image=2, tok_len=64, seed=0,
                           lm_suffix="", lm_len=96):
    """Small shard set in the on-disk format (tests and smoke runs; no network needed)."""
    os.makedirs(root, exist_ok=True)
    rng = np.random.default_rng(seed)
    names = [f"synth-{i:05d}-of-{n_shards:05d}" for i in range(n_shards)]
    for name in names:
        lat = rng.standard_normal((per_shard, 128, side, side)).astype(np.float16)
        np.save(os.path.join(root, f"{name}.lat.npy"), lat)
        n_caps = per_shard * caps_per_image
        tok = np.zeros((n_caps, tok_len), dtype=np.uint16)
        for c in range(n_caps):
            L = rng.integers(3, tok_len - 2)
            tok[c, 0], tok[c, 1:L + 1], tok[c, L + 1] = BOS_ID, rng.integers(6, 8192, L), EOS_ID
        np.save(os.path.join(root, f"{name}.tok.npy"), tok)
        np.save(os.path.join(root, f"{name}.off.npy"), np.arange(0, n_caps + 1, caps_per_image, dtype=np.int64))
        if lm_suffix:
            lm = np.full((n_caps, lm_len), 65535, dtype=np.uint16)
            for c in range(n_caps):
                L = rng.integers(1, lm_len)
                lm[c, :L] = rng.integers(0, 60000, L)
            np.save(os.path.join(root, f"{name}.tok_{lm_suffix}.npy"), lm)
        with open(os.path.join(root, f"{name}.caps.json"), "w") as f:
            json.dump([[f"caption {name} {i} {k}" for k in range(caps_per_image)] for i in range(per_shard)], f)
    with open(os.path.join(root, "manifest.json"), "w") as f:
        json.dump({"shards": names}, f)
    return names
