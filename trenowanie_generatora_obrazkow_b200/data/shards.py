"""Prepared-shard reader and the deterministic training stream.

On-disk format (the reference's, prepare_data.py / aurora/data.py:1-9), one set of files per shard <name>:
  <name>.lat.npy           float16 [N, 128, h, w]  normalised, 2x2-packed FLUX.2 latents (.lat<res>.npy: other grids)
  <name>.tok.npy           uint16  [C, 64]         from-scratch tokenizer captions ([BOS] ids [EOS] PAD)
  <name>.off.npy           int64   [N + 1]         captions of image i are rows off[i]:off[i+1]
  <name>.tok_<enc>[_<lang>].npy uint16 [C, L]      the same caption rows for a frozen-LM tokenizer (PAD 65535)
  <name>.caps[_<lang>].json                         caption strings, flattened in the same row order
  <name>.img.bin + <name>.img.off.npy               encoded images (prepare_images.py)
  manifest.json                                     the full shard list of the source dataset
Everything is memory-mapped, so ranks and loader workers on a node share the page cache.

Stream semantics (reference aurora/data.py:271-334): every epoch is a seeded global permutation; global batch k is
perm[k*G:(k+1)*G] and rank r takes its contiguous slice; loader workers take micro-batches round-robin; resuming at
micro-batch m reproduces the same sequence. The random generators are keyed by (seed, epoch) and
(seed, micro-batch, rank, 1) so a resumed run draws the same captions / crops.
"""
import glob
import io
import json
import os
import re
import resource

import numpy as np
import torch
from torch.utils.data import IterableDataset, get_worker_info

MAX_TOKENS = 64
PAD_ID, BOS_ID, EOS_ID, NULL_ID, MASK_ID = 0, 2, 3, 4, 5


def null_ids(max_tokens=MAX_TOKENS):
    row = np.full(max_tokens, PAD_ID, dtype=np.int64)
    row[:3] = (BOS_ID, NULL_ID, EOS_ID)
    return row


def tok_kind(suffix=""):
    return f"tok_{suffix}" if suffix else "tok"


def list_shards(root, img_root=""):
    """Shards with captions (.off.npy) and latents (or images under img_root)."""
    names = sorted(os.path.basename(p)[: -len(".off.npy")] for p in glob.glob(os.path.join(root, "*.off.npy"))
                   if not p.endswith(".img.off.npy"))
    if img_root:
        return [n for n in names if os.path.exists(os.path.join(img_root, n + ".img.off.npy"))]
    return [n for n in names if os.path.exists(os.path.join(root, n + ".lat.npy"))]


def subsets(names):
    """Group shard names by subset (the name without its -NNNNN-of-NNNNN suffix)."""
    groups = {}
    for n in sorted(names):
        groups.setdefault(re.sub(r"-\d+-of-\d+$", "", n), []).append(n)
    return groups


def split_shards(names, val_names=None):
    """Hold-out: the last shard of every subset with more than one shard (unless val_names is given)."""
    if val_names is None:
        val_names = [g[-1] for g in subsets(names).values() if len(g) > 1]
    hold = set(val_names)
    return [n for n in names if n not in hold], [n for n in names if n in hold]


def select_fraction(train_names, fraction):
    """Evenly spaced shards of every subset, so the subset mix is that of the full data."""
    if fraction >= 1:
        return list(train_names)
    picked = []
    for g in subsets(train_names).values():
        k = max(1, round(fraction * len(g)))
        picked += [g[i] for i in sorted(set(np.linspace(0, len(g) - 1, k).round().astype(int)))]
    return sorted(picked)


def full_shard_list(root, img_root=""):
    manifest = os.path.join(root, "manifest.json")
    if os.path.exists(manifest):
        with open(manifest) as f:
            return json.load(f)["shards"]
    return list_shards(root, img_root)


def select_shards(root, fraction, tok_suffix="", alt_suffix="", img_root=""):
    """(train, val) names for a fraction of the full dataset; exits with a hint when selected shards are missing."""
    kinds = [tok_kind(tok_suffix)] + ([tok_kind(alt_suffix)] if alt_suffix else [])
    present = [n for n in list_shards(root, img_root)
               if all(os.path.exists(os.path.join(root, f"{n}.{k}.npy")) for k in kinds)]
    train, val = split_shards(full_shard_list(root, img_root))
    train = select_fraction(train, fraction)
    missing = sorted(set(train + val) - set(present))
    if missing:
        raise SystemExit(f"{len(missing)} shards selected by fraction {fraction} are not prepared in {root} "
                         f"(e.g. {missing[0]}); prepare them first (prepare_data.py convert / tokenize)")
    assert train, f"no prepared shards in {root}"
    return train, val


def raise_fd_limit(needed):
    """Each memory map holds a descriptor; raise the soft limit to what the shard count needs."""
    soft, hard = resource.getrlimit(resource.RLIMIT_NOFILE)
    if soft == resource.RLIM_INFINITY or soft >= needed:
        return
    target = needed if hard == resource.RLIM_INFINITY else min(max(needed, 65536), hard)
    resource.setrlimit(resource.RLIMIT_NOFILE, (target, hard))
    if target < needed:
        raise SystemExit(f"need ~{needed} open files for the shards, hard limit is {hard}")


def decode_image(data, res):
    """Encoded square image -> (3, res, res) uint8: JPEG draft decode near res, then bicubic resize."""
    from PIL import Image
    im = Image.open(io.BytesIO(bytes(data)))
    im.draft("RGB", (res, res))
    im = im.convert("RGB")
    if im.size != (res, res):
        im = im.resize((res, res), Image.BICUBIC, reducing_gap=None)
    return np.asarray(im).transpose(2, 0, 1)


class ShardStore:
    """Random access to (latents or images, one caption per image[, caption rows][, micro-conditions])."""

    def __init__(self, root, names, tok_suffix="", null_row=None, alt_suffix="", alt_prob=0.0, lat_kind="lat",
                 lat_root="", crops=(), crop_prob=0.0, cond_base=0, img_res=0):
        self.root, self.names, self.lat_kind = root, list(names), lat_kind
        self.lat_root = lat_root or root
        self.crops, self.crop_prob, self.cond_base, self.img_res = list(crops), crop_prob, cond_base, img_res
        assert not self.crops or cond_base, "crops need micro-conditions (cond_base)"
        assert not (img_res and self.crops), "latent crops and images do not mix"
        self.tok = tok_kind(tok_suffix)
        self.alt = tok_kind(alt_suffix) if alt_suffix and alt_prob > 0 else None
        self.alt_prob = alt_prob
        self.null_row = null_ids() if null_row is None else np.asarray(null_row, dtype=np.int64)
        raise_fd_limit(((3 if self.alt else 2) + len(self.crops)) * len(self.names) + 512)
        self.offs = [np.load(os.path.join(root, f"{n}.off.npy")) for n in self.names]
        self.sizes = np.array([len(o) - 1 for o in self.offs], dtype=np.int64)
        self.starts = np.concatenate([[0], np.cumsum(self.sizes)])
        self._lat = self._tok = self._alt = self._crop = None

    def __len__(self):
        return int(self.starts[-1])

    def _open(self, captions_only=False):
        if self._lat is None and not captions_only:
            if self.img_res:
                self._lat = [(np.memmap(os.path.join(self.lat_root, f"{n}.img.bin"), dtype=np.uint8, mode="r"),
                              np.load(os.path.join(self.lat_root, f"{n}.img.off.npy"))) for n in self.names]
            else:
                self._lat = [np.load(os.path.join(self.lat_root, f"{n}.{self.lat_kind}.npy"), mmap_mode="r")
                             for n in self.names]
            self._crop = [[np.load(os.path.join(r or self.root, f"{n}.{k}.npy"), mmap_mode="r") for n in self.names]
                          for k, r in self.crops]
        if self._tok is None:
            self._tok = [np.load(os.path.join(self.root, f"{n}.{self.tok}.npy"), mmap_mode="r") for n in self.names]
            if self.alt:
                self._alt = [np.load(os.path.join(self.root, f"{n}.{self.alt}.npy"), mmap_mode="r")
                             for n in self.names]

    def fetch(self, indices, rng, rows=False, res=0, captions_only=False):
        """Latents (or images at res) + one caption per image (random with rng, else the first);
        rows: also [shard, caption row] (-1 when the image has no caption)."""
        assert not captions_only or not self.crops
        self._open(captions_only)
        indices = np.asarray(indices)
        picked = np.full((len(indices), 2), -1, dtype=np.int64)
        res = res or self.img_res
        if captions_only:
            lat = np.empty((len(indices), 0), dtype=np.float16)
        elif res:
            lat = np.empty((len(indices), 3, res, res), dtype=np.uint8)
        else:
            lat = np.empty((len(indices), *self._lat[0].shape[1:]), dtype=np.float16)
        ids = np.empty((len(indices), self._tok[0].shape[1]), dtype=np.int64)
        n = lat.shape[-1]
        cb = self.cond_base
        cond = np.tile(np.array([cb, cb, 0, 0, cb, cb, 16 * n, 16 * n], np.float32), (len(indices), 1))
        shard = np.searchsorted(self.starts, indices, side="right") - 1
        for j, (s, gi) in enumerate(zip(shard, indices)):
            i = gi - self.starts[s]
            if captions_only:
                pass
            elif self._crop and rng is not None and rng.random() < self.crop_prob:
                src = self._crop[rng.integers(len(self._crop))][s]
                side = src.shape[-1]
                r, c = rng.integers(0, side - n + 1, size=2)
                lat[j] = src[i, :, r:r + n, c:c + n]
                px = cb / side
                cond[j, 2:6] = r * px, c * px, (r + n) * px, (c + n) * px
            elif res:
                blob, off = self._lat[s]
                lat[j] = decode_image(blob[off[i]:off[i + 1]], res)
            else:
                lat[j] = self._lat[s][i]
            lo, hi = self.offs[s][i], self.offs[s][i + 1]
            if hi == lo:
                ids[j] = self.null_row
                continue
            c = lo if rng is None else rng.integers(lo, hi)
            src_tok = self._alt if (rng is not None and self.alt and rng.random() < self.alt_prob) else self._tok
            ids[j] = src_tok[s][c]
            picked[j] = s, c
        out = (lat, ids, picked) if rows else (lat, ids)
        return out + (cond,) if self.cond_base else out


class ConcatStore:
    """Several stores as one index space (same layout, no micro-conditions)."""

    def __init__(self, stores):
        self.stores = list(stores)
        self.starts = np.concatenate([[0], np.cumsum([len(s) for s in self.stores])])

    def __len__(self):
        return int(self.starts[-1])

    def fetch(self, indices, rng, rows=False, res=0):
        indices = np.asarray(indices)
        which = np.searchsorted(self.starts, indices, side="right") - 1
        lat = ids = None
        for k, store in enumerate(self.stores):
            pos = np.nonzero(which == k)[0]
            if not len(pos):
                continue
            got = store.fetch(indices[pos] - self.starts[k], rng, res=res)
            if lat is None:
                lat = np.empty((len(indices), *got[0].shape[1:]), dtype=got[0].dtype)
                ids = np.empty((len(indices), got[1].shape[1]), dtype=got[1].dtype)
            lat[pos], ids[pos] = got[0], got[1]
        return (lat, ids, np.full((len(indices), 2), -1, dtype=np.int64)) if rows else (lat, ids)


class CaptionText:
    """Caption strings by (shard, caption row), a few parsed shards cached."""

    def __init__(self, root, names, lang="", keep=8):
        self.root, self.names, self.lang, self.keep = root, list(names), lang, keep
        self._cache = {}

    def _flat(self, s):
        if s not in self._cache:
            if len(self._cache) >= self.keep:
                self._cache.pop(next(iter(self._cache)))
            suffix = f"caps_{self.lang}" if self.lang else "caps"
            with open(os.path.join(self.root, f"{self.names[s]}.{suffix}.json")) as f:
                self._cache[s] = [c for caps in json.load(f) for c in caps]
        return self._cache[s]

    def __call__(self, rows):
        return ["" if s < 0 else self._flat(int(s))[int(c)] for s, c in rows]


class TrainStream(IterableDataset):
    """Deterministic, resumable per-rank micro-batches (see the module docstring)."""

    def __init__(self, store, micro_batch, rank, world, seed, start_micro=0, sort_pad=None, rows=False,
                 res_groups=None, captions_only=False):
        self.store, self.mb, self.rank, self.world = store, micro_batch, rank, world
        self.seed, self.start, self.sort_pad, self.rows = seed, start_micro, sort_pad, rows
        self.res_groups, self.captions_only = res_groups, captions_only
        assert not res_groups or sum(n for _, n in res_groups) == micro_batch
        self.per_epoch = max(1, len(store) // (micro_batch * world))

    def indices(self, m):
        """Global sample indices of this rank's micro-batch m."""
        epoch, k = divmod(m, self.per_epoch)
        perm = np.random.default_rng([self.seed, epoch]).permutation(len(self.store))
        g0 = k * self.mb * self.world + self.rank * self.mb
        return np.sort(perm[g0:g0 + self.mb])

    def _sorted(self, ids, *rest):
        if self.sort_pad is None:
            return (ids,) + rest
        order = ids.ne(self.sort_pad).sum(1).argsort(stable=True)
        return (ids[order],) + tuple(r[order] for r in rest)

    def __iter__(self):
        info = get_worker_info()
        wid, nw = (info.id, info.num_workers) if info else (0, 1)
        perm_epoch, perm = -1, None
        m = self.start + wid
        while True:
            epoch, k = divmod(m, self.per_epoch)
            if epoch != perm_epoch:
                perm = np.random.default_rng([self.seed, epoch]).permutation(len(self.store))
                perm_epoch = epoch
            g0 = k * self.mb * self.world + self.rank * self.mb
            idx = np.sort(perm[g0:g0 + self.mb])
            if self.res_groups:
                yield self._mixed(idx, m)
            else:
                kw = {"captions_only": True} if self.captions_only else {}
                got = self.store.fetch(idx, np.random.default_rng([self.seed, m, self.rank, 1]), rows=True, **kw)
                lat, ids, picked, *cond = (torch.from_numpy(x) for x in got)
                ids, lat, picked, *cond = self._sorted(ids, lat, picked, *cond)
                yield ((lat, ids, picked) if self.rows else (lat, ids)) + tuple(cond)
            m += nw

    def _mixed(self, idx, m):
        rng = np.random.default_rng([self.seed, m, self.rank, 1])
        idx = idx[np.random.default_rng([self.seed, m, self.rank, 2]).permutation(len(idx))]
        lats, ids, picked, o = [], [], [], 0
        for res, n in self.res_groups:
            lat, ids_g, picked_g = (torch.from_numpy(x) for x in self.store.fetch(np.sort(idx[o:o + n]), rng,
                                                                                  rows=True, res=res))
            o += n
            ids_g, lat, picked_g = self._sorted(ids_g, lat, picked_g)
            lats.append(lat), ids.append(ids_g), picked.append(picked_g)
        out = (tuple(lats), torch.cat(ids))
        return out + (torch.cat(picked),) if self.rows else out


def val_groups(root, names, n):
    per = -(-n // len(names))
    out, left = [], n
    for name in names:
        k = min(per, len(np.load(os.path.join(root, f"{name}.off.npy"))) - 1, left)
        out.append((name, k))
        left -= k
    return out


def load_val(root, names, n, tok_suffix="", null_row=None, lat_kind="lat", lat_root="", img_res=0, encode=None,
             chunk=64):
    """First n images of the held-out shards (round-robin), first caption each."""
    store = ShardStore(root, names, tok_suffix, null_row, lat_kind=lat_kind, lat_root=lat_root, img_res=img_res)
    per = -(-n // len(names))
    idx = np.concatenate([store.starts[s] + np.arange(min(per, store.sizes[s])) for s in range(len(names))])[:n]
    if encode is None:
        lat, ids = store.fetch(idx, None)
        return torch.from_numpy(lat), torch.from_numpy(ids)
    lats, ids = [], []
    for i in range(0, len(idx), chunk):
        lat, ids_c = store.fetch(idx[i:i + chunk], None)
        lats.append(encode(torch.from_numpy(lat)))
        ids.append(torch.from_numpy(ids_c))
    return torch.cat(lats), torch.cat(ids)


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
