"""Shard data layer: sample table lookups, bounded memory maps, caption / translated-caption / crop draws, concat
stores, caption text, validation split and loader-worker determinism (all on CPU, synthetic shards)."""
import json
import os

import numpy as np
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.data import shards as S


@pytest.fixture(scope="module")
def root(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("data"))
    S.write_synthetic_shards(d, n_shards=3, per_shard=6, side=8, caps_per_image=3, lm_suffix="lm")
    # shard 1: image 2 has no caption (offsets with an empty span), translated rows for the alt-caption switch
    name = "synth-00001-of-00003"
    np.save(os.path.join(d, f"{name}.off.npy"), np.array([0, 3, 6, 6, 9, 12, 15], dtype=np.int64))
    for n in S.list_shards(d):
        tok = np.load(os.path.join(d, f"{n}.tok_lm.npy"))
        np.save(os.path.join(d, f"{n}.tok_lm_pl.npy"), np.full_like(tok, 7))
        big = np.load(os.path.join(d, f"{n}.lat.npy"))
        np.save(os.path.join(d, f"{n}.lat16.npy"), np.repeat(np.repeat(big, 2, 2), 2, 3))
    return d


def test_sample_table_matches_offsets(root):
    names = S.list_shards(root)
    offs = [np.load(os.path.join(root, f"{n}.off.npy")) for n in names]
    t = S.SampleTable(offs)
    k = 0
    for s, o in enumerate(offs):
        for r in range(len(o) - 1):
            assert (t.shard[k], t.row[k], t.cap_first[k], t.cap_count[k]) == (s, r, o[r], o[r + 1] - o[r])
            k += 1
    assert len(t) == k


def test_fetch_captions_null_rows_and_alt(root):
    names = S.list_shards(root)
    store = S.ShardStore(root, names, "lm", null_row=np.full(96, 65534), alt_suffix="lm_pl", alt_prob=0.5)
    idx = np.arange(len(store))
    lat, ids, picked = store.fetch(idx, np.random.default_rng(0), rows=True)
    empty = store.starts[1] + 2  # shard 1, image 2 has no caption
    assert (ids[empty] == 65534).all() and (picked[empty] == -1).all()
    tok = {n: np.load(os.path.join(root, f"{n}.tok_lm.npy")) for n in names}
    n_alt = 0
    for j in idx:
        if j == empty:
            continue
        s, c = picked[j]
        lo = np.load(os.path.join(root, f"{names[s]}.off.npy"))[store.table.row[j]]
        assert lo <= c < lo + store.table.cap_count[j]
        if (ids[j] == 7).all():
            n_alt += 1
        else:
            assert (ids[j] == tok[names[s]][c]).all()
        ref = np.load(os.path.join(root, f"{names[s]}.lat.npy"))[store.table.row[j]]
        assert np.array_equal(lat[j], ref)
    assert 0 < n_alt < len(idx) - 1
    _, first = store.fetch(idx[:4], None)  # no rng: the first caption, never the translation
    assert (first[0] == tok[names[0]][0]).all()


def test_crops_and_micro_conditions(root):
    names = S.list_shards(root)
    store = S.ShardStore(root, names, crops=[("lat16", "")], crop_prob=1.0, cond_base=256)
    lat, ids, cond = store.fetch(np.arange(6), np.random.default_rng(1))
    assert lat.shape == (6, 128, 8, 8)
    big = np.load(os.path.join(root, f"{names[0]}.lat16.npy"))
    px = 256 / 16
    for j in range(6):
        r0, c0 = int(round(cond[j, 2] / px)), int(round(cond[j, 3] / px))
        assert np.array_equal(lat[j], big[j, :, r0:r0 + 8, c0:c0 + 8])
        assert cond[j, 4] - cond[j, 2] == 8 * px and (cond[j, :2] == 256).all() and (cond[j, 6:] == 128).all()
    plain = S.ShardStore(root, names, cond_base=256).fetch(np.arange(2), np.random.default_rng(1))[2]
    assert (plain == np.array([256, 256, 0, 0, 256, 256, 128, 128], np.float32)).all()


def test_map_cache_is_bounded(root):
    names = S.list_shards(root)
    store = S.ShardStore(root, names, max_open=2)
    store.fetch(np.arange(len(store)), np.random.default_rng(0))
    assert len(store.maps._maps) <= 2


def test_concat_store_and_caption_text(root):
    names = S.list_shards(root)
    a, b = S.ShardStore(root, names[:1]), S.ShardStore(root, names[1:])
    cat = S.ConcatStore([a, b])
    assert len(cat) == len(a) + len(b)
    lat, ids = cat.fetch(np.array([0, len(a), len(a) + 1]), None)
    assert np.array_equal(lat[1], b.fetch(np.array([0]), None)[0][0])
    text = S.CaptionText(root, names, keep=1)
    caps = text([(0, 1), (-1, -1), (2, 4)])
    assert caps[0] == f"caption {names[0]} 0 1" and caps[1] == "" and caps[2] == f"caption {names[2]} 1 1"
    assert len(text._parsed) == 1


def test_val_split_matches_a_plain_loop(root):
    for sizes, n in (([5, 5, 5], 7), ([3, 3, 3], 4), ([1, 9, 2], 10), ([4], 9)):
        per, left, want = -(-n // len(sizes)), n, []
        for size in sizes:
            k = min(per, size, left)
            want.append(k)
            left -= k
        assert S._val_counts(sizes, n).tolist() == want
    names = S.list_shards(root)
    lat, ids = S.load_val(root, names, 8)
    assert lat.shape[0] == 8 and [k for _, k in S.val_groups(root, names, 8)] == [3, 3, 2]


def test_selection_fraction_and_holdout(tmp_path):
    names = [f"a-{i:05d}-of-00010" for i in range(10)] + [f"b-{i:05d}-of-00002" for i in range(2)] + ["c"]
    train, val = S.split_shards(names)
    assert val == ["a-00009-of-00010", "b-00001-of-00002"]
    picked = S.select_fraction(train, 0.5)  # a: 9 train shards -> 4 of them; b, c: one each
    assert picked == sorted([f"a-{i:05d}-of-00010" for i in (0, 3, 5, 8)] + ["b-00000-of-00002", "c"])
    for count in range(1, 40):
        for k in range(1, count + 1):  # the same positions as rounding an evenly spaced float grid
            assert S.evenly_spaced(count, k) == sorted(set(np.linspace(0, count - 1, k).round().astype(int).tolist()))


def test_stream_workers_and_resume_agree(root):
    names = S.list_shards(root)
    store = S.ShardStore(root, names, "lm", null_row=np.full(96, 65535))
    one = iter(S.TrainStream(store, 2, rank=1, world=2, seed=5, sort_pad=65535, rows=True))
    seq = [next(one) for _ in range(6)]
    loader = torch.utils.data.DataLoader(S.TrainStream(store, 2, rank=1, world=2, seed=5, sort_pad=65535, rows=True),
                                         batch_size=None, num_workers=2)
    par = [b for _, b in zip(range(6), loader)]
    resumed = next(iter(S.TrainStream(store, 2, rank=1, world=2, seed=5, sort_pad=65535, rows=True, start_micro=3)))
    for x, y in zip(seq, par):
        assert all(torch.equal(u, v) for u, v in zip(x, y))
    assert all(torch.equal(u, v) for u, v in zip(seq[3], resumed))
    lens = (seq[0][1] != 65535).sum(1)
    assert (lens[:-1] <= lens[1:]).all()  # sorted by caption length
    per_epoch = len(store) // 4
    epoch = [set(S.TrainStream(store, 2, r, 2, 5).indices(m).tolist()) for m in range(per_epoch) for r in range(2)]
    assert len(set().union(*epoch)) == sum(map(len, epoch))  # an epoch visits each sample at most once


def test_mixed_resolution_groups(tmp_path):
    pytest.importorskip("PIL.Image")
    import io

    from PIL import Image
    d = str(tmp_path)
    blobs = []
    for i in range(4):
        buf = io.BytesIO()
        Image.new("RGB", (64, 64), (40 * i, 10, 200)).save(buf, format="JPEG")
        blobs.append(buf.getvalue())
    name = "imgs-00000-of-00001"
    with open(os.path.join(d, f"{name}.img.bin"), "wb") as f:
        f.write(b"".join(blobs))
    np.save(os.path.join(d, f"{name}.img.off.npy"), np.cumsum([0] + [len(b) for b in blobs]).astype(np.int64))
    np.save(os.path.join(d, f"{name}.off.npy"), np.arange(5, dtype=np.int64))
    np.save(os.path.join(d, f"{name}.tok.npy"), np.tile(S.null_ids().astype(np.uint16), (4, 1)))
    with open(os.path.join(d, f"{name}.caps.json"), "w") as f:
        json.dump([["x"]] * 4, f)
    store = S.ShardStore(d, [name], img_res=32)
    stream = S.TrainStream(store, 4, 0, 1, 0, res_groups=[(16, 1), (32, 3)])
    lats, ids = next(iter(stream))
    assert lats[0].shape == (1, 3, 16, 16) and lats[1].shape == (3, 3, 32, 32) and ids.shape == (4, 64)
