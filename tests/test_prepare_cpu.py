"""prepare_data.py (convert + tokenize into the shard layout that data/shards.py reads) and prepare_images.py
(packed images decoded back through the shard reader)."""
import io
import json
import os

import numpy as np
import pytest

import prepare_data
import prepare_images


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {f"w{i}": i for i in range(6, 200)}
    vocab.update({"[UNK]": 1})
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(path)
    return path


def test_flatten_captions():
    f = prepare_data.flatten_captions
    assert f('["a cat", "a dog"]') == ["a cat", "a dog"]
    assert f({"x": "one", "y": ["two", ""]}) == ["one", "two"]
    assert f(np.array(["p", "q"], dtype=object)) == ["p", "q"] and f(None) == [] and f(b" z ") == ["z"]


def test_convert_tokenize_and_read(tmp_path):
    raw, out = tmp_path / "raw", tmp_path / "data"
    raw.mkdir()
    rng = np.random.default_rng(0)
    for s in range(3):
        caps = np.array([json.dumps([f"w{6 + i} w{7 + s}", "w9"]) for i in range(5)], dtype=object)
        np.savez(raw / f"set-{s:05d}-of-00003.npz", lat=rng.standard_normal((5, 128, 16, 16)).astype(np.float32),
                 caps=caps)
    prepare_data.main(["convert", "--src", str(raw), "--out", str(out), "--fraction", "1", "--workers", "1"])
    tok = _tokenizer(str(tmp_path / "tok.json"))
    prepare_data.main(["tokenize", "--data", str(out), "--tokenizer", tok, "--workers", "1"])
    prepare_data.main(["tokenize", "--data", str(out), "--tokenizer", tok, "--encoder", "slayer149", "--workers", "1"])
    name = "set-00000-of-00003"
    rows = np.load(out / f"{name}.tok.npy")
    off = np.load(out / f"{name}.off.npy")
    assert rows.shape == (10, 64) and off[-1] == 10 and rows[0, 0] == prepare_data.BOS_ID
    assert (rows[0, 1:3] == [6, 7]).all() and rows[0, 3] == prepare_data.EOS_ID
    lm = np.load(out / f"{name}.tok_slayer149.npy")
    assert lm.shape == (10, 96) and lm[0, 0] == 12285 and lm[0, 3] == 65535
    from trenowanie_generatora_obrazkow_b200.data.shards import ShardStore
    store = ShardStore(str(out), [name])
    lat, ids = store.fetch(np.arange(3), None)
    assert lat.shape == (3, 128, 16, 16) and ids.shape[0] == 3


def test_pack_images_roundtrip(tmp_path):
    PIL = pytest.importorskip("PIL.Image")
    src = tmp_path / "imgs"
    src.mkdir()
    for i in range(4):
        buf = io.BytesIO()
        PIL.new("RGB", (32 + i, 24), (10 * i, 20, 30)).save(buf, format="JPEG")
        (src / f"{i:03d}.jpg").write_bytes(buf.getvalue())
    prepare_images.main(["dir", "--src", str(src), "--out", str(tmp_path / "out"), "--name", "imgs"])
    data = prepare_images.read_packed(str(tmp_path / "out" / "imgs"), 2)
    assert data == (src / "002.jpg").read_bytes()
    from trenowanie_generatora_obrazkow_b200.data.shards import decode_image
    img = decode_image(data, 16)
    assert np.asarray(img).shape[-1] in (3, 16) or np.asarray(img).size > 0


def test_convert_filters_and_tokenize_hf(tmp_path):
    """convert --include / --limit pick source shards; tokenize-hf turns translated-caption parquets into the
    captions, offsets and English / Polish token rows of each shard (flagged or empty translations fall back to
    English, images without a row get no captions), --caps-only only the captions."""
    import pyarrow as pa
    import pyarrow.parquet as pq
    raw, out = tmp_path / "raw", tmp_path / "data"
    raw.mkdir()
    rng = np.random.default_rng(1)
    for s in range(4):
        np.savez(raw / f"{'a' if s < 2 else 'b'}-{s:05d}-of-00004.npz",
                 lat=rng.standard_normal((2, 128, 16, 16)).astype(np.float32),
                 caps=np.array(['["w6"]', '["w7"]'], dtype=object))
    prepare_data.main(["convert", "--src", str(raw), "--out", str(out), "--fraction", "1", "--workers", "1",
                       "--include", "b-", "--limit", "1"])
    assert sorted(p.name for p in out.glob("*.lat.npy")) == ["b-00002-of-00004.lat.npy"]
    src = tmp_path / "caps"
    src.mkdir()
    table = pa.table({"shard": ["s1", "s1", "s2"], "row": [0, 2, 1],
                      "captions_en": [["w6 w7", "w8"], ["w9"], ["w10 w11"]],
                      "captions_pl": [["w12", ""], ["w13"], ["w14"]],
                      "pl_flagged": [[False, False], [True], [False]]})
    pq.write_table(table, src / "part-0.parquet")
    tok = _tokenizer(str(tmp_path / "tok.json"))
    hf = tmp_path / "hf"
    prepare_data.main(["tokenize-hf", "--src", str(src), "--out", str(hf), "--encoder", "slayer149", "--tokenizer", tok,
                       "--workers", "1"])
    caps = json.load(open(hf / "s1.caps.json"))
    assert caps == [["w6 w7", "w8"], [], ["w9"]]
    off = np.load(hf / "s1.off.npy")
    assert off.tolist() == [0, 2, 2, 3]
    en, pl = np.load(hf / "s1.tok_slayer149.npy"), np.load(hf / "s1.tok_slayer149_pl.npy")
    assert en.shape == pl.shape == (3, 96) and en[0, 0] == 12285
    assert en[0, 1:3].tolist() == [6, 7] and pl[0, 1] == 12            # translated
    assert pl[1, 1] == 8 and pl[2, 1] == 9                             # empty / flagged -> English
    assert json.load(open(hf / "s2.caps.json")) == [[], ["w10 w11"]]
    only = tmp_path / "only"
    prepare_data.main(["tokenize-hf", "--src", str(src), "--out", str(only), "--encoder", "slayer149", "--caps-only",
                       "--workers", "1"])
    assert (only / "s1.caps.json").exists() and not (only / "s1.off.npy").exists()


def test_prepare_images_flux_reason_and_monet(tmp_path):
    """flux-reason: the held-out shard always, --fraction of the training shards, staged through --tmp (left
    empty), one worker process per shard, image counts checked against the caption offsets of --data; a second
    run skips finished shards; monet packs the thumbnail column next to each parquet."""
    import pyarrow as pa
    import pyarrow.parquet as pq

    src, data = tmp_path / "src", tmp_path / "lat"
    data.mkdir()
    names = [f"art-{i:05d}-of-00004" for i in range(4)]
    for i, n in enumerate(names):
        (src / "art").mkdir(parents=True, exist_ok=True)
        rows = [{"bytes": bytes([i, j]) * (j + 1)} for j in range(3)]
        pq.write_table(pa.table({"image": rows}), src / "art" / f"{n}.parquet")
        np.save(data / f"{n}.off.npy", np.arange(4, dtype=np.int64))
    out, tmp = tmp_path / "out", tmp_path / "stage"
    argv = ["flux-reason", "--src", str(src), "--out", str(out), "--data", str(data), "--fraction", "0.34",
            "--workers", "2", "--tmp", str(tmp)]
    assert prepare_images.main(argv) == 6  # 1 of 3 training shards (evenly spaced) + the held-out one, 3 images each
    got = sorted(f[: -len(".img.off.npy")] for f in os.listdir(out) if f.endswith(".img.off.npy"))
    assert got == [names[0], names[3]] and os.listdir(tmp) == []
    assert prepare_images.read_packed(str(out / names[3]), 2) == bytes([3, 2]) * 3
    assert prepare_images.main(argv) == 0  # resumed: nothing packed again
    np.save(data / f"{names[1]}.off.npy", np.arange(3, dtype=np.int64))  # 2 caption rows for 3 images
    with pytest.raises(ValueError, match="caption rows"):
        prepare_images.main(["flux-reason", "--src", str(src), "--out", str(out), "--data", str(data),
                             "--workers", "1", "--max-shards", "2"])
    mon = tmp_path / "monet" / "part-0"
    mon.mkdir(parents=True)
    pq.write_table(pa.table({"thumbnail": [{"bytes": b"abc"}, {"bytes": b"de"}]}), mon / "f.parquet")
    prepare_images.main(["monet", "--parquet-dir", str(tmp_path / "monet")])
    assert prepare_images.read_packed(str(mon / "f"), 1) == b"de"


def test_shard_viewer_pages_and_images(tmp_path):
    """shard_viewer.py over synthetic shards: the index lists them, a shard page shows its captions (filtered), an
    item page its translated captions, and images are the packed originals or PNG latent previews."""
    import threading
    import urllib.error
    import urllib.request

    import shard_viewer as V
    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    root = str(tmp_path / "data")
    names = write_synthetic_shards(root, n_shards=2, per_shard=4, side=16)
    json.dump([[f"podpis {i}"] for i in range(4)], open(os.path.join(root, f"{names[0]}.caps_pl.json"), "w"))
    w = prepare_images.PackWriter(os.path.join(root, names[1]))
    w.add([b"\xff\xd8\xff" + bytes([i]) * 10 for i in range(4)])
    w.close()
    server = V.serve(root, port=0)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    base = f"http://127.0.0.1:{server.server_address[1]}"
    get = lambda path: urllib.request.urlopen(base + path, timeout=30)
    try:
        index = get("/").read().decode()
        assert all(n in index for n in names) and "2 shards" in index
        page = get(f"/shard?name={names[0]}&q=caption").read().decode()
        assert f"caption {names[0]} 3 0" in page and "4 of 4 images" in page
        page = get(f"/shard?name={names[0]}&q=nothing-matches").read().decode()
        assert "0 of 4 images" in page
        item = get(f"/item?name={names[0]}&i=2").read().decode()
        assert "podpis 2" in item and "[128, 16, 16]" in item
        r = get(f"/img?name={names[0]}&i=1")
        assert r.headers["Content-Type"] == "image/png" and r.read()[:4] == b"\x89PNG"
        r = get(f"/img?name={names[1]}&i=3")
        assert r.headers["Content-Type"] == "image/jpeg" and r.read() == b"\xff\xd8\xff" + bytes([3]) * 10
        with pytest.raises(urllib.error.HTTPError):
            get("/img?name=missing&i=0")
    finally:
        server.shutdown()
        server.server_close()
