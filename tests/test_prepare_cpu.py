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
