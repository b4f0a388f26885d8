"""prepare_lowres.py (latent-pool method, resume), prepare_monet.py (slimming + shortest caption) and blimp_eval.py
(minimal-pair scoring) on small local inputs."""
import json
import os
import subprocess
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _script(name):
    """This repository's root script ``name``.py as a module (the installed reference has scripts of the same
    names, which another test may have imported first)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(f"_repo_{name}", os.path.join(ROOT, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_prepare_lowres_latent_pool(tmp_path):
    prepare_lowres = _script("prepare_lowres")
    d = tmp_path / "shards"
    d.mkdir()
    for i in range(3):
        np.save(d / f"s{i}.lat.npy", np.random.randn(5, 128, 16, 16).astype(np.float16))
    prepare_lowres.main(["--data", str(d), "--latent-pool", "--sizes", "128", "64", "--batch", "2",
                         "--device", "cpu"])
    a = np.load(d / "s1.lat128.npy")
    src = np.load(d / "s1.lat.npy").astype(np.float32)
    assert a.shape == (5, 128, 8, 8) and np.load(d / "s1.lat64.npy").shape == (5, 128, 4, 4)
    assert np.allclose(a, src.reshape(5, 128, 8, 2, 8, 2).mean((3, 5)), atol=2e-3)
    m = os.path.getmtime(d / "s1.lat128.npy")
    prepare_lowres.main(["--data", str(d), "--latent-pool", "--sizes", "128", "64", "--device", "cpu"])
    assert os.path.getmtime(d / "s1.lat128.npy") == m  # resumed: nothing rewritten


def test_prepare_monet_slims_and_picks_the_shortest_caption(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq

    prepare_monet = _script("prepare_monet")
    src = tmp_path / "raw" / "part-0"
    src.mkdir(parents=True)
    t = pa.table({"prompt": ["p1", "p2"], "embedding_clip": [[0.1, 0.2], [0.3, 0.4]],
                  "caption_florence-2-large": ["a  long caption with   many words", ""],
                  "caption_internvl-3-8b": ["short one", "only this"]})
    pq.write_table(t, src / "f.parquet")
    prepare_monet.main(["--src", str(tmp_path / "raw"), "--out", str(tmp_path / "out"), "--workers", "1"])
    out = pq.read_table(tmp_path / "out" / "part-0" / "f.parquet")
    assert "embedding_clip" not in out.column_names
    assert out["caption_short"].to_pylist() == ["short one", "only this"]


def test_blimp_eval_scores_pairs(tmp_path):
    from safetensors.torch import save_model
    from tokenizers import Tokenizer, models, pre_tokenizers

    blimp_eval = _script("blimp_eval")
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    words = "the cat dog sees sleep sleeps a".split()
    vocab = {"<|endoftext|>": 0, "[UNK]": 1, **{w: i + 2 for i, w in enumerate(words)}}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(str(tmp_path / "tok.json"))
    cfg = dict(vocab=16, n_layer=1, n_embd=32, n_head=2, block=16)
    mdir = tmp_path / "lm"
    mdir.mkdir()
    json.dump(cfg, open(mdir / "config.json", "w"))
    torch.manual_seed(0)
    save_model(GPT(GPTConfig(**cfg)), str(mdir / "model.safetensors"))
    data = tmp_path / "blimp"
    data.mkdir()
    with open(data / "agreement.jsonl", "w") as f:
        for g, b in [("the cat sleeps", "the cat sleep"), ("a dog sees the cat", "a dog see the cat")]:
            f.write(json.dumps({"sentence_good": g, "sentence_bad": b}) + "\n")
    res = blimp_eval.main([str(mdir), "--data", str(data), "--tokenizer", str(tmp_path / "tok.json"),
                           "--device", "cpu", "--out", str(tmp_path / "r.json")])
    acc = res[str(mdir)]["accuracy"]
    assert 0.0 <= acc <= 1.0 and set(res[str(mdir)]["paradigms"]) == {"agreement"}
    sc = blimp_eval.Scorer(str(mdir), str(tmp_path / "tok.json"), "cpu")
    ids = torch.tensor([[0, 2, 3, 7]])
    lp = torch.log_softmax(sc.logits(ids).float(), -1)
    want = sum(lp[0, i, ids[0, i + 1]].item() for i in range(3))
    assert abs(sc(["the cat sleeps"])[0] - want) < 1e-4


def test_translate_and_export_captions(tmp_path):
    """Caption translation with a stand-in engine (upper-cases text, placeholders kept, except one caption whose
    placeholder it drops: that one is retranslated without protection), then the dataset export."""
    tr = _script("translate_captions")
    ex = _script("export_captions")

    def generate(prompts):
        outs = []
        for p in prompts:
            text = p.split("\n\n", 1)[1]
            outs.append(text.replace("<<0>>", "") if "DROP" in text.upper() and "<<0>>" in text else text.upper())
        return outs

    t = tr.Translator(generate, lambda text: tr.PROMPT.format(src="English", tgt="Polish", text=text))
    d = tmp_path / "shards"
    d.mkdir()
    caps = [["a sign that says \"Open\"", "a cat"], ["drop \"Keep\" here", "a cat"]]
    json.dump(caps, open(d / "s0.caps.json", "w"))
    tr.main(["--data", str(d)], translator=t)
    out = json.load(open(d / "s0.caps_pl.json"))
    assert out[0][0] == 'A SIGN THAT SAYS "Open"' and out[0][1] == "A CAT" and out[1][1] == "A CAT"
    assert out[1][0] == 'drop "Keep" here'.upper()  # retried without placeholders
    st = json.load(open(d / "s0.caps_pl.stats.json"))
    assert st["captions"] == 3 and st["quoted"] == 2 and st["retried"] == 1
    n = ex.main(["--data", str(d), "--out", str(tmp_path / "export")])
    import pyarrow.parquet as pq
    rows = pq.read_table(tmp_path / "export" / "data" / "train-00000.parquet").to_pylist()
    assert n == 2 and rows[1]["captions_pl"][1] == "A CAT" and os.path.exists(tmp_path / "export" / "README.md")


def test_blimp_eval_hf_overrides_and_int8_experts(tmp_path):
    """An "hf:" transformers MoE model with --set (a config override: one active expert) and --quant int8 (stacked
    int8 experts); the per-phenomenon summary comes from the rows' linguistics_term."""
    import pytest
    pytest.importorskip("transformers")
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    blimp_eval = _script("blimp_eval")
    words = "the cat dog sees sleep sleeps a".split()
    vocab = {"<|endoftext|>": 0, "[UNK]": 1, **{w: i + 2 for i, w in enumerate(words)}}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(str(tmp_path / "tok.json"))
    cfg = Qwen3MoeConfig(vocab_size=32, hidden_size=64, intermediate_size=128, moe_intermediate_size=32,
                         num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=16, num_experts=4,
                         num_experts_per_tok=2, decoder_sparse_step=1, max_position_embeddings=64)
    torch.manual_seed(0)
    Qwen3MoeForCausalLM(cfg).save_pretrained(str(tmp_path / "moe"))
    data = tmp_path / "blimp"
    data.mkdir()
    with open(data / "agreement.jsonl", "w") as f:
        for g, b in [("the cat sleeps", "the cat sleep"), ("a dog sees the cat", "a dog see the cat")]:
            f.write(json.dumps({"sentence_good": g, "sentence_bad": b, "UID": "agr",
                                "linguistics_term": "subject_verb_agreement"}) + "\n")
    spec = "hf:" + str(tmp_path / "moe")
    sc = blimp_eval.Scorer(spec, str(tmp_path / "tok.json"), "cpu", overrides={"num_experts_per_tok": 1},
                           quant="int8")
    assert sc.model.config.num_experts_per_tok == 1
    fused = [m._fused_moe for m in sc.model.modules() if hasattr(m, "_fused_moe")]
    assert len(fused) == 2 and all(f.quant == "int8" and f.k == 1 for f in fused)
    res = blimp_eval.main([spec, "--data", str(data), "--tokenizer", str(tmp_path / "tok.json"), "--device", "cpu",
                           "--set", "num_experts_per_tok=1", "--quant", "int8"])
    (key, r), = res.items()
    assert key == spec + " {'num_experts_per_tok': 1} int8"
    assert set(r["phenomena"]) == {"subject_verb_agreement"} and set(r["paradigms"]) == {"agr"}
    assert blimp_eval.parse_overrides(["a=1", "b=x", "c=[1,2]"]) == {"a": 1, "b": "x", "c": [1, 2]}


def test_prepare_monet_source_folder_and_max_files(tmp_path):
    """--source picks one synthetic source's folder under --src (the Hub's layout); --max-files keeps the first N."""
    import pyarrow as pa
    import pyarrow.parquet as pq

    prepare_monet = _script("prepare_monet")
    for src in ("z-image", "flux-klein"):
        for i in range(3):
            d = tmp_path / "synthetic" / src / f"part-{i}"
            d.mkdir(parents=True)
            pq.write_table(pa.table({"prompt": [f"{src}{i}"], "caption_florence-2-large": ["a cat"]}), d / "f.parquet")
    prepare_monet.main(["--src", str(tmp_path / "synthetic"), "--source", "flux-klein", "--max-files", "2",
                        "--out", str(tmp_path / "out"), "--workers", "1"])
    got = sorted(os.listdir(tmp_path / "out"))
    assert got == ["part-0", "part-1"]
    assert pq.read_table(tmp_path / "out" / "part-1" / "f.parquet")["prompt"].to_pylist() == ["flux-klein1"]


def test_export_captions_shards_per_file_and_card(tmp_path):
    """--shards-per-file cuts the parquet files at shard boundaries; --repo / --source reach the dataset card."""
    ex = _script("export_captions")
    d = tmp_path / "shards"
    d.mkdir()
    for i, n in enumerate((2, 3, 1)):
        json.dump([[f"cap {i}.{j}"] for j in range(n)], open(d / f"s{i}.caps.json", "w"))
        json.dump([[f"PODPIS {i}.{j}"] for j in range(n)], open(d / f"s{i}.caps_pl.json", "w"))
    n = ex.main(["--data", str(d), "--out", str(tmp_path / "e"), "--shards-per-file", "2",
                 "--repo", "someone/captions-pl", "--source", "z-image"])
    import pyarrow.parquet as pq
    f0 = pq.read_table(tmp_path / "e" / "data" / "train-00000.parquet").to_pylist()
    f1 = pq.read_table(tmp_path / "e" / "data" / "train-00001.parquet").to_pylist()
    assert n == 6 and [r["shard"] for r in f0] == ["s0"] * 2 + ["s1"] * 3 and [r["shard"] for r in f1] == ["s2"]
    card = open(tmp_path / "e" / "README.md").read()
    assert 'load_dataset("someone/captions-pl"' in card and "MONET `z-image`" in card and "# captions-pl" in card


def test_prepare_lowres_vae_options_with_stand_in_vaes(tmp_path):
    """VaeResizer with stand-in VAE objects: --decoder decodes with another object but the encoder's latent
    statistics, --channels-last reaches both modules, --compile wraps the calls (direct calls off CUDA); the
    latent-pool method rejects VAE options."""
    import pytest
    prepare_lowres = _script("prepare_lowres")

    class Mod(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.ones(1, 1, 1, 1))
            self.formats = []

        def to(self, *a, memory_format=None, **k):
            self.formats.append(memory_format)
            return self

        def decode(self, x):
            return x

        def encode(self, x):
            return x

    class Dec:
        def __init__(self):
            self.vae, self.mean, self.std = Mod(), None, None

        def decode(self, z):  # uses the statistics it was given
            img = (z * self.std + self.mean).mean(1, keepdim=True).repeat(1, 3, 16, 16)
            return img.clamp(0, 255).permute(0, 2, 3, 1).to(torch.uint8).numpy()

    class Enc:
        def __init__(self):
            self.vae, self.mean, self.std = Mod(), torch.tensor(7.0), torch.tensor(2.0)

        def __call__(self, img):
            return img.float()[:, :1].repeat(1, 128, 1, 1)[..., ::16, ::16]

    dec, enc = Dec(), Enc()
    r = prepare_lowres.VaeResizer("unused", "cpu", channels_last=True, graphs=True, dec=dec, enc=enc)
    assert dec.mean is enc.mean and dec.std is enc.std
    assert dec.vae.formats == [torch.channels_last] and enc.vae.formats == [torch.channels_last]
    assert isinstance(dec.vae.decode, prepare_lowres.GraphedCall) and isinstance(enc.vae.encode,
                                                                                 prepare_lowres.GraphedCall)
    assert torch.equal(dec.vae.decode(torch.ones(2)), torch.ones(2))  # off CUDA: a direct call
    out = r(np.zeros((2, 128, 16, 16), np.float32), [128])
    assert out[128].shape == (2, 128, 8, 8) and np.allclose(out[128], 7.0)  # 0 * std + mean
    with pytest.raises(AssertionError):
        prepare_lowres.main(["--data", str(tmp_path), "--latent-pool", "--channels-last", "--device", "cpu"])


def test_translate_launch_restarts_crashed_workers(tmp_path):
    """translate_launch.py with a stand-in worker script: one worker per GPU index with CUDA_VISIBLE_DEVICES set,
    rank / world and the `--` arguments passed, a crashed worker restarted until it succeeds, a worker that keeps
    failing stopped after --max-restarts; progress counts translated shards."""
    tl = _script("translate_launch")
    data = tmp_path / "shards"
    data.mkdir()
    for i in range(3):
        (data / f"s{i}.caps.json").write_text("[]")
    worker = tmp_path / "worker.py"
    worker.write_text(
        "import json, os, sys\n"
        "a = sys.argv[1:]\n"
        "rank = int(a[a.index('--rank') + 1])\n"
        "state = os.path.join(os.environ['OUT'], f'attempts{rank}')\n"
        "n = int(open(state).read()) + 1 if os.path.exists(state) else 1\n"
        "open(state, 'w').write(str(n))\n"
        "json.dump(dict(argv=a, gpu=os.environ['CUDA_VISIBLE_DEVICES']),"
        " open(os.path.join(os.environ['OUT'], f'args{rank}.json'), 'w'))\n"
        "if rank == 0 and n < 2: sys.exit(3)\n"  # crashes once
        "if rank == 2: sys.exit(5)\n"  # keeps failing
        "open(os.path.join(a[a.index('--data') + 1], f's{rank}.caps_pl.json'), 'w').write('[]')\n")
    os.environ["OUT"] = str(tmp_path)
    try:
        codes = tl.main(["--gpus", "4", "5", "6", "--data", str(data), "--script", str(worker), "--restart-delay",
                         "0", "--max-restarts", "2", "--progress-every", "0", "--log-dir", str(tmp_path / "logs"),
                         "--", "--max-tokens", "99"])
    finally:
        os.environ.pop("OUT")
    assert codes == {0: 0, 1: 0, 2: 5}
    attempts = [int((tmp_path / f"attempts{r}").read_text()) for r in range(3)]
    assert attempts == [2, 1, 3]  # rank 2: the first run and two restarts
    args = json.load(open(tmp_path / "args1.json"))
    assert args["gpu"] == "5" and args["argv"][-2:] == ["--max-tokens", "99"] and "--world" in args["argv"]
    assert tl.progress(str(data)) == (2, 3)
    assert sorted(os.listdir(tmp_path / "logs")) == ["gpu4.log", "gpu5.log", "gpu6.log"]
