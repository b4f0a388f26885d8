"""The export directory's text -> image pipeline (tokeniser, text encoder, CFG Euler loop) gives the latents of
the sampler run directly on the same weights and token rows."""
import os
from dataclasses import asdict

import torch

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, TextEncoderConfig, build_models
from trenowanie_generatora_obrazkow_b200.sampling.euler import sample
from trenowanie_generatora_obrazkow_b200.sampling.pipeline import HomeIMGPipeline
from trenowanie_generatora_obrazkow_b200.utils.export import export_checkpoint


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {"[UNK]": 1}
    for i, w in enumerate("a red fox in the snow blue sky over hills".split()):
        vocab[w] = 10 + i
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(path)


def test_pipeline_matches_direct_sampling(tmp_path):
    torch.manual_seed(0)
    den_cfg = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16,
                             latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=64, depth=1, heads=1, kv_heads=1, mlp_hidden=128, max_tokens=12)
    te, den = build_models(den_cfg, te_cfg)
    ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=None, step=7, args=dict(t_shift=2.0))
    tok = str(tmp_path / "tokenizer.json")
    _tokenizer(tok)
    ex = str(tmp_path / "export")
    export_checkpoint(ck, ex, tokenizer_json=tok)
    pipe = HomeIMGPipeline.from_pretrained(ex, device="cpu")
    prompts = ["a red fox in the snow", "blue sky over hills"]
    out = pipe(prompts, height=64, num_inference_steps=4, guidance_scale=3.0, seed=5, output_type="latent")
    ids = pipe.tokenize(prompts)
    assert ids[0, 0] == 2 and ids[0, 1] == 10 and ids[0, 7] == 3  # [BOS] a red fox in the snow [EOS]
    want = sample(te.eval(), den.eval(), steps=4, cfg=3.0, seed=5, shift=2.0, latent_size=4, ids=ids)
    assert out.latents.shape == (2, 16, 4, 4) and out.images is None
    assert torch.allclose(out.latents, want, atol=1e-5)


def test_guidance_variants_and_eval_grid(tmp_path):
    """cfg through the guidance module equals the sampler; autoguidance by the model itself is the conditional
    velocity alone; CFG-Zero* skips its first step; eval_grid.py writes the grid."""
    import importlib.util
    import os

    from trenowanie_generatora_obrazkow_b200.sampling.euler import encode_prompts, prompt_noise, sample_latents
    from trenowanie_generatora_obrazkow_b200.sampling.guidance import guided_latents, parse_method
    torch.manual_seed(0)
    den_cfg = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16,
                             latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=64, depth=1, heads=1, kv_heads=1, mlp_hidden=128, max_tokens=12)
    te, den = build_models(den_cfg, te_cfg)
    with torch.no_grad():
        for p in den.parameters():
            p.add_(0.05 * torch.randn_like(p))
    te.eval(), den.eval()
    ids = torch.randint(6, 60, (2, 12))
    text, lens, null, nlen = encode_prompts(te, ids=ids)
    noise = prompt_noise(2, 16, 4, 3, 0)
    a = guided_latents(den, text, lens, null, nlen, noise, steps=4, w=3.0, method="cfg", shift=2.0)
    b = sample_latents(den, text, lens, null, nlen, steps=4, cfg=3.0, shift=2.0, latent_size=4, noise=noise)
    assert torch.allclose(a, b, atol=1e-5)
    ag = guided_latents(den, text, lens, null, nlen, noise, steps=4, w=3.0, method="ag", shift=2.0,
                        guide=(den, text, lens))
    cond = guided_latents(den, text, lens, null, nlen, noise, steps=4, w=3.0, method="cfg", shift=2.0, off=2.0)
    assert torch.allclose(ag, cond, atol=1e-5)
    z1 = guided_latents(den, text, lens, null, nlen, noise, steps=1, method="cfgzero")
    assert torch.equal(z1, noise.float())
    assert parse_method("cfg:3|shift=6|off=0.05") == dict(method="cfg", w=3.0, guide=None, shift=6.0, off=0.05)
    # the CLI over an export directory
    ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=None, step=1, args={})
    ex = str(tmp_path / "export")
    export_checkpoint(ck, ex)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("_repo_eval_grid", os.path.join(root, "eval_grid.py"))
    eg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(eg)
    import json
    json.dump(["a red fox", {"prompt": "blue sky"}], open(tmp_path / "p.json", "w"))
    rec = eg.main([ex, "--prompts", str(tmp_path / "p.json"), "--seeds", "0", "1", "--steps", "2",
                   "--methods", "cfg:3", "cfgzero:3|shift=2", f"ag:{ex}:2", "--out-dir", str(tmp_path / "g")])
    assert len(rec) == 6 and os.path.exists(tmp_path / "g" / "grid_latent_preview.png")


def test_web_app_generates_png(tmp_path):
    """app.py: the form page and POST /generate (a latent preview PNG without a VAE) through FastAPI's test client."""
    import importlib.util
    import io
    import os
    import sys

    from fastapi.testclient import TestClient
    from PIL import Image
    torch.manual_seed(0)
    den_cfg = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16,
                             latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=64, depth=1, heads=1, kv_heads=1, mlp_hidden=128, max_tokens=12)
    te, den = build_models(den_cfg, te_cfg)
    ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=None, step=1, args={})
    tok = str(tmp_path / "tokenizer.json")
    _tokenizer(tok)
    ex = str(tmp_path / "export")
    export_checkpoint(ck, ex, tokenizer_json=tok)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    spec = importlib.util.spec_from_file_location("_repo_app", os.path.join(root, "app.py"))
    app_mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(app_mod)
    client = TestClient(app_mod.build_app(HomeIMGPipeline.from_pretrained(ex, device="cpu"), default_res=64,
                                          steps=2))
    assert "HomeIMG" in client.get("/").text
    r = client.post("/generate", json={"prompt": "a red fox", "steps": 2, "guidance": 3.0, "seed": 7, "res": 64})
    assert r.status_code == 200 and r.headers["x-seed"] == "7"
    assert Image.open(io.BytesIO(r.content)).size == (4, 4)
    r = client.post("/generate", json={"prompt": "a red fox", "steps": 2, "seed": 7, "res": 64, "count": 6})
    assert Image.open(io.BytesIO(r.content)).size == (4 * 4, 2 * 4)  # 6 images, 4 per row


def test_homeimg_loader_isolates_exports(tmp_path):
    """homeimg_loader.py: every export is loaded through its own pipeline.py under its own module, the weights are
    the export's, and the bare ``pipeline`` module name is restored afterwards (reference
    tests/check_homeimg_loader.py)."""
    import sys

    import pytest

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from homeimg_loader import load_homeimg_pipeline

    den_cfg = DenoiserConfig(dim=32, depth=1, heads=1, mlp_hidden=64, text_dim=32, latent_channels=16, latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=32, depth=1, heads=1, kv_heads=1, mlp_hidden=64, max_tokens=8)
    sentinel = object()
    sys.modules["pipeline"] = sentinel
    try:
        classes = set()
        for i in range(3):
            torch.manual_seed(i)
            te, den = build_models(den_cfg, te_cfg)
            ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
                      ema=None, step=i, args=dict(t_shift=1.0))
            ex = str(tmp_path / f"export{i}")
            export_checkpoint(ck, ex)
            pipe = load_homeimg_pipeline(ex, device="cpu")
            assert sys.modules["pipeline"] is sentinel
            assert type(pipe).__module__.startswith("_homeimg_export_")
            classes.add(type(pipe))
            for k, v in den.state_dict().items():
                assert torch.equal(pipe.den.state_dict()[k], v)
        assert len(classes) == 3
        # the same export again: the same module (no second import)
        assert type(load_homeimg_pipeline(str(tmp_path / "export0"), device="cpu")) in classes
        with pytest.raises(ValueError):
            load_homeimg_pipeline(str(tmp_path / "export0"), trust_remote_code=False)
    finally:
        sys.modules.pop("pipeline", None)


def test_eval_suite_parts_resume_and_faces(tmp_path):
    """eval_suite.py: the fixed-suite split into parts with manifests (dry run, refusal to mix settings, resume of an
    identical manifest) and the faces grid over two exports (reference tests/homeimg22.py, face_sweep.py)."""
    import json
    import sys

    import pytest
    from PIL import Image

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import eval_suite as E

    den_cfg = DenoiserConfig(dim=32, depth=1, heads=1, mlp_hidden=64, text_dim=32, latent_channels=16, latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=32, depth=1, heads=1, kv_heads=1, mlp_hidden=64, max_tokens=12)
    tok = str(tmp_path / "tokenizer.json")
    _tokenizer(tok)
    exports = []
    for i in range(2):
        torch.manual_seed(i)
        te, den = build_models(den_cfg, te_cfg)
        ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
                  ema=None, step=i, args=dict(t_shift=1.0))
        exports.append(str(tmp_path / f"ex{i}"))
        export_checkpoint(ck, exports[-1], tokenizer_json=tok)
    prompts = str(tmp_path / "prompts.json")
    json.dump(["a red fox", "blue sky", "snow over hills"], open(prompts, "w"))
    settings = str(tmp_path / "settings.json")
    json.dump(dict(resolution=64, guidance_scale=3.0, time_shift=2.0, num_inference_steps=2, seeds=[0, 1]),
              open(settings, "w"))
    out = str(tmp_path / "suite")
    base = ["suite", exports[0], "--prompts", prompts, "--settings", settings, "--out-dir", out, "--device", "cpu"]
    m = E.main(base + ["--dry-run", "--parts", "2"])
    assert [j["file"] for j in m["images"]] == ["prompt_01_seed_0.png", "prompt_02_seed_0.png", "prompt_03_seed_0.png"]
    for part in (0, 1):
        E.main(base + ["--parts", "2", "--part", str(part)])
    files = sorted(f for f in os.listdir(out) if f.endswith(".png"))
    assert len(files) == 6 and Image.open(os.path.join(out, files[0])).size == (64, 64)
    with pytest.raises(SystemExit):  # the same part again without --resume
        E.main(base + ["--parts", "2", "--part", "0"])
    os.remove(os.path.join(out, "prompt_01_seed_0.png"))
    E.main(base + ["--parts", "2", "--part", "0", "--resume"])  # regenerates only the missing image
    assert os.path.exists(os.path.join(out, "prompt_01_seed_0.png"))
    with pytest.raises(SystemExit):  # another split into the same directory
        E.main(base + ["--parts", "3", "--part", "0"])
    paths = E.main(["faces", f"{exports[0]}:3", f"{exports[1]}:1", "--prompts", prompts, "--seeds", "0", "--res",
                    "64", "--steps", "2", "--cell", "32", "--out-dir", str(tmp_path / "faces"), "--device", "cpu"])
    assert Image.open(paths[0]).size == (220 + 3 * 32, 2 * 32)


def test_export_packs_the_frozen_slayer_lm(tmp_path):
    """export --lm-dir: the LM blocks the refiner reads (token embedding + n_layer - skip_last blocks) travel inside
    text_encoder/ with their description and tokenizer; the export's pipeline samples from them alone and matches
    sampling with the original LM directory."""
    import json

    from safetensors.torch import load_file, save_model

    from trenowanie_generatora_obrazkow_b200.models import LMEncoderConfig
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import SlayerFrozenLM
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    torch.manual_seed(5)
    gcfg = dict(vocab=64, n_layer=3, n_embd=48, n_head=2, block=64)
    lm_dir = tmp_path / "slayer"
    lm_dir.mkdir()
    json.dump(gcfg, open(lm_dir / "config.json", "w"))
    gpt = GPT(GPTConfig(**gcfg)).eval()
    with torch.no_grad():
        for p in gpt.parameters():
            p.add_(0.02 * torch.randn_like(p))
    save_model(gpt, str(lm_dir / "model.safetensors"))
    _tokenizer(str(lm_dir / "tokenizer.json"))
    den_cfg = DenoiserConfig(dim=64, depth=1, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16, latent_size=4)
    te_cfg = LMEncoderConfig(repo=str(lm_dir), tok_suffix="", lm_dim=48, skip_last=1, dim=64, depth=1, heads=1,
                             kv_heads=1, head_dim=64, mlp_hidden=128, max_tokens=10, backend="slayer")
    te, den = build_models(den_cfg, te_cfg)
    ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=None, step=3, args=dict(t_shift=1.0))
    ex = str(tmp_path / "export")
    export_checkpoint(ck, ex, lm_dir=str(lm_dir))
    tensors = load_file(os.path.join(ex, "text_encoder", "diffusion_pytorch_model.safetensors"))
    lm_keys = {k for k in tensors if k.startswith("lm.")}
    assert "lm.tok.weight" in lm_keys and any(k.startswith("lm.blocks.1.") for k in lm_keys)
    assert not any(k.startswith("lm.blocks.2.") for k in lm_keys)  # skip_last = 1: the last block is not packed
    cfg = json.load(open(os.path.join(ex, "text_encoder", "config.json")))
    assert cfg["lm_arch"] == "slayer" and cfg["lm_blocks"] == 2
    assert os.path.exists(os.path.join(ex, "tokenizer", "tokenizer.json"))
    pipe = HomeIMGPipeline.from_pretrained(ex, device="cpu")
    prompts = ["a red fox in the snow"]
    out = pipe(prompts, height=64, num_inference_steps=3, guidance_scale=3.0, seed=2, output_type="latent")
    ref = HomeIMGPipeline.from_pretrained(ex, device="cpu",
                                          frozen_lm=SlayerFrozenLM(str(lm_dir), skip_last=1, dtype=torch.float32))
    want = ref(prompts, height=64, num_inference_steps=3, guidance_scale=3.0, seed=2, output_type="latent")
    assert torch.allclose(out.latents, want.latents, atol=1e-5)


def test_sample_grid_from_an_export(tmp_path):
    """sample.py: the 4 x 2 showcase grid from an export, one call per prompt with the same seed (a cell equals a
    lone call of the pipeline), Polish prompts with --lang pl, latent previews without a VAE."""
    import sys

    import numpy as np
    from PIL import Image

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import importlib.util

    import eval_suite
    spec = importlib.util.spec_from_file_location("_repo_sample", os.path.join(sys.path[0], "sample.py"))
    S = importlib.util.module_from_spec(spec)  # by path: the installed reference has a sample.py of its own
    spec.loader.exec_module(S)

    den_cfg = DenoiserConfig(dim=32, depth=1, heads=1, mlp_hidden=64, text_dim=32, latent_channels=16, latent_size=4)
    te_cfg = TextEncoderConfig(vocab_size=64, dim=32, depth=1, heads=1, kv_heads=1, mlp_hidden=64, max_tokens=12)
    tok = str(tmp_path / "tokenizer.json")
    _tokenizer(tok)
    torch.manual_seed(0)
    te, den = build_models(den_cfg, te_cfg)
    ck = dict(den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=None, step=0, args=dict(t_shift=1.0))
    ex = str(tmp_path / "ex")
    export_checkpoint(ck, ex, tokenizer_json=tok)
    out = S.main([ex, "--out", str(tmp_path / "g" / "grid.png"), "--steps", "2", "--res", "64", "--seed", "3",
                  "--lang", "pl", "--device", "cpu"])
    g = np.asarray(Image.open(out))
    assert g.shape == (2 * 64, 4 * 64, 3) and len(S.PROMPTS) == len(S.PROMPTS_PL) == 8
    pipe = eval_suite.open_pipeline(ex, "cpu")
    settings = dict(resolution=64, guidance_scale=3.0, time_shift=None, num_inference_steps=2)
    cell = np.asarray(Image.fromarray(eval_suite.render(pipe, [S.PROMPTS_PL[5]], 3, settings)[0][0]).resize((64, 64)))
    assert np.array_equal(g[64:, 64:128], cell)  # row 2, column 2: prompt 6 alone with seed 3
