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
