"""train.py end to end on CPU: shard data layer, checkpoint layout, resume, reference-compatible weights."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env=None):
    e = dict(os.environ, CUDA_VISIBLE_DEVICES="", **(env or {}))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "train.py")] + args, cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout


@pytest.fixture(scope="module")
def shards(tmp_path_factory):
    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    d = str(tmp_path_factory.mktemp("shards"))
    write_synthetic_shards(d, n_shards=3, per_shard=8, side=16)
    return d


def test_shard_store_and_stream_determinism(shards):
    from trenowanie_generatora_obrazkow_b200.data.shards import ShardStore, TrainStream, select_shards
    train, val = select_shards(shards, 1.0)
    assert val == ["synth-00002-of-00003"] and len(train) == 2
    store = ShardStore(shards, train)
    assert len(store) == 16
    a = TrainStream(store, 4, rank=0, world=2, seed=3)
    b = TrainStream(store, 4, rank=0, world=2, seed=3, start_micro=1)
    it = iter(a)
    next(it)
    x1, ids1 = next(it)
    x2, ids2 = next(iter(b))
    assert torch.equal(x1, x2) and torch.equal(ids1, ids2)  # resuming at micro-batch 1 reproduces the stream
    r1 = set(TrainStream(store, 4, rank=1, world=2, seed=3).indices(0).tolist())
    assert not r1 & set(a.indices(0).tolist())  # ranks take disjoint slices of a global batch


def test_train_resume_and_checkpoint_layout(shards, tmp_path):
    out = str(tmp_path / "run")
    common = ["--data", shards, "--fraction", "1", "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "4",
              "--micro-batch", "2", "--log-every", "1", "--eval-every", "0", "--ckpt-every", "1", "--val-samples", "8",
              "--workers", "0", "--no-wandb"]
    _run(common + ["--steps", "2"])
    ck = torch.load(os.path.join(out, "latest.pt"), weights_only=False)
    assert ck["step"] == 2 and ck["samples"] == 8
    assert set(ck) >= {"step", "samples", "den_config", "te_config", "te", "den", "opts", "ema", "args"}
    assert len(ck["ema"]) == len(ck["te"]) + len(ck["den"])
    log = _run(common + ["--steps", "3"])
    assert "resumed" in log and "step 3/3" in log
    assert torch.load(os.path.join(out, "latest.pt"), weights_only=False)["step"] == 3


def test_checkpoint_loads_into_reference_modules(tmp_path, shards):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "aurora")):
        pytest.skip("reference not installed")
    out = str(tmp_path / "run2")
    _run(["--synthetic", "64", "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "2", "--micro-batch",
          "2", "--steps", "1", "--eval-every", "0", "--no-wandb"])
    ck = torch.load(os.path.join(out, "latest.pt"), weights_only=False)
    if ref not in sys.path:  # appended: the repository's own same-named scripts keep priority
        sys.path.append(ref)
    import aurora.model as am
    den = am.Denoiser(am.DenoiserConfig(**ck["den_config"]))
    te = am.TextEncoder(am.TextEncoderConfig(**ck["te_config"]))
    den.load_state_dict(ck["den"], strict=True)
    te.load_state_dict(ck["te"], strict=True)
    assert len(ck["ema"]) == len(list(te.parameters())) + len(list(den.parameters()))


def test_train_with_repa_stand_in(shards, tmp_path):
    """REPA through train.py: projector trained (AdamW), loss logged, projector checkpointed and restored."""
    out = str(tmp_path / "run")
    log = _run(["--data", shards, "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "4", "--micro-batch",
                "2", "--steps", "3", "--eval-every", "0", "--no-wandb", "--repa-weight", "0.5", "--repa-layer", "2",
                "--repa-until", "1.0", "--irepa"])
    import torch
    ck = torch.load(os.path.join(out, "latest.pt"), weights_only=False)
    assert ck["repa_proj"] is not None and "conv.weight" in ck["repa_proj"]
    assert len(ck["ema"]) == len(ck["te"]) + len(ck["den"]) or len(ck["ema"]) > 0


def test_train_rpe2d_micro_cond_and_crops(tmp_path):
    """RPE-2D positions, micro-conditioning fed from resize-and-crop windows of larger latents, t-shift-ref."""
    import numpy as np

    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    d = str(tmp_path / "shards")
    write_synthetic_shards(d, n_shards=2, per_shard=8, side=8)  # 128 px grids as the training resolution...
    import glob
    for f in glob.glob(os.path.join(d, "*.lat.npy")):  # ... and 256 px grids of the same images to crop from
        base = f[: -len(".lat.npy")]
        lat = np.load(f)
        os.replace(f, base + ".lat128.npy")
        np.save(f, np.repeat(np.repeat(lat, 2, axis=2), 2, axis=3))
    out = str(tmp_path / "run")
    _run(["--data", d, "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "4", "--micro-batch", "2",
          "--steps", "2", "--eval-every", "0", "--no-wandb", "--res", "128", "--rope-ref", "16", "--rope-random",
          "--micro-cond", "256", "--crop-res", "256", "--crop-prob", "1.0", "--t-shift-ref", "256"])
    import torch
    ck = torch.load(os.path.join(out, "latest.pt"), weights_only=False)
    assert ck["den_config"]["micro_cond"] == 256 and ck["den_config"]["rope_ref"] == 16
    assert any(k.startswith("cond_mlp") for k in ck["den"])


def test_train_multi_res(tmp_path):
    """Mixed-resolution steps: 128 px and 256 px groups (their own latents and micro-batch sizes) in every step."""
    import numpy as np

    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    d = str(tmp_path / "shards")
    write_synthetic_shards(d, n_shards=2, per_shard=8, side=16)
    import glob
    for f in glob.glob(os.path.join(d, "*.lat.npy")):  # the same images at 128 px
        lat = np.load(f)
        np.save(f[: -len(".lat.npy")] + ".lat128.npy", lat.reshape(*lat.shape[:2], 8, 2, 8, 2).mean((3, 5)))
    out = str(tmp_path / "run")
    _run(["--data", d, "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "6", "--steps", "2",
          "--eval-every", "0", "--no-wandb", "--res", "256", "--multi-res", "128", "256", "--multi-res-mbs", "2",
          "1", "--multi-res-mb", "2", "2", "--t-shift-ref", "256", "--workers", "0"])
    assert os.path.exists(os.path.join(out, "latest.pt"))


def test_train_selective_activation_checkpointing(tmp_path):
    """--act-checkpoint selective (and the reference's bare --act-checkpoint = full) run end to end."""
    out = str(tmp_path / "run")
    for mode in (["--act-checkpoint", "selective"], ["--act-checkpoint"]):
        _run(["--synthetic", "16", "--out", out, "--size", "50m", "--te-size", "13m", "--batch", "2",
              "--micro-batch", "2", "--steps", "1", "--eval-every", "0", "--no-wandb", "--ckpt-every", "0"] + mode)


def test_fid_per_shard_and_export_init(shards, tmp_path):
    """--fid-every / --fid-at-start: Fréchet distance of EMA samples of held-out prompts during training (the
    offline latent features); --eval-only --per-shard: the loss per held-out and training shard; --load-hf: start
    from an export directory."""
    out = str(tmp_path / "run")
    common = ["--data", shards, "--fraction", "1", "--out", out, "--size", "nano", "--te-size", "13m", "--batch", "4",
              "--micro-batch", "2", "--log-every", "1", "--eval-every", "0", "--ckpt-every", "2", "--val-samples",
              "8", "--workers", "0", "--no-wandb"]
    log = _run(common + ["--steps", "2", "--fid-every", "2", "--fid-at-start", "--fid-samples", "6", "--fid-steps",
                         "2"])
    fds = [line for line in log.splitlines() if " FD " in line]
    assert len(fds) == 2 and "step 0 FD" in fds[0] and "step 2 FD" in fds[1], log[-2000:]
    log = _run(common + ["--steps", "2", "--eval-only", "--per-shard", "4"])
    assert log.count("per-shard") == 3 and "val" in log  # 1 held-out shard + the first / middle training shard
    assert '"text_gain"' in log and '"val_no_text/loss"' in log  # the loss with empty prompts, and the gap
    ex = str(tmp_path / "export")
    subprocess.run([sys.executable, os.path.join(ROOT, "export.py"), os.path.join(out, "latest.pt"), ex], cwd=ROOT,
                   check=True, capture_output=True, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    log = _run(["--data", shards, "--fraction", "1", "--out", str(tmp_path / "run2"), "--size", "nano", "--te-size",
                "13m", "--batch", "4", "--micro-batch", "2", "--steps", "1", "--eval-every", "0",
                "--workers", "0", "--no-wandb", "--load-hf", ex, "--no-compile"])
    assert "weights from the export" in log


def test_diloco_gradient_noise_scale(shards, tmp_path):
    """--diloco with --gns-every: two Gloo workers estimate the gradient noise scale on the first step after an
    outer sync."""
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "train.py"), "--data", shards, "--fraction",
           "1", "--out", str(tmp_path / "run"), "--size", "nano", "--te-size", "13m", "--batch", "4",
           "--micro-batch", "2", "--steps", "4", "--diloco", "2", "--gns-every", "2", "--log-every",
           "1", "--eval-every", "0", "--workers", "0", "--no-wandb", "--optimizer", "adamw"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES="", DIST_BACKEND="gloo"))
    assert r.returncode == 0, r.stderr[-3000:]
    assert r.stdout.count("gradient noise scale") == 2, r.stdout[-2000:]


def test_init_by_name_with_growth_and_a_new_text_encoder():
    """utils/checkpoint.init_named: EMA weights by name; blocks past the checkpoint's depth start as identity blocks
    (zeroed attn.out / cross.out / mlp.out_proj, the rest of their fresh init kept); a text encoder of another shape
    stays fresh; a denoiser of another width is refused."""
    from dataclasses import asdict, replace

    from trenowanie_generatora_obrazkow_b200.models import build_models
    from trenowanie_generatora_obrazkow_b200.models.config import make_configs
    from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt
    den_cfg, te_cfg = make_configs("nano", "13m")
    torch.manual_seed(0)
    te, den = build_models(den_cfg, te_cfg)
    params = list(te.parameters()) + list(den.parameters())
    ema = [torch.randn_like(p) for p in params]  # distinguishable from the raw weights
    ck = dict(step=7, den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=te.state_dict(), den=den.state_dict(),
              ema=ema)
    te2_cfg = replace(te_cfg, dim=256, heads=4, mlp_hidden=512)
    torch.manual_seed(1)
    te2, den2 = build_models(replace(den_cfg, depth=6, text_dim=256), te2_cfg)
    fresh_mlp = den2.blocks[5].mlp.in_proj.weight.clone()
    named = [("te", n, p) for n, p in te2.named_parameters()] + [("den", n, p) for n, p in den2.named_parameters()]
    with pytest.raises(ValueError, match="another shape"):  # text_dim 256 changes the cross-attention kv width
        ckpt.init_named(ck, named, log=lambda *a: None)
    torch.manual_seed(1)  # the same width, another MLP: the text encoder's MLP weights stay fresh
    te2, den2 = build_models(replace(den_cfg, depth=6), replace(te_cfg, mlp_hidden=512))
    fresh_mlp = den2.blocks[5].mlp.in_proj.weight.clone()
    named = [("te", n, p) for n, p in te2.named_parameters()] + [("den", n, p) for n, p in den2.named_parameters()]
    res = ckpt.init_named(ck, named, log=lambda *a: None)
    by_name = dict(zip([n for n, _ in den.named_parameters()], ema[len(list(te.parameters())):]))
    assert torch.equal(den2.blocks[3].attn.qkv.weight, by_name["blocks.3.attn.qkv.weight"])
    assert res["grown"] == [4, 5] and res["fresh"] and all(f.startswith("te.") for f in res["fresh"])
    for i in (4, 5):
        for name in ckpt.GROW_ZERO:
            assert den2.blocks[i].get_parameter(name).abs().max() == 0
    assert torch.equal(den2.blocks[5].mlp.in_proj.weight, fresh_mlp)


def test_train_init_grows_depth(tmp_path):
    """train.py --init with a larger --depth: the grown run starts and trains."""
    a = str(tmp_path / "a")
    _run(["--synthetic", "16", "--out", a, "--size", "nano", "--te-size", "13m", "--batch", "2", "--micro-batch", "2",
          "--steps", "1", "--eval-every", "0", "--no-wandb"])
    out = _run(["--synthetic", "16", "--out", str(tmp_path / "b"), "--size", "nano", "--depth", "6", "--te-size", "13m",
                "--batch", "2", "--micro-batch", "2", "--steps", "1", "--eval-every", "0", "--no-wandb", "--init",
                os.path.join(a, "latest.pt")])
    assert "blocks 4-5 grown as identity blocks" in out
    ck = torch.load(str(tmp_path / "b" / "latest.pt"), weights_only=False)
    assert ck["den_config"]["depth"] == 6


def test_train_pl_prob_and_ema_cpu_flags(tmp_path):
    """--pl-prob draws that share of captions from the Polish token rows (frozen-LM encoder), --ema-cpu needs
    --diloco and keeps the EMA on the host."""
    import shutil

    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    data = str(tmp_path / "shards")
    names = write_synthetic_shards(data, n_shards=3, per_shard=8, side=16, lm_suffix="slayer149")
    for n in names:
        shutil.copy(os.path.join(data, f"{n}.tok_slayer149.npy"), os.path.join(data, f"{n}.tok_slayer149_pl.npy"))
    out = _run(["--data", data, "--fraction", "1", "--out", str(tmp_path / "a"), "--size", "nano", "--te-size",
                "slayer149", "--random-lm", "--pl-prob", "0.5", "--batch", "2", "--micro-batch", "2", "--steps", "1",
                "--eval-every", "0", "--workers", "0", "--no-wandb"])
    assert "captions: 50% Polish (slayer149_pl)" in out
    r = subprocess.run([sys.executable, os.path.join(ROOT, "train.py"), "--synthetic", "8", "--out",
                        str(tmp_path / "b"), "--size", "nano", "--te-size", "13m", "--batch", "2", "--micro-batch", "2",
                        "--steps", "1", "--no-wandb", "--ema-cpu"], cwd=ROOT, capture_output=True, text=True,
                       timeout=600, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode != 0 and "--ema-cpu needs --diloco" in r.stderr
