"""Tooling on CPU: WSM / QAM coefficients, merge.py, sample_ckpt.py with export, checkpoint helpers."""
import glob
import os
import subprocess
import sys

import pytest
import torch

from trenowanie_generatora_obrazkow_b200.optim.merge import merge_coefficients

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_wsm_mean_is_uniform_and_qam_sums_to_one():
    assert merge_coefficients("mean", 5, "wsm") == pytest.approx([0.2] * 5)
    for scheme in ("mean", "1-sqrt", "cosine"):
        for method in ("wsm", "qam"):
            c = merge_coefficients(scheme, 6, method)
            assert sum(c) == pytest.approx(1.0) and min(c) >= -1e-9
    assert merge_coefficients("cosine", 1) == [1.0]


def test_qam_matches_polynomial_product():
    w = [0.9, 0.5, 0.2]
    import numpy as np
    poly = np.array([1.0])
    for wj in w:
        poly = np.convolve(poly, [1 - wj, wj])
    from trenowanie_generatora_obrazkow_b200.optim import merge as M
    old = M.decay_profile
    M.decay_profile = lambda scheme, k: w
    try:
        assert M.merge_coefficients("mean", 4, "qam") == pytest.approx(list(poly))
    finally:
        M.decay_profile = old


def _py(script, *args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, script), *args], cwd=ROOT, capture_output=True, text=True,
                       timeout=600, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout


def test_train_merge_sample_export_chain(tmp_path):
    run = str(tmp_path / "run")
    _py("train.py", "--synthetic", "64", "--out", run, "--size", "50m", "--te-size", "13m", "--batch", "2",
        "--micro-batch", "2", "--steps", "5", "--eval-every", "0", "--merge-every", "1", "--merge-start", "0.2",
        "--no-wandb")
    assert len(glob.glob(os.path.join(run, "merge", "step_*.pt"))) >= 3
    out = _py("merge.py", run, "--synthetic-val", "16", "--windows", "0.6", "--schemes", "mean")
    assert "best:" in out and os.path.exists(os.path.join(run, "merged.pt"))
    so = str(tmp_path / "samples")
    _py("sample_ckpt.py", os.path.join(run, "merged.pt"), "--out-dir", so, "--steps", "2", "--prompt", "a cat",
        "--export")
    assert os.path.exists(os.path.join(so, "transformer", "diffusion_pytorch_model.safetensors"))
    # the export reloads through the directory path
    _py("sample_ckpt.py", so, "--out-dir", str(tmp_path / "s2"), "--steps", "1", "--prompt", "x")
    # no --prompt: the English and Polish showcase grids, the same noise per prompt in both
    _py("sample_ckpt.py", so, "--out-dir", str(tmp_path / "s3"), "--steps", "1", "--batch", "8")
    made = set(os.listdir(tmp_path / "s3"))
    assert {"grid_en_latent_preview.png", "grid_pl_latent_preview.png", "en_latents.pt", "pl_latents.pt"} <= made


def test_export_import_roundtrip(tmp_path):
    """train.py checkpoint -> export.py (diffusers layout) -> import_homeimg.py init checkpoint -> same weights; the
    exported transformer loads strictly into the reference's Denoiser when the reference is installed."""
    import json

    from safetensors.torch import load_file
    run = str(tmp_path / "run")
    _py("train.py", "--synthetic", "32", "--out", run, "--size", "50m", "--te-size", "13m", "--batch", "2",
        "--micro-batch", "2", "--steps", "2", "--eval-every", "0", "--no-wandb")
    ex = str(tmp_path / "export")
    _py("export.py", os.path.join(run, "latest.pt"), ex, "--time-shift", "3")
    index = json.load(open(os.path.join(ex, "model_index.json")))
    assert index["transformer"][1] == "AuroraDenoiser" and index["weights"] == "EMA"
    tcfg = json.load(open(os.path.join(ex, "transformer", "config.json")))
    assert tcfg["time_shift"] == 3.0 and tcfg["dim"] == 640
    # --ref: another export's vae/ and tokenizer/ are carried over
    ref_dir = tmp_path / "released"
    (ref_dir / "vae").mkdir(parents=True)
    (ref_dir / "tokenizer").mkdir()
    json.dump({"_class_name": "AutoencoderKLFlux2"}, open(ref_dir / "vae" / "config.json", "w"))
    json.dump({"model": {"type": "BPE"}}, open(ref_dir / "tokenizer" / "tokenizer.json", "w"))
    ex2 = str(tmp_path / "export2")
    _py("export.py", os.path.join(run, "latest.pt"), ex2, "--ref", str(ref_dir))
    assert json.load(open(os.path.join(ex2, "vae", "config.json")))["_class_name"] == "AutoencoderKLFlux2"
    assert json.load(open(os.path.join(ex2, "tokenizer", "tokenizer.json")))["model"]["type"] == "BPE"
    init = str(tmp_path / "init.pt")
    _py("import_homeimg.py", ex, init)
    ck = torch.load(os.path.join(run, "latest.pt"), weights_only=False)
    ini = torch.load(init, weights_only=False)
    den_params = list(ck["den"].keys())
    n_te = len(ck["te"])
    # the export holds the EMA: the imported live weights equal the checkpoint's EMA list
    for i, k in enumerate(den_params):
        assert torch.equal(ini["den"][k], ck["ema"][n_te + i])
    ref = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(os.path.join(ref, "aurora")):
        sys.path.insert(0, ref)
        try:
            from aurora.model import Denoiser, DenoiserConfig as RefCfg
            fields = {k: v for k, v in tcfg.items() if k in RefCfg.__dataclass_fields__}
            Denoiser(RefCfg(**fields)).load_state_dict(
                load_file(os.path.join(ex, "transformer", "diffusion_pytorch_model.safetensors")))
        finally:
            sys.path.remove(ref)
    # the init checkpoint trains
    _py("train.py", "--synthetic", "32", "--out", str(tmp_path / "run2"), "--init", init, "--size", "50m",
        "--te-size", "13m", "--batch", "2",
        "--micro-batch", "2", "--steps", "1", "--eval-every", "0", "--no-wandb")


def test_merge_assemble_streams_a_weighted_sum(tmp_path):
    """merge.assemble builds sum_i c_i theta_i in place from checkpoints opened one at a time."""
    import merge as M
    files = []
    for i in range(3):
        f = str(tmp_path / f"step_{i:07d}.pt")
        torch.save({"step": 10 * i, "te": {"w": torch.full((3,), float(i))}, "den": {"b": torch.arange(4.0) * i}}, f)
        files.append(f)
    stream = M.CheckpointStream(files)
    assert stream.steps == [0, 10, 20]
    targets = {"te": {"w": torch.zeros(3)}, "den": {"b": torch.zeros(4, dtype=torch.bfloat16)}}
    M.assemble(targets, stream, {1: 0.25, 2: 0.75})
    assert torch.allclose(targets["te"]["w"], torch.full((3,), 1.75))
    assert torch.allclose(targets["den"]["b"].float(), torch.arange(4.0) * 1.75)
    table = M.candidate_table([0, 10, 20], 100, [0.15], ["mean"], ["wsm", "qam"])
    assert [sorted(c.weights) for c in table] == [[1, 2], [1, 2]]


def test_ckpt_tools_info_block_norms_and_resume_cmd(tmp_path):
    """ckpt_tools.py (the reference's tests/block_norms.py and tests/resume_cmd.py): block norms relative to the old
    blocks, raw and EMA; a continuation command that keeps the stored settings, lets `--` flags replace them and
    runs (here one step on CPU) from a copy of the checkpoint."""
    import importlib.util
    import shlex
    import shutil

    spec = importlib.util.spec_from_file_location("_repo_ckpt_tools", os.path.join(ROOT, "ckpt_tools.py"))
    T = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(T)
    run = str(tmp_path / "run")
    _py("train.py", "--synthetic", "32", "--out", run, "--size", "nano", "--te-size", "13m", "--batch", "2",
        "--micro-batch", "2", "--steps", "2", "--eval-every", "0", "--no-wandb", "--wd", "0.05")
    latest = os.path.join(run, "latest.pt")
    ck = torch.load(latest, weights_only=False)
    res = T.main(["info", latest])
    assert res["step"] == 2 and res["ema"] and res["den_params"] > 0 and res["extra"] == {}
    norms, depth = T.block_norms(ck, 2)
    assert set(norms) == {"raw", "EMA"} and depth == 4
    raw = dict(norms["raw"])
    want = ck["den"]["blocks.3.mlp.out_proj.weight"].float().pow(2).mean().sqrt().item()
    assert abs(raw[3]["mlp.out_proj.weight"][0] - want) < 1e-7
    mean_old = sum(raw[i]["attn.out.weight"][0] for i in range(2)) / 2
    assert abs(raw[0]["attn.out.weight"][1] - raw[0]["attn.out.weight"][0] / mean_old) < 1e-6
    cont = str(tmp_path / "cont")
    cmd = T.main(["resume-cmd", latest, "--out", cont, "--extra-steps", "1", "--nproc", "1", "--", "--wd", "0.1"])
    args = shlex.split(cmd)
    assert args[:6] == ["torchrun", "--nproc-per-node", "1", "--master-addr", "127.0.0.1", "train.py"]
    assert "--size" in args and args[args.index("--size") + 1] == "nano"
    assert args.count("--wd") == 1 and args[args.index("--wd") + 1] == "0.1"  # the `--` flag replaces the stored one
    assert args[args.index("--steps") + 1] == "3" and args[args.index("--out") + 1] == cont
    os.makedirs(cont)
    shutil.copy(latest, os.path.join(cont, "latest.pt"))
    _py(*args[5:])  # the same flags through the plain interpreter (one process)
    assert torch.load(os.path.join(cont, "latest.pt"), weights_only=False)["step"] == 3


def test_bench_gpus_flag_launches_ranks(monkeypatch):
    """bench.py --gpus N run directly re-runs itself under torch.distributed.run with N ranks; under a launcher the
    world size must agree with --gpus."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_repo_bench", os.path.join(ROOT, "bench.py"))
    B = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(B)
    args = B.parse.__globals__["argparse"].Namespace(gpus=4)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    cmd = B.launch_ranks(args, ["--gpus", "4", "--steps", "2"])
    assert cmd[1:4] == ["-m", "torch.distributed.run", "--nnodes"] and cmd[cmd.index("--nproc-per-node") + 1] == "4"
    assert cmd[-4:] == [os.path.join(ROOT, "bench.py"), "--gpus", "4", "--steps", "2"][-4:]
    assert "127.0.0.1" in cmd
    monkeypatch.setenv("WORLD_SIZE", "4")
    assert B.launch_ranks(args, []) is None
    monkeypatch.setenv("WORLD_SIZE", "2")
    with pytest.raises(SystemExit):
        B.launch_ranks(args, [])
