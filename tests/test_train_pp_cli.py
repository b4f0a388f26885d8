"""train_pp.py on CPU ranks (Gloo): the 1F1B flow-matching mode and the OPD mode with an actor and a teacher rank."""
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _torchrun(n, *args):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(n),
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(ROOT, "train_pp.py"), *args]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES="", DIST_BACKEND="gloo"))
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout


def test_pipeline_mode(tmp_path):
    out = _torchrun(2, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--pp", "2",
                    "--microbatches", "4", "--micro-batch", "2", "--res", "128", "--steps", "3", "--log-every", "3")
    assert "step 3/3" in out


def test_opd_mode_with_actor_and_teacher(tmp_path):
    out = _torchrun(4, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--dance-opd",
                    "--opd-actor", "--teacher-ranks", "1", "--teacher-size", "nano", "--res", "128",
                    "--batch", "8", "--micro-batch", "2", "--steps", "3", "--log-every", "1", "--opd-reuse", "2",
                    "--opd-rollout-steps", "4")
    # two learners, reuse 2: fresh batches at steps 0 (rolled out while the learners wait) and 2 (requested at
    # step 0 and rolled out during the cycle; its teacher request goes out at step 1, the last replay step)
    assert "step 3/3" in out and "[actor 2] 4 rollout jobs" in out and "[teacher 3] served 4 requests" in out


def test_pipeline_with_distributed_lm_states(tmp_path):
    """Caption ids through a frozen LM: per-stage LM work gathered to stage 0, then the LM layer split."""
    for extra in ([], ["--lm-split"]):
        out = _torchrun(2, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--pp", "2",
                        "--microbatches", "4", "--micro-batch", "2", "--res", "128", "--steps", "2", "--log-every",
                        "2", "--random-lm", "--lm-layers", "2", *extra)
        assert "step 2/2" in out


def test_pipeline_with_lm_and_vae_servers(tmp_path):
    """Two learners (pp 2) + an LM server rank + a VAE server rank; the LM server reports what it served."""
    out = _torchrun(4, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--pp", "2",
                    "--microbatches", "2", "--micro-batch", "2", "--res", "128", "--steps", "2", "--log-every", "2",
                    "--random-lm", "--lm-layers", "2", "--lm-rank", "1", "--vae-rank", "1")
    assert "step 2/2" in out and "[lm server 2] served 8 captions" in out and "[vae server 3]" in out


def test_opd_with_lm_server_text_lookahead(tmp_path):
    out = _torchrun(3, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--dance-opd",
                    "--res", "128", "--batch", "4", "--micro-batch", "2", "--steps", "3", "--log-every", "1",
                    "--opd-rollout-steps", "2", "--teacher-size", "nano", "--random-lm", "--lm-layers", "2",
                    "--lm-rank", "1", "--opd-text-ahead", "2")
    assert "step 3/3" in out and "[lm server 2] served" in out


def _torchrun_rc(n, *args):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(n),
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(ROOT, "train_pp.py"), *args]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES="", DIST_BACKEND="gloo"))
    return r.returncode, r.stdout + r.stderr


def test_pipeline_shards_checkpoint_and_resume(tmp_path):
    """--data shards (latents + caption rows through a frozen LM), latest.pt in the single-model layout (loads into
    the unsplit modules), per-rank optimizer files, resume at the same pipeline layout and, only with
    --resume-opt-mismatch, at another one."""
    import torch

    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, build_models
    from trenowanie_generatora_obrazkow_b200.models.config import te_config_from_dict
    from trenowanie_generatora_obrazkow_b200.utils.checkpoint import load_weights
    import glob
    data = str(tmp_path / "shards")
    write_synthetic_shards(data, n_shards=3, per_shard=8, side=8)
    import shutil
    for f in glob.glob(os.path.join(data, "*.lat.npy")):  # 8 x 8 latents serve as the 128 px grids (.lat128.npy)
        shutil.copy(f, f[: -len(".lat.npy")] + ".lat128.npy")
    out = str(tmp_path / "run")
    common = ["--out", out, "--data", data, "--fraction", "1", "--size", "nano", "--te-size", "states-nano",
              "--microbatches", "2", "--micro-batch", "2", "--res", "128", "--log-every", "1", "--random-lm",
              "--lm-layers", "2", "--ckpt-every", "2", "--workers", "0", "--keep-ckpt-steps", "2"]
    log = _torchrun(2, *common, "--pp", "2", "--steps", "2")
    assert "step 2/2" in log and "data: latents from" in log
    ck = torch.load(os.path.join(out, "latest.pt"), weights_only=False)
    assert ck["step"] == 2 and ck["samples"] == 8 and len(ck["ema"]) == len(ck["te"]) + len(ck["den"])
    te, den = build_models(DenoiserConfig(**ck["den_config"]), te_config_from_dict(ck["te_config"]))
    load_weights(ck, te, den)  # strict: every parameter of the unsplit model, under its own name
    assert all(os.path.exists(os.path.join(out, f)) for f in ("opt_stage0_rep0.pt", "opt_stage1_rep0.pt",
                                                              "step_0000002.pt"))
    log = _torchrun(2, *common, "--pp", "2", "--steps", "4")
    assert "resumed" in log and "step 4/4" in log
    rc, msg = _torchrun_rc(1, *common, "--pp", "1", "--steps", "5")
    assert rc != 0 and "resume-opt-mismatch" in msg
    log = _torchrun(1, *common, "--pp", "1", "--steps", "5", "--resume-opt-mismatch")
    assert "fresh" in log and "step 5/5" in log


def test_pipeline_flags_stage0_lm_profile_and_unsupported(tmp_path):
    """--lm-stage0, --te-checkpoint, --bench, --mem-debug and the profiler window; flags the pipeline trainer does
    not run stop it with a pointer to train.py."""
    prof = str(tmp_path / "prof")
    log = _torchrun(2, "--out", str(tmp_path / "a"), "--size", "nano", "--te-size", "states-nano", "--pp", "2",
                    "--microbatches", "2", "--micro-batch", "2", "--res", "128", "--steps", "3", "--log-every", "3",
                    "--random-lm", "--lm-layers", "2", "--lm-stage0", "--te-checkpoint", "--bench", "--mem-debug",
                    "--profile-dir", prof, "--profile-start", "1", "--profile-steps", "1", "--synthetic", "64")
    assert "step 3/3" in log and "[bench]" in log and "memory:" in log
    assert os.path.exists(os.path.join(prof, "kernels_rank0.json"))
    rc, msg = _torchrun_rc(1, "--out", str(tmp_path / "b"), "--size", "nano", "--te-size", "states-nano",
                           "--steps", "1", "--diloco", "4")
    assert rc != 0 and "use train.py" in msg
    rc, msg = _torchrun_rc(1, "--out", str(tmp_path / "c"), "--size", "nano", "--te-size", "states-nano",
                           "--steps", "1", "--klein")
    assert rc != 0 and "unavailable on this box" in msg


def test_pipeline_packed_images_local_encode(tmp_path):
    """--img-dir: packed JPEG shards decoded by the loader and encoded on stage 0 (the VAE stand-in here)."""
    import io

    import numpy as np
    import pytest
    PIL = pytest.importorskip("PIL.Image")
    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    data = str(tmp_path / "imgs")
    names = write_synthetic_shards(data, n_shards=3, per_shard=6, side=8)
    rng = np.random.default_rng(0)
    for name in names:
        blobs = []
        for _ in range(6):
            buf = io.BytesIO()
            PIL.fromarray(rng.integers(0, 256, (128, 128, 3), dtype=np.uint8)).save(buf, format="JPEG")
            blobs.append(buf.getvalue())
        with open(os.path.join(data, f"{name}.img.bin"), "wb") as f:
            f.write(b"".join(blobs))
        np.save(os.path.join(data, f"{name}.img.off.npy"), np.cumsum([0] + [len(b) for b in blobs]).astype(np.int64))
    log = _torchrun(2, "--out", str(tmp_path / "run"), "--img-dir", data, "--fraction", "1", "--size", "nano",
                    "--te-size", "states-nano", "--pp", "2", "--microbatches", "2", "--micro-batch", "2", "--res",
                    "128", "--steps", "2", "--log-every", "2", "--random-lm", "--lm-layers", "2", "--workers", "0",
                    "--enc-chunk", "2", "--eval-every", "2", "--val-samples", "4")
    assert "step 2/2" in log and "data: images from" in log and "[eval] step 2 | EMA val/loss=" in log
    cache = os.listdir(tmp_path / "run" / "val_cache")  # the held-out images encoded once, then read from here
    assert len(cache) == 1 and cache[0].startswith("val_") and cache[0].endswith(".pt")


def test_opd_prefetch_with_a_teacher_rank(tmp_path):
    """--opd-prefetch: the next cycle's rollouts are made after the first update of a cache and the teacher's reply
    (computed in --opd-parts chunks on the teacher rank) is collected when that cycle starts; with reuse 2 over 5
    steps the fresh batches start at steps 0, 2 and 4: step 0 as two --opd-parts requests, steps 2 and 4 prefetched
    as one chunked request each, so the teacher serves 4 requests."""
    out = _torchrun(2, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--dance-opd",
                    "--teacher-ranks", "1", "--teacher-size", "nano", "--res", "128", "--batch", "4",
                    "--micro-batch", "2", "--steps", "5", "--log-every", "1", "--opd-reuse", "2",
                    "--opd-rollout-steps", "4", "--opd-prefetch", "--opd-parts", "2", "--opd-learner-profile")
    assert "step 5/5" in out and "[teacher 1] served 4 requests" in out and "prefetch" in out


def test_opd_init_checkpoint_and_resume(tmp_path):
    """OPD learners: the student starts from a flow-matching checkpoint (--init, one block grown), checkpoints
    carry the EMA and per-learner optimizer files, and a rerun resumes from latest.pt (with a fresh batch first)."""
    import torch
    fm = str(tmp_path / "fm")
    _torchrun(1, "--out", fm, "--size", "nano", "--te-size", "states-nano", "--res", "128", "--batch", "2",
              "--micro-batch", "2", "--steps", "1", "--log-every", "1", "--ckpt-every", "1")
    opd = str(tmp_path / "opd")
    common = ["--out", opd, "--size", "nano", "--depth", "5", "--te-size", "states-nano", "--dance-opd",
              "--teacher-size", "nano", "--res", "128", "--batch", "4", "--micro-batch", "2", "--log-every", "1",
              "--opd-reuse", "2", "--opd-rollout-steps", "2", "--ckpt-every", "2"]
    out = _torchrun(2, *common, "--steps", "3", "--init", os.path.join(fm, "latest.pt"), "--eval-every", "3",
                    "--val-samples", "4")
    assert "step 3/3" in out and "blocks 4-4 grown as identity blocks" in out and "[eval] step 3 | EMA val/loss=" in out
    ck = torch.load(os.path.join(opd, "latest.pt"), weights_only=False)
    assert ck["step"] == 3 and ck["ema"] and ck["den_config"]["depth"] == 5 and "opd_caption_micro" in ck["extra"]
    assert sorted(f for f in os.listdir(opd) if f.startswith("opt_")) == ["opt_stage0_rep0.pt", "opt_stage0_rep1.pt"]
    out = _torchrun(2, *common, "--steps", "5")
    assert "resumed from" in out and "at step 3" in out and "step 5/5" in out and "step 1/5" not in out
    assert torch.load(os.path.join(opd, "latest.pt"), weights_only=False)["step"] == 5


def test_opd_caption_position_survives_a_resume(tmp_path):
    """OPD on shard captions: the checkpoint records how many caption micro-batches the trained fresh batches
    used (2 fresh batches of 4 captions in micro-batches of 2 = 4), and a resume continues the caption stream."""
    import torch

    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    data = str(tmp_path / "shards")
    write_synthetic_shards(data, n_shards=2, per_shard=8, side=8)
    out = str(tmp_path / "opd")
    common = ["--out", out, "--data", data, "--fraction", "1", "--size", "nano", "--te-size", "states-nano",
              "--dance-opd", "--teacher-size", "nano", "--res", "128", "--batch", "4", "--micro-batch", "2",
              "--log-every", "1", "--opd-reuse", "2", "--opd-rollout-steps", "2", "--random-lm", "--lm-layers", "1",
              "--ckpt-every", "3", "--workers", "0"]
    _torchrun(1, *common, "--steps", "3")
    assert torch.load(os.path.join(out, "latest.pt"), weights_only=False)["extra"]["opd_caption_micro"] == 4
    _torchrun(1, *common, "--steps", "4")  # one more fresh batch from the resumed stream
    assert torch.load(os.path.join(out, "latest.pt"), weights_only=False)["extra"]["opd_caption_micro"] == 6


def test_pipeline_ema_eval_and_merge_checkpoints(tmp_path):
    """--eval-every: validation loss of the EMA weights on the unsplit model rebuilt on rank 0; --merge-every: raw
    weights as merge/step_<n>.pt in train.py's layout, gathered from both stages."""
    import torch
    out = _torchrun(2, "--out", str(tmp_path), "--size", "nano", "--te-size", "states-nano", "--pp", "2",
                    "--microbatches", "2", "--micro-batch", "2", "--res", "128", "--steps", "2", "--log-every", "2",
                    "--eval-every", "2", "--val-samples", "8", "--merge-every", "1", "--merge-start", "0")
    assert "[eval] step 2 | EMA val/loss=" in out
    merged = sorted(os.listdir(tmp_path / "merge"))
    assert merged == ["step_0000001.pt", "step_0000002.pt"]
    ck = torch.load(tmp_path / "merge" / merged[-1], weights_only=False)
    assert ck["step"] == 2 and ck["total_steps"] == 2 and "blocks.3.mlp.out_proj.weight" in ck["den"] and ck["te"]
    import json
    rows = [json.loads(line) for line in open(tmp_path / "log.jsonl")]  # written by the last stage's rank
    assert any("train/loss" in r and r["step"] == 2 for r in rows)
