"""Fréchet distance (train/fid.py) against the textbook sqrtm formula, the round-robin gather on Gloo ranks, and
fid_eval.py end to end on CPU with the latent stand-in features."""
import os
import socket
import subprocess
import sys
import tempfile

import numpy as np
import scipy.linalg
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.train.fid import feature_stats, frechet_distance

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_frechet_matches_sqrtm_formula():
    g = torch.Generator().manual_seed(0)
    a = torch.randn(400, 24, generator=g, dtype=torch.float64)
    b = torch.randn(300, 24, generator=g, dtype=torch.float64) @ torch.randn(24, 24, generator=g, dtype=torch.float64) * 0.5 + 0.3
    m1, s1 = feature_stats(a)
    m2, s2 = feature_stats(b)
    covmean = scipy.linalg.sqrtm(s1.numpy() @ s2.numpy()).real
    want = float(((m1 - m2) ** 2).sum() + np.trace(s1.numpy()) + np.trace(s2.numpy()) - 2 * np.trace(covmean))
    got = frechet_distance(m1, s1, m2, s2)
    assert abs(got - want) < 1e-6 * max(1.0, abs(want))
    assert abs(frechet_distance(m1, s1, m1, s1)) < 1e-8
    assert np.allclose(s1.numpy(), np.cov(a.numpy().T))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trenowanie_generatora_obrazkow_b200.train.fid import gather_in_order, my_prompts
    n = 11
    local = torch.tensor([[float(i), -float(i)] for i in my_prompts(n, rank, world)])
    torch.save(gather_in_order(local, n), os.path.join(out, f"g{rank}.pt"))
    dist.destroy_process_group()


def test_gather_in_prompt_order():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_gather_worker, args=(3, _port(), d), nprocs=3, join=True)
        for r in range(3):
            g = torch.load(os.path.join(d, f"g{r}.pt"))
            assert torch.equal(g[:, 0], torch.arange(11.0))


def test_fid_eval_cli_latent_features(tmp_path):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    data = str(tmp_path / "data")
    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    write_synthetic_shards(data, n_shards=2, per_shard=8, side=16)
    run = str(tmp_path / "run")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "train.py"), "--data", data, "--out", run, "--size", "50m",
                        "--te-size", "13m", "--batch", "2", "--micro-batch", "2", "--steps", "2", "--eval-every", "0",
                        "--no-wandb"], cwd=ROOT, capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = str(tmp_path / "fd.jsonl")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "fid_eval.py"), os.path.join(run, "latest.pt"), "--data",
                        data, "--features", "latent", "--samples", "6", "--steps", "2", "--out", out], cwd=ROOT,
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    import json
    res = json.loads(open(out).read().splitlines()[0])
    assert res["samples"] == 6 and np.isfinite(res["fd"])


def test_fid_eval_cli_frozen_lm_encoder_and_lang(tmp_path):
    """fid_eval.py with a frozen-LM refiner: prompts through the LM's states (random stand-in LM), --lang reads the
    translated token rows of the same held-out images."""
    import json
    import shutil
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    data = str(tmp_path / "data")
    from trenowanie_generatora_obrazkow_b200.data.shards import write_synthetic_shards
    names = write_synthetic_shards(data, n_shards=2, per_shard=8, side=16, lm_suffix="slayer149")
    for n in names:
        shutil.copy(os.path.join(data, f"{n}.tok_slayer149.npy"), os.path.join(data, f"{n}.tok_slayer149_pl.npy"))
    run = str(tmp_path / "run")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "train.py"), "--data", data, "--out", run, "--size", "nano",
                        "--te-size", "slayer149", "--random-lm", "--batch", "2", "--micro-batch", "2", "--steps", "1",
                        "--eval-every", "0", "--no-wandb", "--workers", "0"], cwd=ROOT, capture_output=True, text=True,
                       env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = str(tmp_path / "fd.jsonl")
    for lang in ("", "pl"):
        r = subprocess.run([sys.executable, os.path.join(ROOT, "fid_eval.py"), os.path.join(run, "latest.pt"), "--data",
                            data, "--features", "latent", "--samples", "4", "--steps", "2", "--random-lm", "--lang",
                            lang, "--out", out], cwd=ROOT, capture_output=True, text=True, env=env, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
    res = [json.loads(line) for line in open(out).read().splitlines()]
    assert len(res) == 2 and all(np.isfinite(x["fd"]) for x in res)
    assert abs(res[0]["fd"] - res[1]["fd"]) < 1e-6  # identical rows under both names: the same distance
