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
    assert "step 3/3" in out and "served" in out and "rollout jobs" in out


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
