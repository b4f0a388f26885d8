"""Failure detection and recovery on the host (no GPU is faulted, trapped or hung): a checkpoint write that fails
(full disk) keeps the previous file, a truncated checkpoint names the ones that remain, a two-phase commit across
Gloo ranks aborts on every rank when one rank's write fails, an interrupted commit is finished or undone before a
resume, a pipeline resume refuses optimizer state of another step, and a rank that never joins a collective ends
its peer's collective with an error after the process-group timeout."""
import errno
import os
import socket
import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.utils import checkpoint as ckpt


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _full_disk_save(limit=64):
    """A torch.save that writes ``limit`` bytes and then fails as a full disk does."""
    def save(obj, path):
        with open(path, "wb") as f:
            f.write(b"\0" * limit)
        raise OSError(errno.ENOSPC, "No space left on device", path)
    return save


def test_atomic_save_keeps_the_previous_file_on_a_full_disk(tmp_path, monkeypatch):
    path = str(tmp_path / "latest.pt")
    ckpt.atomic_save({"step": 1}, path)
    monkeypatch.setattr(ckpt.torch, "save", _full_disk_save())
    with pytest.raises(OSError) as e:
        ckpt.atomic_save({"step": 2}, path)
    assert e.value.errno == errno.ENOSPC
    monkeypatch.undo()
    assert ckpt.load(path)["step"] == 1 and not os.path.exists(path + ".tmp")


def test_truncated_checkpoint_raises_a_clear_error(tmp_path):
    good = str(tmp_path / "snap_0000100.pt")
    ckpt.atomic_save({"step": 100, "w": torch.randn(1000)}, good)
    data = open(good, "rb").read()
    bad = str(tmp_path / "latest.pt")
    with open(bad, "wb") as f:
        f.write(data[: len(data) // 2])
    with pytest.raises(ckpt.CheckpointError, match="snap_0000100.pt"):
        ckpt.load(bad)
    assert ckpt.step_of(bad) is None and ckpt.step_of(good) == 100
    with pytest.raises(FileNotFoundError):
        ckpt.load(str(tmp_path / "missing.pt"))


def _commit_worker(rank, world, port, out, fail_rank, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    path = os.path.join(out, f"opt_stage{rank}_rep0.pt")
    writes = [({"step": 1, "rank": rank}, path)]
    ckpt.two_phase_commit(writes, agree=ckpt.agree_all())  # a first, successful commit
    writes = [({"step": 2, "rank": rank}, path)]
    if rank == fail_rank:
        ckpt.torch.save = _full_disk_save()
    outcome = "committed"
    try:
        ckpt.two_phase_commit(writes, agree=ckpt.agree_all())
    except ckpt.CheckpointError:
        outcome = "aborted by a peer"
    except OSError as e:
        outcome = f"own error {e.errno}"
    with open(os.path.join(result_dir, f"r{rank}.txt"), "w") as f:
        f.write(outcome)
    dist.barrier()
    dist.destroy_process_group()


def test_two_phase_commit_aborts_on_every_rank_when_one_write_fails():
    with tempfile.TemporaryDirectory() as out, tempfile.TemporaryDirectory() as res:
        mp.spawn(_commit_worker, args=(2, _free_port(), out, 1, res), nprocs=2, join=True)
        got = [open(os.path.join(res, f"r{r}.txt")).read() for r in range(2)]
        assert got == ["aborted by a peer", f"own error {errno.ENOSPC}"]
        assert sorted(os.listdir(out)) == ["opt_stage0_rep0.pt", "opt_stage1_rep0.pt"]  # no temporaries left
        assert [ckpt.load(os.path.join(out, f"opt_stage{r}_rep0.pt"))["step"] for r in range(2)] == [1, 1]


def _write_set(out, latest=None, opts=(), tmp_latest=None, tmp_opts=(), truncated=()):
    if latest is not None:
        torch.save({"step": latest}, os.path.join(out, "latest.pt"))
    if tmp_latest is not None:
        torch.save({"step": tmp_latest}, os.path.join(out, "latest.pt.tmp"))
    for r, s in opts:
        torch.save({"step": s}, os.path.join(out, f"opt_stage{r}_rep0.pt"))
    for r, s in tmp_opts:
        torch.save({"step": s}, os.path.join(out, f"opt_stage{r}_rep0.pt.tmp"))
    for name in truncated:
        p = os.path.join(out, name)
        data = open(p, "rb").read()
        open(p, "wb").write(data[:10])


def _steps(out):
    return {f: ckpt.step_of(os.path.join(out, f)) for f in sorted(os.listdir(out))}


def test_recover_commit_rolls_forward_after_phase_two_began(tmp_path):
    """latest.pt and stage 0's file were renamed (step 2), stage 1's temporary was not: finished."""
    out = str(tmp_path)
    _write_set(out, latest=2, opts=[(0, 2), (1, 1)], tmp_opts=[(1, 2)])
    assert ckpt.recover_commit(out, log=lambda *a: None) == ("forward", 2)
    assert _steps(out) == {"latest.pt": 2, "opt_stage0_rep0.pt": 2, "opt_stage1_rep0.pt": 2}


def test_recover_commit_rolls_back_when_phase_one_was_cut(tmp_path):
    """A crash while writing: one temporary is truncated, nothing was renamed; the step-1 checkpoint stays."""
    out = str(tmp_path)
    _write_set(out, latest=1, opts=[(0, 1), (1, 1)], tmp_latest=2, tmp_opts=[(0, 2)], truncated=["latest.pt.tmp"])
    (tmp_path / "snap_0000002.pt.tmp").write_bytes(b"partial")
    assert ckpt.recover_commit(out, log=lambda *a: None) == ("back", 2)
    assert _steps(out) == {"latest.pt": 1, "opt_stage0_rep0.pt": 1, "opt_stage1_rep0.pt": 1}
    assert ckpt.recover_commit(out, log=lambda *a: None) == ("clean", None)


def test_recover_commit_rolls_back_before_any_rename(tmp_path):
    """Every temporary complete but the crash came before the first rename: nothing was committed."""
    out = str(tmp_path)
    _write_set(out, latest=1, opts=[(0, 1)], tmp_latest=2, tmp_opts=[(0, 2)])
    assert ckpt.recover_commit(out, log=lambda *a: None)[0] == "back"
    assert _steps(out) == {"latest.pt": 1, "opt_stage0_rep0.pt": 1}


def test_pipeline_resume_refuses_optimizer_state_of_another_step(tmp_path):
    """pp_checkpoint.resume: an optimizer file of another step than latest.pt (a commit interrupted in a way the
    recovery could not repair, or files copied by hand) stops the resume unless fresh optimizer state is asked for."""
    from types import SimpleNamespace

    from trenowanie_generatora_obrazkow_b200.models import build_models
    from trenowanie_generatora_obrazkow_b200.models.config import make_configs
    from trenowanie_generatora_obrazkow_b200.train import pp_checkpoint as P
    den_cfg, te_cfg = make_configs("nano", "13m")
    te, den = build_models(den_cfg, te_cfg)
    named = [("te", n, p) for n, p in te.named_parameters()] + [("den", n, p) for n, p in den.named_parameters()]
    opt = torch.optim.SGD([p for _, _, p in named], lr=0.1, momentum=0.9)
    tr = SimpleNamespace(den_cfg=den_cfg, te_cfg=te_cfg, named=named, ema=None, opts=[opt], pp=1, dp=1, stage=0,
                         te_cost=0.0, replica=0)
    out = str(tmp_path)
    ckpt.save_latest(os.path.join(out, "latest.pt"), 5, 40, den_cfg, te_cfg, te, den, None, None)
    torch.save(dict(layout=P.layout(tr), step=4, opts=[opt.state_dict()]), P.opt_path(out, tr))
    with pytest.raises(RuntimeError, match="another step"):
        P.resume(tr, out)
    assert P.resume(tr, out, resume_opt_mismatch=True, log=lambda *a: None) == (5, 40)
    torch.save(dict(layout=P.layout(tr), step=5, opts=[opt.state_dict()]), P.opt_path(out, tr))
    assert P.resume(tr, out) == (5, 40)


def _silent_peer_worker(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    outcome = "joined"
    if rank == 0:
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
            outcome = "completed"
        except RuntimeError:
            outcome = f"error after {time.time() - t0:.0f} s"
    else:
        time.sleep(8)  # never joins the collective (a stuck or lost rank)
    with open(os.path.join(result_dir, f"r{rank}.txt"), "w") as f:
        f.write(outcome)


def test_rank_that_never_joins_ends_the_peers_collective_with_an_error():
    """The process-group timeout (train_pp.py --dist-timeout) turns a lost rank into an error on the others."""
    with tempfile.TemporaryDirectory() as res:
        mp.spawn(_silent_peer_worker, args=(2, _free_port(), res), nprocs=2, join=True)
        r0 = open(os.path.join(res, "r0.txt")).read()
        assert r0.startswith("error after") and int(r0.split()[2]) < 8, r0
