"""OPD service roles over Gloo on CPU (learner, rollout actor, teacher): the snapshot reaches the actor, the
actor's rollouts equal the learner's own, the remote teacher's targets equal a local teacher's, and a job that
needs a newer snapshot than the actor holds is refused (host-side failure, no device involved)."""
import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig, build_models

DEN = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16, latent_size=4)
TE = LMEncoderConfig(lm_dim=32, dim=64, depth=1, heads=1, kv_heads=1, head_dim=64, mlp_hidden=128, max_tokens=8,
                     backend="states")
KW = dict(K=4, m=2, method="dance", beta=(5.0, 2.0), shift=2.0, mb=2, seed=0)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _models(seed):
    torch.manual_seed(seed)
    te, den = build_models(DEN, TE)
    with torch.no_grad():
        for p in den.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return te, den


def _worker(rank, world, port, d):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctl = dist.new_group(backend="gloo")
    from trenowanie_generatora_obrazkow_b200.parallel.roles import (ActorClient, RoleLayout, RolloutActor,
                                                                    SnapshotSender, TeacherClient, TeacherServer)
    from trenowanie_generatora_obrazkow_b200.train.opd import DiTTeacher
    lay = RoleLayout(world, 1, 1, 1)
    role = lay.role(rank)
    if role == "teacher":
        tte, tden = _models(2)
        TeacherServer(DiTTeacher(tte, tden, 3.0), "cpu", ctl).serve()
    elif role == "actor":
        te, den = _models(99)  # wrong weights until the snapshot arrives
        params = list(te.parameters()) + list(den.parameters())
        try:
            RolloutActor(te, den, params, "cpu", ctl, KW).serve()
        except RuntimeError as e:
            torch.save(str(e), os.path.join(d, "actor_error.pt"))
    else:
        te, den = _models(1)
        params = list(te.parameters()) + list(den.parameters())
        client = ActorClient(lay.actors[0], ctl, KW["m"])
        teacher = TeacherClient(lay.teachers, ctl, rank)
        v = SnapshotSender(params, lay.actors, ctl).send()
        g = torch.Generator().manual_seed(3)
        noise, st = torch.randn(2, 16, 4, 4, generator=g), torch.randn(2, 8, 32, generator=g)
        valid = torch.ones(2, 8, dtype=torch.bool)
        states, t = client.rollouts(noise, st, valid, step=5, version=v)
        tgt = teacher.velocity(states, t, dict(lm_states=st.repeat_interleave(2, 0),
                                               valid=valid.repeat_interleave(2, 0)))
        torch.save(dict(states=states, t=t, tgt=tgt, noise=noise, st=st), os.path.join(d, "learner.pt"))
        teacher.stop()
        client.rollouts(noise, st, valid, step=6, version=v + 1)  # needs a snapshot the actor does not have
    dist.destroy_process_group()


def test_opd_roles_round_trip():
    with tempfile.TemporaryDirectory() as d:
        try:
            mp.spawn(_worker, args=(3, _port(), d), nprocs=3, join=True)
        except Exception:
            pass  # the learner's last job is refused on purpose; its recv then fails
        res = torch.load(os.path.join(d, "learner.pt"))
        err = torch.load(os.path.join(d, "actor_error.pt"))
    assert "needs" in err
    from trenowanie_generatora_obrazkow_b200.ops.reference import valid_to_len
    from trenowanie_generatora_obrazkow_b200.train.opd import DiTTeacher, dance_picks, opd_grid, rollout
    te, den = _models(1)
    valid = torch.ones(2, 8, dtype=torch.bool)
    g = torch.Generator().manual_seed(0 * 1_000_003 + 0 * 1009 + 5 + 7)
    picks = dance_picks(2, 2, 4, (5.0, 2.0), 0, 0, 5)
    ts = opd_grid(4, 2.0, torch.rand((), generator=g).item())
    text, v = te(lm_states=res["st"], valid=valid)
    states = rollout(den, text, valid_to_len(v), res["noise"], ts, picks, 2).flatten(0, 1)
    assert torch.allclose(states, res["states"], atol=1e-5)
    tte, tden = _models(2)
    tgt = DiTTeacher(tte, tden, 3.0).velocity(states, res["t"], dict(lm_states=res["st"].repeat_interleave(2, 0),
                                                                      valid=valid.repeat_interleave(2, 0)))
    assert torch.allclose(tgt, res["tgt"], atol=1e-5)


def _deferred_worker(rank, world, port, d):
    """Ranks 0, 1 learners, rank 2 the teacher. Both learners leave a deferred request with the teacher, run a
    gradient-style all-reduce among themselves, then collect; a plain request follows."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctl = dist.new_group(backend="gloo")
    learners = dist.new_group([0, 1])
    from trenowanie_generatora_obrazkow_b200.parallel.roles import TeacherClient, TeacherServer
    from trenowanie_generatora_obrazkow_b200.train.opd import DiTTeacher
    if rank == 2:
        tte, tden = _models(2)
        served = TeacherServer(DiTTeacher(tte, tden, 3.0), "cpu", ctl).serve()
        torch.save(served, os.path.join(d, "served.pt"))
    else:
        teacher = TeacherClient([2], ctl, rank)
        g = torch.Generator().manual_seed(10 + rank)
        x, t = torch.randn(3, 16, 4, 4, generator=g), torch.rand(3, generator=g)
        kw = dict(lm_states=torch.randn(3, 8, 32, generator=g), valid=torch.ones(3, 8, dtype=torch.bool))
        h = teacher.request(x, t, kw, chunks=2, deferred=True)
        s = torch.ones(4)
        dist.all_reduce(s, group=learners)  # the learners meet while both replies are held
        deferred = teacher.collect(h)
        plain = teacher.velocity(x, t, kw)
        torch.save(dict(x=x, t=t, kw=kw, deferred=deferred, plain=plain, s=s), os.path.join(d, f"l{rank}.pt"))
        dist.barrier(group=learners)
        if rank == 0:
            teacher.stop()
    dist.destroy_process_group()


def test_deferred_teacher_requests_from_two_learners():
    from trenowanie_generatora_obrazkow_b200.train.opd import DiTTeacher
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_deferred_worker, args=(3, _port(), d), nprocs=3, join=True)
        tte, tden = _models(2)
        local = DiTTeacher(tte, tden, 3.0)
        for r in range(2):
            got = torch.load(os.path.join(d, f"l{r}.pt"))
            want = local.velocity(got["x"], got["t"], got["kw"])
            assert torch.allclose(got["deferred"], want, atol=1e-5) and torch.allclose(got["plain"], want, atol=1e-5)
            assert torch.equal(got["s"], torch.full((4,), 2.0))
        assert torch.load(os.path.join(d, "served.pt")) == 4


def _deferred_actor_worker(rank, world, port, d):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctl = dist.new_group(backend="gloo")
    from trenowanie_generatora_obrazkow_b200.parallel.roles import (ActorClient, RoleLayout, RolloutActor,
                                                                    SnapshotSender)
    lay = RoleLayout(world, 1, 1, 0)
    if lay.role(rank) == "actor":
        te, den = _models(99)
        jobs = RolloutActor(te, den, list(te.parameters()) + list(den.parameters()), "cpu", ctl, KW).serve()
        torch.save(jobs, os.path.join(d, "jobs.pt"))
    else:
        te, den = _models(1)
        client = ActorClient(lay.actors[0], ctl, KW["m"])
        v = SnapshotSender(list(te.parameters()) + list(den.parameters()), lay.actors, ctl).send()
        g = torch.Generator().manual_seed(4)
        noise, st = torch.randn(2, 16, 4, 4, generator=g), torch.randn(2, 8, 32, generator=g)
        valid = torch.ones(2, 8, dtype=torch.bool)
        job = client.request(noise, st, valid, 5, v, deferred=True)  # held by the actor ...
        plain = client.rollouts(noise, st, valid, 5, v)  # ... while a plain job of the same batch goes through
        held = client.collect(job)
        shifted = client.rollouts(noise, st, valid, 5, v, shift=3.0)  # the batch resolution's shift
        torch.save(dict(plain=plain, held=held, shifted=shifted), os.path.join(d, "out.pt"))
        client.stop()
    dist.destroy_process_group()


def test_deferred_actor_job_equals_a_plain_one():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_deferred_actor_worker, args=(2, _port(), d), nprocs=2, join=True)
        out = torch.load(os.path.join(d, "out.pt"))
        assert torch.equal(out["plain"][0], out["held"][0]) and torch.equal(out["plain"][1], out["held"][1])
        from trenowanie_generatora_obrazkow_b200.train.opd import dance_picks, opd_grid
        g = torch.Generator().manual_seed(KW["seed"] * 1_000_003 + 0 * 1009 + 5 + 7)
        picks = dance_picks(2, KW["m"], KW["K"], KW["beta"], KW["seed"], 0, 5)
        want = opd_grid(KW["K"], 3.0, torch.rand((), generator=g).item())[picks].flatten()
        assert torch.allclose(out["shifted"][1], want) and not torch.allclose(out["shifted"][1], out["plain"][1])
        assert torch.load(os.path.join(d, "jobs.pt")) == 3
