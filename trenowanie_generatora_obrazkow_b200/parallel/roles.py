"""MPMD service roles for on-policy distillation: teacher servers, rollout actors, and the student-to-actor weight
snapshot broadcast (reference aurora/klein.py:198-320, aurora/opd_actor.py, train_pp.py:1146-1326).

Layout: ranks [0, L) learners, [L, L + A) rollout actors, [L + A, world) teachers. Control messages (small int64
headers) travel over a Gloo group, so servers can receive from any learner; tensors travel over the default group
(NCCL on GPUs). Protocols:

* Teacher: header [KIND_VELOCITY, B, C, h, w, L, D, chunks, deferred] from a learner, then x (B, C, h, w) fp32, t
  (B,), LM states (B, L, D), valid (B, L) uint8; reply: the teacher's CFG velocity (B, C, h, w) fp32, computed in
  ``chunks`` row chunks (bounded teacher memory; 0 or 1 = the whole part at once). A learner spreads a batch over
  the teacher ranks (a rotating first rank per request). A deferred request (``request(..., deferred=True)``, then
  ``collect``) is computed at once but its reply is held by the teacher until the learner sends [KIND_COLLECT] and
  waits for it: the teacher never leaves a send pending on its stream, where it would hold up the next learner's
  request while that learner's stream (and through the gradient all-reduce, every learner) waits on it. One deferred
  request per learner and teacher at a time. KIND_STOP ends the server.
* Every tensor send of these protocols (a learner's request data, a server's reply) is an ``isend`` whose handle
  (and tensor) is kept until the exchange is over, never a blocking ``send``: on NCCL a ``send`` makes the sender's
  compute stream wait until the receiver takes the data, and with several learners and several servers those waits
  can close a cycle (learner X's stream waits on its send to server 2, which waits on server 2's send to learner Y,
  which waits on Y's send to server 1, which waits on server 1's send to X). With ``isend`` a compute stream waits
  only on the receives its own work reads, and the protocols' data dependencies form no cycle.
* Actor: header [KIND_ROLLOUT, B, C, h, w, L, D, step, version, deferred, shift x 1000 (0: the actor's default)] with
  noise / LM states / valid (the shift is the batch resolution's, as a local rollout would use); the actor
  generates the rollout states with the snapshot it holds and replies with (states (B m, C, h, w), t (B m,)); a
  deferred job's reply is held until the learner's [KIND_COLLECT] (one job per learner at a time), so a learner
  trains while its next batch is rolled out. It refuses a job whose required snapshot version is newer than its own
  (the learner always sends the snapshot first).
* Snapshot: learner 0 flattens the student's parameters and streams them into every actor's mapped buffer with the
  peer-copy kernel (NVLink stores, then a version word), then tells each actor (Gloo) the version; on CPU the flat
  tensor is sent over the process group instead. Versions only grow; an actor applies a snapshot only between jobs.
"""
import torch
import torch.distributed as dist

KIND_STOP, KIND_VELOCITY, KIND_ROLLOUT, KIND_SNAPSHOT, KIND_COLLECT = 0, 1, 2, 3, 4
HDR = 12


class RoleLayout:
    def __init__(self, world, learners, actors=0, teachers=0):
        assert learners + actors + teachers == world, "learners + actors + teachers must equal the world size"
        self.learners = list(range(learners))
        self.actors = list(range(learners, learners + actors))
        self.teachers = list(range(learners + actors, world))

    def role(self, rank):
        if rank in self.learners:
            return "learner"
        return "actor" if rank in self.actors else "teacher"


def _hdr(*vals):
    h = torch.zeros(HDR, dtype=torch.int64)
    h[:len(vals)] = torch.tensor(vals, dtype=torch.int64)
    return h


class _Outgoing:
    """Sends in flight: (work, tensor) kept until complete, so neither the stream nor the buffer is waited on early."""

    def __init__(self):
        self.items = []

    def send(self, tensor, dst):
        self.items.append((dist.isend(tensor, dst=dst), tensor))
        self.items = [(w, t) for w, t in self.items if not w.is_completed()]

    def wait(self):
        for w, _ in self.items:
            w.wait()
        self.items = []


class TeacherServer:
    def __init__(self, teacher, device, control_group, dtype=torch.float32):
        self.teacher, self.device, self.ctl, self.dtype = teacher, device, control_group, dtype

    def serve(self):
        served = 0
        held = {}  # learner rank -> the reply of its deferred request
        out = _Outgoing()
        while True:
            h = torch.zeros(HDR, dtype=torch.int64)
            src = dist.recv(h, group=self.ctl)
            kind, B, C, hh, w, L, D, chunks, deferred = h[:9].tolist()
            if kind == KIND_STOP:
                out.wait()
                return served
            if kind == KIND_COLLECT:
                if src not in held:
                    raise RuntimeError(f"teacher: rank {src} collects a reply it never requested")
                out.send(held.pop(src), src)
                continue
            x = torch.empty(B, C, hh, w, device=self.device)
            t = torch.empty(B, device=self.device)
            st = torch.empty(B, L, D, device=self.device, dtype=self.dtype)
            valid = torch.empty(B, L, device=self.device, dtype=torch.uint8)
            for buf in (x, t, st, valid):
                dist.recv(buf, src=src)
            v = chunked_velocity(self.teacher, x, t, dict(lm_states=st, valid=valid.bool()), chunks)
            v = v.float().contiguous()
            served += 1
            if deferred:
                if src in held:
                    raise RuntimeError(f"teacher: rank {src} sent a second deferred request before collecting")
                held[src] = v
            else:
                out.send(v, src)


def chunked_velocity(teacher, x, t, text_kw, chunks=1):
    """teacher.velocity over ``chunks`` row chunks of the batch (concatenated in order)."""
    B = x.shape[0]
    n = max(1, min(int(chunks), B))
    if n == 1:
        return teacher.velocity(x, t, text_kw)
    cuts = [(i * B // n, (i + 1) * B // n) for i in range(n)]
    return torch.cat([teacher.velocity(x[a:b], t[a:b], {k: v[a:b] for k, v in text_kw.items()}) for a, b in cuts])


class TeacherClient:
    def __init__(self, teachers, control_group, rank):
        self.teachers, self.ctl, self.rank = teachers, control_group, rank
        self.turn = rank

    def velocity(self, x, t, text_kw):
        """Split the batch over the teacher ranks, send every part, then collect the replies in order."""
        return self.collect(self.request(x, t, text_kw))

    def request(self, x, t, text_kw, chunks=1, deferred=False):
        """Send the parts of a batch to the teachers (one part per teacher, computed there in ``chunks`` row
        chunks) and return a handle for ``collect``. Not deferred: the teachers send their replies at once and the
        caller must collect next. Deferred: the teachers hold the replies until ``collect`` asks for them, so the
        caller trains meanwhile (one deferred request per teacher at a time)."""
        st, valid = text_kw["lm_states"], text_kw["valid"]
        B = x.shape[0]
        n = len(self.teachers)
        parts = [(i * B // n, (i + 1) * B // n) for i in range(n)]
        order = [self.teachers[(self.turn + i) % n] for i in range(n)]
        self.turn += 1
        replies, sends = [], _Outgoing()
        for (b0, b1), dst in zip(parts, order):
            if b1 <= b0:
                continue
            xs = x[b0:b1].float().contiguous()
            dist.send(_hdr(KIND_VELOCITY, b1 - b0, *xs.shape[1:], *st.shape[1:], chunks, int(deferred)), dst=dst,
                      group=self.ctl)
            for buf in (xs, t[b0:b1].float().contiguous(), st[b0:b1].contiguous(),
                        valid[b0:b1].to(torch.uint8).contiguous()):
                sends.send(buf, dst)
            replies.append((b0, b1, dst))
        return replies, B, tuple(x.shape[1:]), x.device, deferred, sends

    def collect(self, handle):
        replies, B, shape, device, deferred, sends = handle
        out = torch.empty(B, *shape, device=device)
        for b0, b1, dst in replies:
            if deferred:
                dist.send(_hdr(KIND_COLLECT), dst=dst, group=self.ctl)
            buf = torch.empty(b1 - b0, *shape, device=device)
            dist.recv(buf, src=dst)
            out[b0:b1] = buf
        sends.wait()  # long complete: each teacher replied after receiving its part
        return out

    def stop(self):
        for dst in self.teachers:
            dist.send(_hdr(KIND_STOP), dst=dst, group=self.ctl)


def flat_params(params):
    return torch.cat([p.detach().reshape(-1).float() for p in params])


@torch.no_grad()
def load_flat(params, flat):
    off = 0
    for p in params:
        n = p.numel()
        p.copy_(flat[off:off + n].view_as(p).to(p.dtype))
        off += n


class SnapshotSender:
    """Learner 0 -> actors. On CUDA: peer-copy kernel into each actor's IPC-mapped buffer; else process-group
    sends."""

    def __init__(self, params, actors, control_group, peer_buffers=None):
        self.params, self.actors, self.ctl = list(params), actors, control_group
        self.n = sum(p.numel() for p in self.params)
        self.pb = peer_buffers
        self.version = 0
        self.counter = None
        self.last_copy = None  # (bytes, device ms) of the last snapshot's peer copies, summed over the actors
        if self.pb is not None:
            self.counter = torch.zeros(1, dtype=torch.int64, device=self.params[0].device)

    def send(self):
        self.version += 1
        flat = flat_params(self.params)
        nbytes, ms = 0, 0.0
        for dst in self.actors:
            dist.send(_hdr(KIND_SNAPSHOT, self.version, self.n), dst=dst, group=self.ctl)
            if self.pb is not None:
                from ..ops._ext import ext
                j = self.pb.group_ranks.index(dst)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                ext().peer_copy(self.pb.ptrs["flat"][j], flat, self.pb.ptrs["version"][j], self.counter.data_ptr(),
                                self.version, 64)
                e1.record()
                torch.cuda.current_stream().synchronize()
                nbytes += flat.numel() * flat.element_size()
                ms += e0.elapsed_time(e1)
                self.last_copy = (nbytes, ms)
                dist.send(_hdr(KIND_SNAPSHOT, self.version), dst=dst, group=self.ctl)  # data landed
            else:
                dist.send(flat, dst=dst)
        return self.version


class RolloutActor:
    """Holds a student copy; applies snapshots; serves rollout jobs from learners."""

    def __init__(self, te, den, params, device, control_group, opd_kwargs, peer_buffers=None, local_flat=None):
        self.te, self.den, self.params, self.device, self.ctl = te, den, list(params), device, control_group
        self.kw = opd_kwargs
        self.version = 0
        self.pb, self.local_flat = peer_buffers, local_flat
        self.n = sum(p.numel() for p in self.params)

    def _apply_snapshot(self, src, version):
        if self.pb is None:
            flat = torch.empty(self.n, device=self.device)
            dist.recv(flat, src=src)
        else:
            h = torch.zeros(HDR, dtype=torch.int64)
            dist.recv(h, src=src, group=self.ctl)  # the learner finished the peer copy
            flat = self.local_flat
            assert h[1].item() == version
        load_flat(self.params, flat)
        self.version = version

    @torch.no_grad()
    def serve(self):
        from ..ops.reference import valid_to_len
        from ..train.opd import dance_picks, diffusion_picks, opd_grid, rollout
        jobs = 0
        held = {}  # learner rank -> (states, t) of its deferred job
        out = _Outgoing()
        while True:
            h = torch.zeros(HDR, dtype=torch.int64)
            src = dist.recv(h, group=self.ctl)
            kind = int(h[0])
            if kind == KIND_STOP:
                out.wait()
                return jobs
            if kind == KIND_SNAPSHOT:
                self._apply_snapshot(src, int(h[1]))
                continue
            if kind == KIND_COLLECT:
                if src not in held:
                    raise RuntimeError(f"actor: rank {src} collects a job it never submitted")
                for buf in held.pop(src):
                    out.send(buf, src)
                continue
            _, B, C, hh, w, L, D, step, need, deferred, shift_milli = h[:11].tolist()
            if need > self.version:
                raise RuntimeError(f"actor holds snapshot {self.version}, job needs {need}")
            noise = torch.empty(B, C, hh, w, device=self.device)
            st = torch.empty(B, L, D, device=self.device, dtype=self.kw.get("dtype", torch.float32))
            valid = torch.empty(B, L, device=self.device, dtype=torch.uint8)
            for buf in (noise, st, valid):
                dist.recv(buf, src=src)
            K, m = self.kw["K"], self.kw["m"]
            g = torch.Generator().manual_seed(self.kw["seed"] * 1_000_003 + src * 1009 + step + 7)
            picks = dance_picks(B, m, K, self.kw["beta"], self.kw["seed"], src, step) if self.kw["method"] == "dance" \
                else diffusion_picks(B, m, K, g)
            shift = shift_milli / 1000 if shift_milli > 0 else self.kw["shift"]
            ts = opd_grid(K, shift, torch.rand((), generator=g).item(), self.device)
            text, v = self.te(lm_states=st, valid=valid.bool())
            states = rollout(self.den, text, valid_to_len(v), noise, ts, picks, self.kw["mb"]).flatten(0, 1)
            t = ts[picks.to(self.device)].flatten().contiguous()
            jobs += 1
            if deferred:
                if src in held:
                    raise RuntimeError(f"actor: rank {src} submitted a second deferred job before collecting")
                held[src] = (states.contiguous(), t)
                continue
            out.send(states.contiguous(), src)
            out.send(t, src)


class ActorClient:
    def __init__(self, actor, control_group, m):
        self.actor, self.ctl, self.m = actor, control_group, m

    def rollouts(self, noise, lm_states, valid, step, version, shift=None):
        return self.collect(self.request(noise, lm_states, valid, step, version, shift=shift))

    def request(self, noise, lm_states, valid, step, version, deferred=False, shift=None):
        """Submit a rollout job; ``collect`` returns (states, t). Deferred: the actor holds the result until it is
        collected (one deferred job per learner and actor at a time)."""
        B = noise.shape[0]
        dist.send(_hdr(KIND_ROLLOUT, B, *noise.shape[1:], *lm_states.shape[1:], step, version, int(deferred),
                       round(shift * 1000) if shift else 0),
                  dst=self.actor, group=self.ctl)
        sends = _Outgoing()
        for buf in (noise.float().contiguous(), lm_states.contiguous(), valid.to(torch.uint8).contiguous()):
            sends.send(buf, self.actor)
        return B, tuple(noise.shape[1:]), noise.device, deferred, sends

    def collect(self, handle):
        B, shape, device, deferred, sends = handle
        if deferred:
            dist.send(_hdr(KIND_COLLECT), dst=self.actor, group=self.ctl)
        states = torch.empty(B * self.m, *shape, device=device)
        t = torch.empty(B * self.m, device=device)
        dist.recv(states, src=self.actor)
        dist.recv(t, src=self.actor)
        sends.wait()  # long complete: the actor replied after receiving the job
        return states, t

    def stop(self):
        dist.send(_hdr(KIND_STOP), dst=self.actor, group=self.ctl)
