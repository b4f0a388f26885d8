"""Frozen-LM / VAE services on dedicated ranks and the distributed LM-state helpers of the pipeline trainer
(reference train_pp.py:457-732 for the LM server, its client and the stage helpers; aurora/opd_text.py:1-79 for
the text lookahead).

Layout and planes. Service ranks sit after the learners (and actors / teachers, see ``placement.RankLayout``).
Control: a Gloo group carries 3-word int64 headers ``[kind, n, L]`` received from ANY source, so a server takes
whichever client is ready first, plus the CPU caption ids. Data: LM states, images and latents travel over the
default group, which is NCCL over NVLink on GPUs (Gloo on CPU). Both peers derive the same ``chunk_plan`` from the
CPU ids, so receives are posted before any device work and no device value is read on the host.

Header kinds:
  0 STOP     the client is done (a server ends once every client has stopped)
  1 LM       ids (n, L) int64 follow on the control group (tag 2); one states tensor per plan chunk comes back
  2 TEACHER  handed to the ``teacher`` callback (the OPD teacher protocol, parallel/roles.py)
  3 VAE      uint8 images (n, 3, L, L) follow on the data plane; float32 latents go back
  4 TEXT     a CPU job (ids + caption texts) follows on the text group; CPU LM states (+ the optional second text
             encoder's states) go back: the text lookahead of on-policy distillation

The server keeps a utilisation window (LM compute timed by CUDA events, the transfer / dispatch residual, idle
time waiting for requests) and logs it every ``report_every`` seconds.
"""
import pickle
import time
from collections import deque
from concurrent.futures import ThreadPoolExecutor

import torch
import torch.distributed as dist

from ..models.frozen_lm import LM_NULL, LM_PAD

KIND_STOP, KIND_LM, KIND_TEACHER, KIND_VAE, KIND_TEXT = 0, 1, 2, 3, 4
TAG_HDR, TAG_IDS = 1, 2


# ---------------------------------------------------------------------------------------------------------------
# request planning (identical on both peers, CPU only)
# ---------------------------------------------------------------------------------------------------------------
def trim_ids(ids, multiple=8):
    """Drop all-padding tail columns of right-padded caption rows, keeping a multiple of ``multiple`` columns."""
    n = int(ids.ne(LM_PAD).sum(1).max()) if ids.numel() else 1
    return ids[:, :min(ids.shape[1], max(multiple, -(-n // multiple) * multiple))]


def chunk_plan(ids, chunk=32):
    """[(first row, real row indices within the chunk, trimmed ids of those rows)] per chunk of ``chunk`` rows;
    null-prompt rows are not run (the refiner replaces them by its learned null vector)."""
    assert ids.device.type == "cpu", "plan LM requests from CPU ids"
    plan = []
    for i in range(0, ids.shape[0], chunk):
        c = ids[i:i + chunk]
        rows = c[:, 0].ne(LM_NULL).nonzero().flatten()
        if rows.numel():
            plan.append((i, rows, trim_ids(c[rows])))
    return plan


def scatter_plan(plan, outs, shape, width, device, dtype=torch.bfloat16):
    """Chunk results back into a zero (n, L, width) tensor."""
    full = torch.zeros(*shape, width, dtype=dtype, device=device)
    for (i, rows, sub), h in zip(plan, outs):
        full[:, :sub.shape[1]].index_copy_(0, (rows + i).to(device), h.to(device, dtype))
    return full


# ---------------------------------------------------------------------------------------------------------------
# CPU payloads (dicts of tensors and small metadata) over a Gloo group
# ---------------------------------------------------------------------------------------------------------------
def send_payload(payload, dst, group):
    """Metadata pickled into one uint8 tensor (length first); tensors sent raw, without pickling their storage."""
    tensors = {k: v for k, v in payload.items() if isinstance(v, torch.Tensor)}
    meta = {k: v for k, v in payload.items() if k not in tensors}
    specs = [(k, tuple(t.shape), t.dtype) for k, t in tensors.items()]
    blob = torch.frombuffer(bytearray(pickle.dumps((meta, specs))), dtype=torch.uint8)
    dist.send(torch.tensor([blob.numel()], dtype=torch.int64), dst, group=group)
    dist.send(blob, dst, group=group)
    for t in tensors.values():
        assert t.device.type == "cpu", "payload tensors live on the host"
        dist.send(t.contiguous(), dst, group=group)


def recv_payload(src, group):
    n = torch.empty(1, dtype=torch.int64)
    dist.recv(n, src, group=group)
    blob = torch.empty(int(n), dtype=torch.uint8)
    dist.recv(blob, src, group=group)
    meta, specs = pickle.loads(blob.numpy().tobytes())
    for key, shape, dtype in specs:
        t = torch.empty(shape, dtype=dtype)
        dist.recv(t, src, group=group)
        meta[key] = t
    return meta


# ---------------------------------------------------------------------------------------------------------------
# server
# ---------------------------------------------------------------------------------------------------------------
class _Window:
    def __init__(self):
        self.reset()

    def reset(self):
        self.t0 = time.perf_counter()
        self.idle = self.compute = self.transfer = self.vae = 0.0
        self.captions = self.images = 0


class LMService:
    """Serve LM states (and optionally VAE encodes, text jobs, teacher requests) to ``clients`` until each of them
    has sent STOP. ``states_fn(sub)``: (rows, L) caption ids with LM_PAD -> (rows, L, width) states on ``device``
    (e.g. ``SlayerFrozenLM.states``, packed on CUDA). ``vae(u8)``: (n, 3, H, H) uint8 -> float32 latents.
    ``text_fn(job)``: CPU job dict -> dict of extra CPU tensors (a second text encoder). ``teacher(src, hdr)``:
    serves one teacher request. Clients that also use this rank as their teacher are listed in
    ``teacher_clients``: each of them sends one STOP per role."""

    def __init__(self, states_fn, width, device, control_group, clients, *, vae=None, text_group=None, text_fn=None,
                 teacher=None, teacher_clients=(), log=print, report_every=60.0):
        self.states_fn, self.width, self.device = states_fn, width, torch.device(device)
        self.ctl, self.text_group = control_group, text_group
        self.vae, self.text_fn, self.teacher = vae, text_fn, teacher
        self.stops = {c: int(c in clients) + int(c in teacher_clients) for c in set(clients) | set(teacher_clients)}
        self.log, self.report_every = log, report_every
        self.win = _Window()
        self.served = 0

    def _timed_states(self, sub):
        cuda = self.device.type == "cuda"
        if cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        h = self.states_fn(sub.to(self.device)).to(torch.bfloat16).contiguous()
        return h, ((a, b) if cuda else None)

    def _lm(self, src, hdr):
        ids = torch.empty(int(hdr[1]), int(hdr[2]), dtype=torch.int64)
        dist.recv(ids, src, group=self.ctl, tag=TAG_IDS)
        start = time.perf_counter()
        sends, events = [], []
        for _, _, sub in chunk_plan(ids):
            h, ev = self._timed_states(sub)
            if ev is not None:
                ev[1].record()
                events.append(ev)
            sends.append((dist.isend(h, dst=src), h))
        for req, _ in sends:
            req.wait()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        gpu = sum(a.elapsed_time(b) for a, b in events) / 1e3
        cpu_gpu = time.perf_counter() - start
        self.win.compute += gpu if events else cpu_gpu
        self.win.transfer += max(0.0, cpu_gpu - gpu) if events else 0.0
        self.win.captions += ids.shape[0]
        self.served += ids.shape[0]

    def _vae(self, src, hdr):
        assert self.vae is not None, "VAE request to a server without a VAE"
        n, side = int(hdr[1]), int(hdr[2])
        u8 = torch.empty(n, 3, side, side, dtype=torch.uint8, device=self.device)
        dist.recv(u8, src=src)
        start = time.perf_counter()
        lat = self.vae(u8).float().contiguous()
        dist.isend(lat, dst=src).wait()
        self.win.vae += time.perf_counter() - start
        self.win.images += n

    def _text(self, src):
        assert self.text_group is not None, "text job to a server without a text group"
        job = recv_payload(src, self.text_group)
        ids = job["ids"]
        plan = chunk_plan(ids)
        outs = [self._timed_states(sub)[0].cpu() for _, _, sub in plan]
        reply = dict(lm=scatter_plan(plan, outs, ids.shape, self.width, "cpu"))
        if self.text_fn is not None:
            reply.update(self.text_fn(job))
        send_payload(reply, src, self.text_group)
        self.served += ids.shape[0]

    def _report(self, force=False):
        dt = time.perf_counter() - self.win.t0
        if not force and dt < self.report_every:
            return
        w = self.win
        msg = (f"LM server (rank {dist.get_rank()}): LM forward {100 * w.compute / dt:.0f}%, transfer/dispatch "
               f"{100 * w.transfer / dt:.0f}%, waiting {100 * w.idle / dt:.0f}%, {w.captions / dt:.0f} captions/s")
        if self.vae is not None:
            msg += f", VAE {100 * w.vae / dt:.0f}% ({w.images / dt:.1f} images/s)"
        self.log(msg)
        w.reset()

    def serve(self):
        active = {c for c, n in self.stops.items() if n > 0}
        t0 = time.perf_counter()
        while active:
            hdr = torch.empty(3, dtype=torch.int64)
            start = time.perf_counter()
            src = dist.recv(hdr, group=self.ctl, tag=TAG_HDR)  # any ready client
            self.win.idle += time.perf_counter() - start
            if src not in active:
                raise RuntimeError(f"LM server: request from unexpected rank {src}")
            kind = int(hdr[0])
            if kind == KIND_STOP:
                self.stops[src] -= 1
                if self.stops[src] == 0:
                    active.discard(src)
            elif kind == KIND_LM:
                self._lm(src, hdr)
            elif kind == KIND_VAE:
                self._vae(src, hdr)
            elif kind == KIND_TEXT:
                self._text(src)
            elif kind == KIND_TEACHER:
                assert self.teacher is not None, "teacher request to a server without a teacher"
                self.teacher(src, hdr)
            else:
                raise RuntimeError(f"LM server: unknown request kind {kind} from rank {src}")
            self._report()
        self.log(f"LM server (rank {dist.get_rank()}): {self.served:,} captions in "
                 f"{time.perf_counter() - t0:.0f} s, done")
        return self.served


# ---------------------------------------------------------------------------------------------------------------
# client
# ---------------------------------------------------------------------------------------------------------------
class LMClient:
    """One outstanding request at a time per kind; control on the host, results on ``device``. Requests are
    answered in issue order (the server handles one client's headers in order, and the data plane matches a pair
    of ranks' sends and receives in issue order), so a VAE request goes out before the LM request of the same
    batch."""

    def __init__(self, server, width, device, control_group):
        self.server, self.width, self.device, self.ctl = server, width, torch.device(device), control_group

    def _header(self, *vals):
        return dist.isend(torch.tensor(vals, dtype=torch.int64), dst=self.server, group=self.ctl, tag=TAG_HDR)

    def request(self, ids):
        ids = ids.to("cpu", torch.int64).contiguous()
        reqs = [self._header(KIND_LM, ids.shape[0], ids.shape[1]),
                dist.isend(ids, dst=self.server, group=self.ctl, tag=TAG_IDS)]
        plan, bufs = chunk_plan(ids), []
        for _, _, sub in plan:
            bufs.append(torch.empty(*sub.shape, self.width, dtype=torch.bfloat16, device=self.device))
            reqs.append(dist.irecv(bufs[-1], src=self.server))
        return dict(shape=tuple(ids.shape), plan=plan, bufs=bufs, reqs=reqs)

    def collect(self, handle, device=None):
        for r in handle["reqs"]:
            r.wait()
        return scatter_plan(handle["plan"], handle["bufs"], handle["shape"], self.width, device or self.device)

    def states(self, ids):
        return self.collect(self.request(ids))

    def request_vae(self, u8, latent_shape):
        u8 = u8.to(self.device, torch.uint8).contiguous()
        out = torch.empty(*latent_shape, dtype=torch.float32, device=self.device)
        reqs = [self._header(KIND_VAE, u8.shape[0], u8.shape[-1]), dist.isend(u8, dst=self.server),
                dist.irecv(out, src=self.server)]
        return dict(out=out, reqs=reqs, u8=u8)

    @staticmethod
    def vae_collect(handle):
        for r in handle["reqs"]:
            r.wait()
        return handle["out"]

    def stop(self):
        self._header(KIND_STOP, 0, 0).wait()


def encode_remote(job, server, control_group, text_group):
    """Send one CPU text job (ids, texts, ...) to the LM server and merge its CPU states into the job."""
    dist.send(torch.tensor([KIND_TEXT, 0, 0], dtype=torch.int64), server, group=control_group, tag=TAG_HDR)
    send_payload(job, server, text_group)
    job.update(recv_payload(server, text_group))
    return job


class TextLookahead:
    """Bounded queue of future caption batches encoded off the critical path: one worker thread prepares the
    batch of step ``s`` (``prepare(s)``), encodes it (``encode(job)``, e.g. ``encode_remote``) and keeps up to
    ``depth`` results ahead of the consumer; steps advance by ``period``. ``take(s)`` must follow that order."""

    def __init__(self, prepare, encode, start, stop, period=1, depth=2):
        assert period > 0 and depth > 0
        self.prepare, self.encode = prepare, encode
        self.next, self.stop_at, self.period, self.depth = start, stop, period, depth
        self.pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="text-lookahead")
        self.queue = deque()
        self._fill()

    def _fill(self):
        while len(self.queue) < self.depth and self.next < self.stop_at:
            s = self.next
            self.queue.append((s, self.pool.submit(lambda s=s: self.encode(self.prepare(s)))))
            self.next += self.period

    def take(self, step):
        if not self.queue or self.queue[0][0] != step:
            raise RuntimeError(f"text lookahead: step {step} requested out of order")
        _, fut = self.queue.popleft()
        self._fill()
        return fut.result()

    def close(self):
        """Finish the queued jobs (their replies are in flight on the server) before the client sends STOP."""
        try:
            for _, fut in self.queue:
                fut.result()
        finally:
            self.pool.shutdown(wait=True)
            self.queue.clear()


# ---------------------------------------------------------------------------------------------------------------
# LM states inside a pipeline (no server): per-stage LM work, then point-to-point to the consuming stage
# ---------------------------------------------------------------------------------------------------------------
def gather_to_stage(mine, M, s, pp, dst, base):
    """Stage s computed the LM states of micro-batches k with k % pp == s (``mine``: {k: tensor}). Send them to
    stage ``dst`` of the pipeline whose stage 0 is global rank ``base``; there, return all M in order. Sends and
    receives go in increasing k on every rank, so the point-to-point pairs cannot deadlock."""
    if s != dst:
        for k in sorted(mine):
            dist.send(mine[k].contiguous(), dst=base + dst)
        return None
    ref = mine[dst]
    out = []
    for k in range(M):
        if k % pp == s:
            out.append(mine[k])
        else:
            buf = torch.empty_like(ref)
            dist.recv(buf, src=base + k % pp)
            out.append(buf)
    return out


def lm_split_forward(run_slice, chunks, s, pp, base, device, width, carry_width=None):
    """LM layer split: stage s holds LM layers [s L / pp, (s + 1) L / pp) (``run_slice(x)``: ids on stage 0, the
    previous stage's carry (rows, L, carry_width) elsewhere -> the carry for the next stage, or the final states
    (rows, L, width) on the last stage). Each chunk of caption rows flows stage 0 -> ... -> pp - 1 -> stage 0;
    chunk i + 1 starts on stage 0 while later stages work on chunk i. Every rank of the pipeline calls it with the
    same CPU chunks; stage 0 returns one (rows, L, width) bf16 tensor per chunk (zeros on null-prompt rows and
    pads), the others None. A pair of ranks matches its sends and receives in issue order, so both sides issue
    them mirrored: stage 0 "send chunk i, post the receive of its result", stage s "receive chunk i, send it on"."""
    carry_width = carry_width or width
    plans = []
    for c in chunks:
        real = c[:, 0].ne(LM_NULL).nonzero().flatten()
        plans.append((c, real, trim_ids(c[real]) if real.numel() else None))
    results, recvs, sends = [None] * len(plans), [], []
    for i, (c, real, sub) in enumerate(plans):
        if sub is None:
            continue
        if s == 0:
            x = sub.masked_fill(sub.eq(LM_PAD) | sub.eq(LM_NULL), 0).to(device)
        else:
            x = torch.empty(*sub.shape, carry_width, dtype=torch.bfloat16, device=device)
            dist.recv(x, src=base + s - 1)
        h = run_slice(x).to(torch.bfloat16).contiguous()
        if pp > 1:
            sends.append((dist.isend(h, dst=base + (s + 1) % pp), h))
        if s == 0:
            if pp > 1:
                results[i] = torch.empty(*sub.shape, width, dtype=torch.bfloat16, device=device)
                recvs.append(dist.irecv(results[i], src=base + pp - 1))
            else:
                results[i] = h
    for req, _ in sends:
        req.wait()
    if s != 0:
        return None
    for req in recvs:
        req.wait()
    out = []
    for (c, real, sub), h in zip(plans, results):
        full = torch.zeros(c.shape[0], c.shape[1], width, dtype=torch.bfloat16, device=device)
        if h is not None:
            full[real.to(device), :h.shape[1]] = h
        out.append(full)
    return out
