"""Opt-in training profiler (reference aurora/profiling.py:11-85; train_pp.py phases).

``TrainingProfile`` costs nothing when disabled (no CUDA events, no synchronisation). When enabled it runs a
``torch.profiler`` window of ``steps`` optimizer steps starting at ``start`` on the selected ranks and labels the
phases of a step with ``record_function('train/<phase>')``. ``export_profile`` writes a chrome trace, a per-kernel
table that excludes the user annotations (so time is not double counted) and a per-op table with shapes. With
``stacks`` (or PROFILE_STACK=1 in the environment) the profiler also records Python stacks, and ``stacks_rank<r>.txt``
holds the collapsed stacks weighted by device time (CPU time on a CPU run; flame-graph input), while
``ops_by_frame_rank<r>.txt`` lists the ops with the Python frame that issued them.
"""
import contextlib
import json
import os

import torch


class TrainingProfile:
    def __init__(self, out_dir=None, start=0, steps=0, ranks=(0,), rank=0, stacks=None):
        self.enabled = bool(out_dir) and steps > 0 and rank in ranks
        self.out_dir, self.start, self.steps, self.rank = out_dir, start, steps, rank
        self.stacks = bool(os.environ.get("PROFILE_STACK")) if stacks is None else stacks
        self.prof = None

    def phase(self, name):
        if self.prof is None:
            return contextlib.nullcontext()
        return torch.profiler.record_function(f"train/{name}")

    def step_begin(self, step):
        if not self.enabled or self.prof is not None or step != self.start:
            return
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.prof = torch.profiler.profile(activities=acts, record_shapes=True, with_stack=self.stacks,
                                           experimental_config=_stack_config() if self.stacks else None)
        self.prof.__enter__()

    def step_end(self, step):
        if self.prof is None or step + 1 < self.start + self.steps:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        export_profile(self.prof, self.out_dir, self.rank, stacks=self.stacks)
        self.prof = None
        self.enabled = False


def kernel_table(prof, top=40):
    """[(name, total_ms, calls, share)] of device kernels (user annotations excluded)."""
    rows = {}
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        if evt.name.startswith("train/"):
            continue
        r = rows.setdefault(evt.name, [0.0, 0])
        r[0] += evt.device_time_total / 1e3 if hasattr(evt, "device_time_total") else evt.cuda_time_total / 1e3
        r[1] += 1
    total = sum(v[0] for v in rows.values()) or 1.0
    out = sorted(((k, v[0], v[1], v[0] / total) for k, v in rows.items()), key=lambda x: -x[1])
    return out[:top], total


def _stack_config():
    """Keep Python stacks for every op (needed by export_stacks)."""
    return torch._C._profiler._ExperimentalConfig(verbose=True)


def export_profile(prof, out_dir, rank=0, stacks=False):
    os.makedirs(out_dir, exist_ok=True)
    prof.export_chrome_trace(os.path.join(out_dir, f"trace_rank{rank}.json"))
    table, total = kernel_table(prof, top=200)
    with open(os.path.join(out_dir, f"kernels_rank{rank}.json"), "w") as f:
        json.dump({"total_ms": total, "kernels": [dict(name=n, ms=ms, calls=c, share=s) for n, ms, c, s in table]},
                  f, indent=1)
    ops = prof.key_averages(group_by_input_shape=True)
    with open(os.path.join(out_dir, f"ops_rank{rank}.txt"), "w") as f:
        f.write(ops.table(sort_by="self_cpu_time_total", row_limit=200))
    if stacks:
        metric = "self_cuda_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
        prof.export_stacks(os.path.join(out_dir, f"stacks_rank{rank}.txt"), metric)
        by_frame = prof.key_averages(group_by_stack_n=5)
        with open(os.path.join(out_dir, f"ops_by_frame_rank{rank}.txt"), "w") as f:
            f.write(by_frame.table(sort_by="self_cpu_time_total", row_limit=100))
    return table, total


def summarize_kernels(table, total, width=90):
    lines = [f"{'kernel':{width}s} {'ms':>9s} {'calls':>6s} {'share':>6s}"]
    for n, ms, c, s in table:
        lines.append(f"{n[:width]:{width}s} {ms:9.2f} {c:6d} {100 * s:5.1f}%")
    lines.append(f"{'total':{width}s} {total:9.2f}")
    return "\n".join(lines)


class PhaseTimer:
    """Device-time breakdown of a training step: ``mark(name)`` records a CUDA event on the current stream; the
    phase called `name` is the device time from the previous mark to this one. Marks are cheap (no
    synchronisation); ``collect()`` synchronises once and returns {phase: ms} summed over the recorded steps.
    On CPU tensors it does nothing."""

    def __init__(self, device):
        self.enabled = torch.device(device).type == "cuda"
        self.steps = []   # per step: [(name, event)]
        self._cur = None

    def begin(self):
        if not self.enabled:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self._cur = [("begin", e)]
        self.steps.append(self._cur)

    def mark(self, name):
        if not self.enabled or self._cur is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self._cur.append((name, e))

    def collect(self):
        """{phase: total ms over the recorded steps} (then cleared); the phases keep their first-seen order."""
        if not self.enabled:
            return {}
        torch.cuda.synchronize()
        out = {}
        for marks in self.steps:
            for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
                out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        self.steps, self._cur = [], None
        return out


def arm_stack_dump():
    """With TGO_STACK_DUMP_S=N in the environment, print every thread's Python stack to stderr once, N seconds from
    now (faulthandler; the process keeps running): shows where each rank of a stuck multi-rank run waits."""
    import os
    secs = os.environ.get("TGO_STACK_DUMP_S")
    if secs:
        import faulthandler
        faulthandler.dump_traceback_later(float(secs), repeat=False)
