"""Memory diagnostics (reference train_pp.py:401-426, :1852-1900, :2278-2281, :2400-2420): a per-category breakdown
of what a rank holds (weights, gradients, optimizer state, EMA, outer/DiLoCo copies, frozen LM), allocator figures
(allocated, reserved, peak, allocation retries), host RSS including worker processes, and an OOM guard that prints
the breakdown and dumps an allocator snapshot before re-raising (no collective: peers may be stuck)."""
import contextlib
import os

import torch


def tensor_bytes(tensors):
    seen, total = set(), 0
    for t in tensors:
        if t is None or not torch.is_tensor(t):
            continue
        key = (t.untyped_storage().data_ptr(), t.device)
        if key in seen:
            continue
        seen.add(key)
        total += t.untyped_storage().nbytes()
    return total


def optimizer_tensors(opt):
    for st in opt.state.values():
        for v in st.values():
            if torch.is_tensor(v):
                yield v


def breakdown(params=(), grads=(), opts=(), ema=None, extra=None):
    """{category: GB}. ``extra``: {name: iterable of tensors} (e.g. the frozen LM, DiLoCo global copies)."""
    gb = 1024 ** 3
    out = {"weights": tensor_bytes(params) / gb, "grads": tensor_bytes(grads) / gb,
           "optimizer": tensor_bytes(t for o in opts for t in optimizer_tensors(o)) / gb}
    if ema is not None:
        out["ema"] = tensor_bytes(getattr(ema, "shadow", ema)) / gb
    for k, ts in (extra or {}).items():
        out[k] = tensor_bytes(ts) / gb
    return out


def allocator_stats(device=None):
    if not torch.cuda.is_available():
        return {}
    s = torch.cuda.memory_stats(device)
    gb = 1024 ** 3
    return {"allocated_gb": s.get("allocated_bytes.all.current", 0) / gb,
            "reserved_gb": s.get("reserved_bytes.all.current", 0) / gb,
            "peak_gb": s.get("allocated_bytes.all.peak", 0) / gb,
            "alloc_retries": s.get("num_alloc_retries", 0), "ooms": s.get("num_ooms", 0)}


def host_rss_gb(include_children=True):
    import psutil
    proc = psutil.Process(os.getpid())
    rss = proc.memory_info().rss
    if include_children:
        for c in proc.children(recursive=True):
            try:
                rss += c.memory_info().rss
            except psutil.Error:
                pass
    return rss / 1024 ** 3


def report(rank=0, **kw):
    parts = breakdown(**kw)
    parts.update(allocator_stats())
    parts["host_rss_gb"] = host_rss_gb()
    return f"[rank {rank}] memory: " + ", ".join(f"{k} {v:.2f}" if isinstance(v, float) else f"{k} {v}"
                                                 for k, v in parts.items())


@contextlib.contextmanager
def oom_guard(describe, snapshot_path=None, log=print):
    """Run the body; on CUDA out-of-memory print ``describe()`` and save an allocator snapshot, then re-raise."""
    try:
        yield
    except torch.OutOfMemoryError:
        log(describe())
        if snapshot_path and torch.cuda.is_available():
            try:
                import pickle
                with open(snapshot_path, "wb") as f:
                    pickle.dump(torch.cuda.memory._snapshot(), f)
                log(f"allocator snapshot written to {snapshot_path}")
            except Exception as e:  # diagnostics must not hide the original error
                log(f"snapshot failed: {e}")
        raise
