"""Profiling and FLOP accounting (reference tests/check_profiling.py): a disabled profile creates no profiler and
labels nothing, the window runs only on the selected ranks and only for its steps, the kernel table leaves the
phase annotations out (their device time would count every kernel twice), and the FLOP count of a step grows with
the text width and the image tokens as the model's linear layers and attention do."""
import json
import os
from dataclasses import replace
from types import SimpleNamespace

import torch

from trenowanie_generatora_obrazkow_b200.models.config import make_configs
from trenowanie_generatora_obrazkow_b200.utils import profiling as P
from trenowanie_generatora_obrazkow_b200.utils.flops import train_flops_per_sample


def test_disabled_profile_is_free(tmp_path, monkeypatch):
    started = []
    monkeypatch.setattr(torch.profiler, "profile", lambda *a, **k: started.append(1))
    for prof in (P.TrainingProfile(None, start=0, steps=2),                       # no output directory
                 P.TrainingProfile(str(tmp_path), start=0, steps=0),              # no steps
                 P.TrainingProfile(str(tmp_path), start=0, steps=2, ranks=(1,), rank=0)):  # another rank
        assert not prof.enabled
        for step in range(3):
            prof.step_begin(step)
            with prof.phase("forward_backward") as ctx:
                assert ctx is None  # a null context: no record_function
            prof.step_end(step)
    assert started == [] and os.listdir(tmp_path) == []


def test_profile_window_on_the_selected_rank(tmp_path):
    prof = P.TrainingProfile(str(tmp_path), start=2, steps=2, ranks=(0, 3), rank=3)
    active = []
    for step in range(6):
        prof.step_begin(step)
        active.append(prof.prof is not None)
        with prof.phase("optimizer"):
            torch.ones(8).mul_(2)
        prof.step_end(step)
    assert active == [False, False, True, True, False, False] and not prof.enabled
    assert sorted(os.listdir(tmp_path)) == ["kernels_rank3.json", "ops_rank3.txt", "trace_rank3.json"]
    trace = json.load(open(tmp_path / "trace_rank3.json"))
    names = {e.get("name") for e in trace["traceEvents"]}
    assert "train/optimizer" in names


def test_kernel_table_excludes_phase_annotations():
    cuda = torch.autograd.DeviceType.CUDA
    ev = lambda name, us, dev=cuda: SimpleNamespace(name=name, device_type=dev, device_time_total=us)
    fake = SimpleNamespace(events=lambda: [ev("train/forward_backward", 3000.0), ev("gemm_tcgen05", 2000.0),
                                           ev("gemm_tcgen05", 500.0), ev("flash_fwd_tc", 500.0),
                                           ev("aten::mm", 9999.0, torch.autograd.DeviceType.CPU)])
    table, total = P.kernel_table(fake)
    assert total == 3.0  # ms: the annotation's 3 ms and the CPU op are not added
    assert [(n, ms, c) for n, ms, c, _ in table] == [("gemm_tcgen05", 2.5, 2), ("flash_fwd_tc", 0.5, 1)]
    assert abs(sum(s for *_, s in table) - 1.0) < 1e-9
    assert "total" in P.summarize_kernels(table, total)


def test_flops_scale_with_text_width_and_tokens():
    den, te = make_configs("1.24b", "states1024")
    base = train_flops_per_sample(den, te, 1024)
    wider = train_flops_per_sample(replace(den, text_dim=2 * den.text_dim), replace(te, dim=2 * te.dim), 1024)
    assert wider > base
    # the linear layers grow linearly in the image tokens, attention quadratically
    f1, f2, f4 = (train_flops_per_sample(den, te, t) for t in (1024, 2048, 4096))
    assert f4 - f2 > 2 * (f2 - f1) > 0
    # 3 x forward (forward + two backward GEMMs): about 6 N T for the 1.24B denoiser at 1024 tokens, plus attention
    n_params = 1.24e9
    assert 6 * n_params * 1024 * 0.8 < base < 6 * n_params * 1024 * 1.6


def test_phase_timer_is_inert_on_cpu():
    t = P.PhaseTimer("cpu")
    t.begin()
    t.mark("forward")
    assert t.collect() == {}


def test_profile_stacks_map_ops_to_python_frames(tmp_path, monkeypatch):
    """PROFILE_STACK=1: collapsed stacks (weighted by op time) and an op table grouped by the issuing frames."""
    monkeypatch.setenv("PROFILE_STACK", "1")
    prof = P.TrainingProfile(str(tmp_path), start=0, steps=1)
    assert prof.stacks

    def my_training_phase(x):
        return (x @ x).relu().sum()

    prof.step_begin(0)
    with prof.phase("forward_backward"):
        my_training_phase(torch.randn(64, 64))
    prof.step_end(0)
    assert {"stacks_rank0.txt", "ops_by_frame_rank0.txt"} <= set(os.listdir(tmp_path))
    assert "my_training_phase" in open(tmp_path / "ops_by_frame_rank0.txt").read()


def test_component_bench_harness_on_cpu():
    """ops/component_bench.py (the reference's tests/bench_ckpt.py and bench_te.py) runs its patterns on a tiny
    case: one row per checkpointing mode and per LM depth (CPU wall clock, no memory figures)."""
    from trenowanie_generatora_obrazkow_b200.ops import component_bench as C
    rows = C.ckpt_bench(size="nano", blocks=2, mb=2, inflight=2, res=128, text_len=8, modes=("none", "full"),
                        iters=1, warmup=0, device="cpu", log=lambda s: None)
    assert [r["mode"] for r in rows] == ["none", "full"] and all(r["ms_per_microbatch"] > 0 for r in rows)
    assert rows[0]["peak_mb"] is None
    rows = C.te_bench(layers=(1, 2), batch=3, tokens=8, n_embd=64, n_head=2, iters=1, warmup=0, device="cpu",
                      log=lambda s: None)
    assert [r["layers"] for r in rows] == [1, 2] and rows[1]["weights_mb"] > rows[0]["weights_mb"]
