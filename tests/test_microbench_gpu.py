"""The kernel micro-benchmark runs end to end (one timed launch per op, small shapes)."""
import pytest

pytestmark = pytest.mark.gpu


def test_microbench_small():
    from trenowanie_generatora_obrazkow_b200.ops import microbench
    ops = "gemm_out,attn_fwd,attn_cross_4k,adanorm_bwd,qknorm_rope_bwd,swiglu_bwd,euler_cfg,gemm_swiglu,gemm_grouped"
    rows = microbench.main(["--op", ops, "--small", "--iters", "1", "--warmup", "1"])
    assert len(rows) == 9 and all(r["ours"]["ms"] > 0 and r["library"]["ms"] > 0 for r in rows)
