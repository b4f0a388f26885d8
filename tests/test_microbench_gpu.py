"""The kernel micro-benchmark runs end to end (one timed launch per op, small shapes)."""
import pytest

pytestmark = pytest.mark.gpu


def test_microbench_small():
    from trenowanie_generatora_obrazkow_b200.ops import microbench
    rows = microbench.main(["--op", "gemm_out,attn_fwd,adanorm_bwd,qknorm_rope_bwd,swiglu_bwd,euler_cfg", "--small",
                            "--iters", "1", "--warmup", "1"])
    assert len(rows) == 6 and all(r["ours"]["ms"] > 0 and r["library"]["ms"] > 0 for r in rows)
