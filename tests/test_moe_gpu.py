"""MoE layer on the GPU (batched tcgen05 expert GEMMs) against the same layer on the CPU in fp32."""
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.models.moe import MoEMLP

pytestmark = pytest.mark.gpu


def test_moe_gpu_matches_cpu():
    torch.manual_seed(0)
    cpu = MoEMLP(256, 384, experts=8, top_k=2, capacity_factor=4.0)
    gpu = MoEMLP(256, 384, experts=8, top_k=2, capacity_factor=4.0).cuda()
    gpu.load_state_dict(cpu.state_dict())
    h = torch.randn(4, 64, 256)
    hc = h.clone().requires_grad_()
    out_c = cpu(hc)
    out_c.square().mean().backward()
    hg = h.cuda().bfloat16().requires_grad_()
    out_g = gpu(hg)
    out_g.float().square().mean().backward()
    rel = lambda a, b: ((a.float().cpu() - b.float()).norm() / b.float().norm()).item()
    assert rel(out_g, out_c) < 2e-2
    assert rel(hg.grad, hc.grad) < 4e-2
    assert rel(gpu.w_in.grad, cpu.w_in.grad) < 4e-2
    assert rel(gpu.w_out.grad, cpu.w_out.grad) < 4e-2
