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


def test_moe_peer_exchange_matches_nccl_path_one_gpu():
    """The peer-memory exchange fused with the expert GEMMs (here with one rank: dispatch to itself, flag waits,
    scatter epilogue, combine) against the all_to_all path, over several steps (epochs, back-pressure) and a
    no-grad forward in between."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    torch.manual_seed(1)
    ref = MoEMLP(512, 256, experts=4, top_k=2, capacity_factor=3.0, transport="nccl").cuda()
    fus = MoEMLP(512, 256, experts=4, top_k=2, capacity_factor=3.0, transport="p2p").cuda()
    fus.load_state_dict(ref.state_dict())
    for it in range(3):
        h = torch.randn(2, 300, 512, device="cuda").bfloat16()
        outs, grads = [], []
        for m in (ref, fus):
            m.zero_grad(set_to_none=True)
            x = h.clone().requires_grad_()
            o = m(x)
            o.float().square().mean().backward()
            outs.append(o.float())
            grads.append((x.grad.float(), m.w_in.grad.clone(), m.w_out.grad.clone(), m.router.weight.grad.clone()))
        check_errors()
        rel = lambda a, b: ((a - b).norm() / b.norm().clamp(min=1e-12)).item()
        assert rel(outs[1], outs[0]) < 1e-2, it
        for a, b in zip(grads[1], grads[0]):
            assert rel(a.float(), b.float()) < 3e-2, it
        with torch.no_grad():
            fus(h)
        check_errors()
