"""The fused single-owner Muon step on the GPU (segment-table momentum, tcgen05 Newton-Schulz, fused apply with
the bf16 shadow refresh) against the per-matrix oracle of the update rule."""
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.optim.muon import Muon

from test_muon_cpu import oracle_step

pytestmark = pytest.mark.gpu

SHAPES = [(256, 128), (128, 384), (256, 128), (384, 128), (192, 192), (1024, 512)]
SPLITS = {3: [128, 128, 128]}


@pytest.mark.parametrize("mdt", [None, torch.bfloat16])
def test_fused_muon_matches_oracle(mdt):
    from trenowanie_generatora_obrazkow_b200.ops.fused import bf16_weight
    torch.manual_seed(0)
    init = [torch.randn(*s, device="cuda") * 0.05 for s in SHAPES]
    pa = [torch.nn.Parameter(t.clone()) for t in init]
    pb = [torch.nn.Parameter(t.clone()) for t in init]
    opt = Muon(pa, lr=0.02, momentum=0.9, weight_decay=0.01, shard=False,
               splits={pa[k]: v for k, v in SPLITS.items()}, momentum_dtype=mdt)
    bufs = [torch.zeros_like(p) for p in pb]
    for p in pa:
        bf16_weight(p)  # shadows exist before the step: the fused apply must refresh them in place
    for step in range(3):
        g = torch.Generator(device="cuda").manual_seed(11 + step)
        for a, b in zip(pa, pb):
            a.grad = torch.randn(a.shape, device="cuda", generator=g)
            b.grad = a.grad.clone()
        opt.step()
        oracle_step(pb, bufs, 0.02, 0.9, 0.01, SPLITS)
    torch.cuda.synchronize()
    for a, b, m in zip(pa, pb, bufs):
        tol = 2e-3 if mdt is None else 4e-3
        assert (a.detach() - b.detach()).abs().max() < tol
        assert torch.equal(bf16_weight(a), a.detach().bfloat16())
        mm = opt.momentum_buffer(a).float()
        assert torch.allclose(mm, m, atol=1e-6 if mdt is None else 2e-2, rtol=0 if mdt is None else 1e-2)
