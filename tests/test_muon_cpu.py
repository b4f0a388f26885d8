"""Muon over the flat layout against a per-matrix oracle of the update rule, and its checkpoint round trip."""
import math

import pytest
import torch

from trenowanie_generatora_obrazkow_b200.optim.muon import Muon, MuonLayout
from trenowanie_generatora_obrazkow_b200.optim.newton_schulz import zeropower_reference

SHAPES = [(64, 32), (32, 96), (64, 32), (96, 32), (48, 48)]
SPLITS = {3: [32, 32, 32]}  # the 96 x 32 matrix is a fused q / k / v (CMuon row blocks)


def oracle_step(ps, bufs, lr, mu, wd, splits):
    """The update rule, matrix by matrix, in plain torch."""
    for i, (p, m) in enumerate(zip(ps, bufs)):
        g = p.grad
        m.lerp_(g, 1 - mu)
        d = g.lerp(m, mu)
        scale = math.sqrt(max(1.0, p.shape[0] / p.shape[1]))
        with torch.no_grad():
            p.mul_(1 - lr * wd)
            r0 = 0
            for n in splits.get(i, [p.shape[0]]):
                p[r0:r0 + n] -= lr * scale * zeropower_reference(d[r0:r0 + n]).float()
                r0 += n


def _params(seed=0):
    torch.manual_seed(seed)
    return [torch.nn.Parameter(torch.randn(*s) * 0.1) for s in SHAPES]


def test_flat_muon_matches_per_matrix_oracle():
    pa, pb = _params(), _params()
    opt = Muon(pa, lr=0.02, momentum=0.9, weight_decay=0.01, shard=False, splits={pa[k]: v for k, v in SPLITS.items()})
    bufs = [torch.zeros_like(p) for p in pb]
    for step in range(3):
        g = torch.Generator().manual_seed(7 + step)
        for a, b in zip(pa, pb):
            a.grad = torch.randn(a.shape, generator=g)
            b.grad = a.grad.clone()
        opt.step()
        oracle_step(pb, bufs, 0.02, 0.9, 0.01, SPLITS)
    for a, b, m in zip(pa, pb, bufs):
        assert (a.detach() - b.detach()).abs().max() < 2e-3
        assert torch.allclose(opt.momentum_buffer(a), m, atol=1e-6)


def test_layout_buckets_are_contiguous_and_padded():
    ps = _params()
    L = MuonLayout([{"params": ps}], {ps[3]: [32, 32, 32]}, world=3, rank=1, pad=True)
    assert [(b.rows, b.cols, len(b.entries)) for b in L.buckets] == [(64, 32, 2), (32, 96, 1), (32, 32, 3), (48, 48, 1)]
    for b in L.buckets:
        offs = [L.entries[k].off for k in b.entries]
        assert offs == [b.off + j * b.rows * b.cols for j in range(len(offs))]
        assert b.span == 3 * b.per * b.rows * b.cols
    assert [L.entries[k].owner for k in L.buckets[2].entries] == [0, 1, 2]
    assert L.buckets[0].owned_slots(1) == (1, 2) and L.buckets[1].owned_slots(1) == (1, 1)


@pytest.mark.parametrize("mdt", [None, torch.bfloat16])
def test_state_dict_round_trip(mdt):
    pa = _params()
    opt = Muon(pa, lr=0.02, shard=False, splits={pa[3]: [32, 32, 32]}, momentum_dtype=mdt)
    for p in pa:
        p.grad = torch.randn_like(p)
    opt.step()
    sd = opt.state_dict()
    assert all(sd["state"][i]["momentum_buffer"].shape == p.shape for i, p in enumerate(pa))
    pb = _params()
    opt2 = Muon(pb, lr=0.02, shard=False, splits={pb[3]: [32, 32, 32]}, momentum_dtype=mdt)
    opt2.load_state_dict(sd)
    assert opt2.momentum.dtype == (mdt or torch.float32)
    assert torch.equal(opt2.momentum, opt.momentum)
