"""Fused MoE inference (stacked experts, grouped GEMM, routing weight in the epilogue) against the per-expert loop of
a transformers-style MoE block, on CPU (the grouped GEMM's CPU path)."""
import torch
import torch.nn as nn
import torch.nn.functional as F

from trenowanie_generatora_obrazkow_b200.models.moe_infer import FusedMoE, patch_moe_blocks


class _Expert(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.gate_proj, self.up_proj = nn.Linear(h, i, bias=False), nn.Linear(h, i, bias=False)
        self.down_proj = nn.Linear(i, h, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class _Block(nn.Module):
    """The per-expert loop the fused path replaces (softmax top-k, renormalised), plus a shared expert."""

    def __init__(self, h=32, i=48, e=6, k=2):
        super().__init__()
        self.gate = nn.Linear(h, e, bias=False)
        self.experts = nn.ModuleList(_Expert(h, i) for _ in range(e))
        self.shared_experts = _Expert(h, i)
        self.top_k = k

    def forward(self, x):
        x2 = x.reshape(-1, x.shape[-1])
        p = self.gate(x2).float().softmax(-1)
        w, idx = p.topk(self.top_k, -1)
        w = w / w.sum(-1, keepdim=True)
        out = torch.zeros_like(x2)
        for e, ex in enumerate(self.experts):
            for k in range(self.top_k):
                m = idx[:, k] == e
                if m.any():
                    out[m] += w[m, k, None] * ex(x2[m])
        return out.view(x.shape) + self.shared_experts(x)


def test_fused_moe_matches_expert_loop():
    torch.manual_seed(0)
    blk = _Block()
    x = torch.randn(3, 17, 32)
    with torch.no_grad():
        want = blk(x)
        assert patch_moe_blocks(blk) == 1
        got = blk(x)
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()


def test_fused_moe_int8_close():
    torch.manual_seed(1)
    blk = _Block()
    x = torch.randn(40, 32)
    with torch.no_grad():
        want = blk(x) - blk.shared_experts(x)
        got = FusedMoE.from_block(blk, quant="int8")(x)
    assert ((got - want).norm() / want.norm()).item() < 2e-2
