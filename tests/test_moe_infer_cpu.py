"""Fused MoE inference (stacked experts, grouped GEMM, routing weight in the epilogue) against the per-expert loop of
a transformers-style MoE block, on CPU (the grouped GEMM's CPU path)."""
import pytest
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


def _tiny_qwen3_moe():
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM
    cfg = Qwen3MoeConfig(vocab_size=128, hidden_size=64, intermediate_size=128, moe_intermediate_size=32,
                         num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2, head_dim=16, num_experts=4,
                         num_experts_per_tok=2, decoder_sparse_step=1, max_position_embeddings=64)
    torch.manual_seed(3)
    m = Qwen3MoeForCausalLM(cfg).eval()
    with torch.no_grad():
        for p in m.parameters():  # the init leaves some tensors at zero (routers, experts): give every one values
            p.add_(0.05 * torch.randn_like(p))
    return m


def test_fused_moe_patches_transformers5_fused_experts():
    """transformers 5 keeps a block's experts as one module with stacked gate_up_proj / down_proj tensors and a
    top-k router module; the patched forward matches the library's per-expert loop."""
    pytest.importorskip("transformers")
    m = _tiny_qwen3_moe()
    ids = torch.randint(0, 128, (2, 11))
    with torch.no_grad():
        want = m.model(input_ids=ids).last_hidden_state
        assert patch_moe_blocks(m.model) == 3
        got = m.model(input_ids=ids).last_hidden_state
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()


def test_hf_frozen_lm_loads_a_local_model(tmp_path):
    """HFFrozenLM (models/frozen_lm.py): a local transformers causal LM directory, the last layers skipped, MoE
    blocks fused; states equal the library model's truncated forward."""
    pytest.importorskip("transformers")
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD, HFFrozenLM
    m = _tiny_qwen3_moe()
    m.save_pretrained(str(tmp_path / "lm"))
    lm = HFFrozenLM(str(tmp_path / "lm"), skip_last=1, device="cpu")
    assert len(lm.model.layers) == 2
    ids = torch.randint(0, 128, (2, 9))
    ids[1, 6:] = LM_PAD
    ref = m.model.to(torch.bfloat16)
    ref.layers = ref.layers[:2]
    with torch.no_grad():
        want = ref(input_ids=ids.masked_fill(ids.eq(LM_PAD), 0)).last_hidden_state.float()
        got = lm.states(ids).float()
    assert got.shape == (2, 9, 64)
    assert ((got - want).norm() / want.norm()).item() < 3e-2


class _SelfRoutingBlock(nn.Module):
    """DeepSeek / Bailing-style block: its forward routes (sigmoid scores, group-limited top-k, scaled weights: a
    routing FusedMoE does not reimplement) and calls moe_infer for the experts."""

    def __init__(self, E=6, H=32, I=16, k=2):
        super().__init__()
        self.gate = nn.Linear(H, E, bias=False)
        self.experts = nn.ModuleList(_Expert(H, I) for _ in range(E))
        self.k, self.groups = k, 2

    def forward(self, x):
        x2 = x.reshape(-1, x.shape[-1])
        s = torch.sigmoid(self.gate(x2).float())
        g = s.view(len(x2), self.groups, -1).amax(-1)                 # best score per expert group
        keep = g.topk(1, dim=-1).indices                                # one group per token
        mask = torch.zeros_like(g).scatter_(1, keep, 1).repeat_interleave(s.shape[1] // self.groups, 1)
        w, idx = (s * mask).topk(self.k, dim=-1)
        w = 2.5 * w / w.sum(-1, keepdim=True)
        return self.moe_infer(x2, idx, w).view(x.shape)

    def moe_infer(self, x, idx, w):
        out = torch.zeros_like(x)
        for m in range(len(x)):
            for j in range(idx.shape[1]):
                out[m] += w[m, j] * self.experts[int(idx[m, j])](x[m])
        return out


def test_fused_moe_keeps_the_blocks_own_routing():
    torch.manual_seed(4)
    blk = _SelfRoutingBlock()
    x = torch.randn(2, 9, 32)
    with torch.no_grad():
        want = blk(x)
        assert patch_moe_blocks(blk) == 1
        assert len(blk.experts) == 6 and not isinstance(blk.experts, nn.ModuleList)  # per-expert modules dropped
        got = blk(x)
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()


def test_transformers5_compat_and_rope_refresh():
    """Shims for transformers-4 remote code: the "default" RoPE init reads theta / partial factor also from the
    rope dicts; RoPE buffers left uninitialised by meta-device loading are recomputed from the init function."""
    pytest.importorskip("transformers")
    import types

    import transformers.modeling_rope_utils as rope_utils
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import refresh_rope_buffers, transformers5_compat
    transformers5_compat()
    import transformers.utils.import_utils as import_utils
    assert import_utils.is_torch_fx_available() is False
    cfg = types.SimpleNamespace(hidden_size=64, num_attention_heads=4, head_dim=None, rope_theta=None,
                                partial_rotary_factor=None, rope_scaling={"rope_theta": 5000.0,
                                                                          "partial_rotary_factor": 0.5})
    inv, scale = rope_utils.ROPE_INIT_FUNCTIONS["default"](cfg, "cpu")
    want = 1.0 / 5000.0 ** (torch.arange(0, 8, 2).float() / 8)
    assert scale == 1.0 and torch.allclose(inv, want)
    class Rotary(nn.Module):  # a transformers-4 style rotary module (what old remote code builds)
        def __init__(self, config):
            super().__init__()
            self.config, self.rope_init_fn = config, rope_utils.ROPE_INIT_FUNCTIONS["default"]
            inv, self.attention_scaling = self.rope_init_fn(config, None)
            self.register_buffer("inv_freq", torch.full_like(inv, float("nan")), persistent=False)  # "uninitialised"
            self.original_inv_freq = self.inv_freq

    m = nn.Sequential(nn.Linear(4, 4), Rotary(cfg))
    assert refresh_rope_buffers(m) == 1
    assert torch.allclose(m[1].inv_freq, want) and torch.allclose(m[1].original_inv_freq, want)
