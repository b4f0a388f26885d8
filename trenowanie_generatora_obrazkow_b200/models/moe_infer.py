"""Fused MoE inference for the frozen caption LM's mixture-of-experts layers (reference aurora/hf_compat.py:62-169,
which replaces the transformers per-expert loop with stacked weights and a Triton grouped GEMM).

``FusedMoE`` holds the experts stacked: gate and up projections as one (E, 2I, H) weight (one GEMM computes both),
down projections as (E, H, I), optionally int8 with a per-(expert, output column) scale, dequantised per call.
A forward: router logits in fp32 -> top-k -> assignments sorted by expert (stable) -> token rows gathered in that
order -> grouped GEMM (gate | up) -> SwiGLU -> grouped GEMM (down) with the routing weight as a per-row epilogue
scale -> rows summed back per token. The grouped GEMM's tile schedule comes from the expert offsets on the device
(ops/gemm.py:gemm_grouped), so there is no host synchronisation and one launch per projection, whatever the
routing.

``patch_moe_blocks(model)`` finds transformers-style MoE blocks and replaces their forward (or, for blocks that route
themselves and call ``moe_infer(x, topk_ids, topk_weight)``, only that method). Two expert layouts:
an ``experts`` list of gate_proj / up_proj / down_proj MLPs (transformers 4), or one fused ``experts`` module
holding ``gate_up_proj`` (E, 2I, H; gate rows first) and ``down_proj`` (E, H, I) tensors with a ``gate`` router module
carrying ``weight``, ``top_k`` and ``norm_topk_prob`` (transformers 5). Shared experts: ``shared_experts`` (added),
or ``shared_expert`` scaled by ``sigmoid(shared_expert_gate(x))``.
"""
import torch
import torch.nn.functional as F

from ..ops import fused as Fz
from ..ops.gemm import gemm_grouped


def _quant_int8(w):
    """Per-(expert, output row) symmetric int8: w (E, N, K) -> (int8 (E, N, K), scale (E, N))."""
    s = w.float().abs().amax(-1).clamp(min=1e-8) / 127.0
    return (w.float() / s[..., None]).round().clamp(-127, 127).to(torch.int8), s


class FusedMoE:
    def __init__(self, router_w, gate_up, down, top_k, norm_topk=True, quant=""):
        self.router_w = router_w.float()
        self.E, self.k, self.norm = router_w.shape[0], top_k, norm_topk
        self.quant = quant
        if quant == "int8":
            self.gu, self.gu_s = _quant_int8(gate_up)
            self.dn, self.dn_s = _quant_int8(down)
        else:  # bf16 once on a GPU (to()), the given precision on the CPU
            self.gu, self.dn = gate_up, down

    @classmethod
    def from_block(cls, block, top_k=None, norm_topk=None, quant=""):
        ex, gate = block.experts, block.gate
        if _fused_experts(ex):
            gate_up, down = ex.gate_up_proj.detach(), ex.down_proj.detach()
        else:
            gate_up = torch.stack([torch.cat([e.gate_proj.weight, e.up_proj.weight], 0) for e in ex]).detach()
            down = torch.stack([e.down_proj.weight for e in ex]).detach()
        cfg = getattr(block, "config", None)
        k = top_k or getattr(block, "top_k", None) or getattr(gate, "top_k", None) or \
            getattr(cfg, "num_experts_per_tok", 2)
        norm = norm_topk
        if norm is None:
            norm = getattr(gate, "norm_topk_prob", None)
        if norm is None:
            norm = getattr(cfg, "norm_topk_prob", True)
        return cls(gate.weight.detach(), gate_up, down, int(k), bool(norm), quant)

    def to(self, device):
        cuda = torch.device(device).type == "cuda"
        for name in ("router_w", "gu", "dn", "gu_s", "dn_s"):
            if hasattr(self, name):
                t = getattr(self, name).to(device)
                if cuda and name in ("gu", "dn") and t.is_floating_point():
                    t = t.to(torch.bfloat16)
                setattr(self, name, t)
        return self

    def _weights(self):
        if self.quant == "int8":
            return ((self.gu.float() * self.gu_s[..., None]).to(torch.bfloat16),
                    (self.dn.float() * self.dn_s[..., None]).to(torch.bfloat16))
        return self.gu, self.dn

    def route(self, x):
        probs = F.linear(x.float(), self.router_w).softmax(-1)
        w, idx = probs.topk(self.k, dim=-1)
        if self.norm:
            w = w / w.sum(-1, keepdim=True)
        return w, idx

    @torch.no_grad()
    def __call__(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        w, idx = self.route(x2)
        return self.combine(x2, idx, w).view(shape)

    @torch.no_grad()
    def combine(self, x2, idx, w):
        """The expert part for a given routing: x2 (N, H), idx / w (N, k) expert ids and weights -> (N, H)."""
        shape = x2.shape
        N, k = idx.shape
        flat = idx.reshape(-1)
        order = flat.argsort(stable=True)
        tok = order // k
        counts = torch.bincount(flat, minlength=self.E)
        offsets = torch.zeros(self.E + 1, dtype=torch.int32, device=x2.device)
        offsets[1:] = counts.cumsum(0)
        xs = x2.to(torch.bfloat16 if x2.is_cuda else torch.float32)[tok]
        gu, dn = (w_.to(xs.dtype) for w_ in self._weights())
        ab = gemm_grouped(xs, gu, offsets)
        h = Fz.swiglu(ab)
        y = gemm_grouped(h.to(xs.dtype), dn, offsets, row_scale=w.reshape(-1)[order])
        out = torch.zeros(N, shape[-1], dtype=torch.float32, device=x2.device)
        out.index_add_(0, tok, y.float())
        return out.to(x2.dtype)


def _fused_experts(ex):
    return isinstance(getattr(ex, "gate_up_proj", None), torch.Tensor) and \
        isinstance(getattr(ex, "down_proj", None), torch.Tensor)


def _expert_list(ex):
    try:
        items = list(ex)
    except TypeError:
        return False
    return len(items) > 0 and all(hasattr(e, a) for e in items for a in ("gate_proj", "up_proj", "down_proj"))


def patch_moe_blocks(model, quant=""):
    """Replace the forward of every transformers-style MoE block of ``model`` by FusedMoE (+ its shared experts).
    Returns the number of blocks patched."""
    n = 0
    for mod in list(model.modules()):
        ex = getattr(mod, "experts", None)
        gate = getattr(mod, "gate", None)
        if ex is None or gate is None or not isinstance(getattr(gate, "weight", None), torch.Tensor):
            continue
        if not (_fused_experts(ex) or _expert_list(ex)):
            continue
        fused = FusedMoE.from_block(mod, quant=quant).to(gate.weight.device)
        if callable(getattr(mod, "moe_infer", None)) and _expert_list(ex):
            # DeepSeek / Bailing-style block: its forward routes (grouped top-k, scaling, ...) and then calls
            # moe_infer(x, topk_ids, topk_weight) for the experts: only that part is replaced, the routing stays
            # the model's own; the per-expert modules are dropped (the stacked weights replace them)
            def moe_infer(x, topk_ids, topk_weight, _f=fused):
                x2 = x.reshape(-1, x.shape[-1])
                n = x2.shape[0]
                return _f.combine(x2, topk_ids.reshape(n, -1), topk_weight.reshape(n, -1)).to(x.dtype)
            mod.moe_infer = moe_infer
            del mod.experts  # a registered child module: removed before a plain attribute can take the name
            mod.experts = list(range(fused.E))  # len(self.experts) keeps working for the block's own code
            mod._fused_moe = fused
            n += 1
            continue
        shared = getattr(mod, "shared_experts", None)
        shared_one = getattr(mod, "shared_expert", None)
        shared_gate = getattr(mod, "shared_expert_gate", None)

        def forward(hidden_states, *a, _f=fused, _s=shared, _s1=shared_one, _g=shared_gate, **k):
            out = _f(hidden_states)
            if _s is not None:
                out = out + _s(hidden_states)
            if _s1 is not None:
                y = _s1(hidden_states)
                out = out + (torch.sigmoid(_g(hidden_states)) * y if _g is not None else y)
            return out
        mod.forward = forward
        mod._fused_moe = fused
        n += 1
    return n
