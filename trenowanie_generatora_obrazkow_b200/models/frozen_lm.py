"""Frozen language-model backends that turn caption token ids into the hidden states the refiner consumes.

The reference runs a frozen pretrained LM (SlayerLab/Slayer149 GPT or the Poziomka MoE through transformers,
aurora/slayer.py:30-146, :238-432) on each caption batch, outside the trainable parameters. Backends here:

* ``slayer`` the Slayer GPT (models/slayer.py) from a local directory (config.json + model.safetensors): the
             residual stream after ``n_layer - skip_last`` blocks, as the reference's LMTextEncoder reads it.
* ``hf``     a transformers causal LM loaded from a local directory (``cfg.repo`` must be a path or a cached
             model id; there is no network on the training boxes): first ``num_layers - skip_last`` layers, bf16,
             the last hidden state.
* ``random`` a fixed random embedding table of the LM's width (seeded): stands in for a pretrained LM in smoke
             runs and tests where no weights exist. Rows of PAD / NULL ids get zeros.
* ``states`` none: the caller passes states directly (the synthetic benchmarks).
The LM is never registered as a submodule, so it stays out of state dicts, optimizers and gradient reduction.
"""
import torch

LM_PAD, LM_NULL = 65535, 65534


class RandomFrozenLM:
    def __init__(self, lm_dim, vocab=65536, seed=0, device=None, dtype=torch.bfloat16):
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.table = torch.randn(vocab, lm_dim, generator=g).to(device=device, dtype=dtype)

    def to(self, device):
        self.table = self.table.to(device)
        return self

    @torch.no_grad()
    def states(self, ids):
        special = ids.eq(LM_PAD) | ids.eq(LM_NULL)
        h = self.table[ids.clamp(max=self.table.shape[0] - 1).masked_fill(special, 0)]
        return h.masked_fill(special[..., None], 0)


class HFFrozenLM:
    """fused_moe: the LM's mixture-of-experts blocks run as stacked experts + grouped GEMMs (models/moe_infer.py),
    optionally with int8 expert weights (quant="int8")."""

    def __init__(self, repo, skip_last=0, device=None, fused_moe=True, quant=""):
        from transformers import AutoModelForCausalLM
        model = AutoModelForCausalLM.from_pretrained(repo, torch_dtype=torch.bfloat16, trust_remote_code=True,
                                                     local_files_only=True)
        layers = model.model.layers
        keep = len(layers) - skip_last
        model.model.layers = layers[:keep]
        self.model = model.model.to(device).eval().requires_grad_(False)
        if fused_moe:
            from .moe_infer import patch_moe_blocks
            patch_moe_blocks(self.model, quant=quant)

    def to(self, device):
        self.model.to(device)
        return self

    @torch.no_grad()
    def states(self, ids):
        real = ids.masked_fill(ids.eq(LM_PAD) | ids.eq(LM_NULL), 0)
        return self.model(input_ids=real, use_cache=False).last_hidden_state


class SlayerFrozenLM:
    """packed: on CUDA, captions run packed without padding (varlen causal attention) up to max_tokens real tokens
    per LM call; null-prompt rows are not run (zeros), as the refiner replaces them by its learned null vector."""

    def __init__(self, repo, skip_last=0, device=None, model=None, dtype=torch.bfloat16, packed=None,
                 max_tokens=8192):
        from .slayer import load_gpt
        self.model = model if model is not None else load_gpt(repo)[0]
        self.model = self.model.to(device=device, dtype=dtype).eval().requires_grad_(False)
        self.n_blocks = len(self.model.blocks) - skip_last
        self.packed, self.max_tokens = packed, max_tokens

    def to(self, device):
        self.model.to(device)
        return self

    @torch.no_grad()
    def states(self, ids):
        packed = self.packed if self.packed is not None else self.model.tok.weight.is_cuda
        if packed:
            return self.states_packed(ids)
        real = ids.masked_fill(ids.eq(LM_PAD) | ids.eq(LM_NULL), 0).long()
        return self.model.hidden(real, self.n_blocks)

    @torch.no_grad()
    def states_packed(self, ids):
        """(B, T) caption rows -> (B, T, n_embd) states; zeros at pads and null-prompt rows."""
        return packed_states(lambda seqs: self.model.hidden_packed(seqs, self.n_blocks), ids,
                             self.model.cfg.n_embd, self.max_tokens, self.model.tok.weight.dtype)


def packed_states(run, ids, width, max_tokens=8192, dtype=torch.bfloat16):
    """Scatter the packed LM states of the real tokens of the real (non-null) rows of ids back into (B, T, width).
    run(list of 1-D CPU id tensors) -> (sum of lengths, width); calls are cut at max_tokens real tokens."""
    B, T = ids.shape
    ids_c = ids.cpu()
    keep = ids_c.ne(LM_PAD) & ids_c[:, :1].ne(LM_NULL)
    lens = keep.sum(1)
    seqs = [q for q in ids_c[keep].split(lens.tolist()) if len(q)]
    out = torch.zeros(B * T, width, device=ids.device, dtype=dtype)
    if seqs:
        flat, pack, n = [], [], 0
        for q in seqs + [None]:
            if q is None or (pack and n + len(q) > max_tokens):
                flat.append(run(pack))
                pack, n = [], 0
            if q is not None:
                pack.append(q)
                n += len(q)
        out.index_copy_(0, keep.flatten().nonzero().flatten().to(ids.device), torch.cat(flat).to(out.device, dtype))
    return out.view(B, T, width)


def build_frozen_lm(cfg, device=None, allow_random=False):
    backend = getattr(cfg, "backend", "states")
    if backend == "states":
        return None
    if backend == "random" or allow_random:
        try:
            if backend == "hf":
                return HFFrozenLM(cfg.repo, cfg.skip_last, device)
            if backend == "slayer":
                return SlayerFrozenLM(cfg.repo, cfg.skip_last, device)
        except Exception:
            if not allow_random:
                raise
        return RandomFrozenLM(cfg.lm_dim, device=device)
    if backend == "hf":
        return HFFrozenLM(cfg.repo, cfg.skip_last, device, quant=getattr(cfg, "quant", ""))
    if backend == "slayer":
        return SlayerFrozenLM(cfg.repo, cfg.skip_last, device)
    raise RuntimeError(f"frozen LM backend {backend!r} needs pretrained weights that are not available offline; "
                       "use --te-size 13m / 27m, synthetic states, or --random-lm for a smoke run")
