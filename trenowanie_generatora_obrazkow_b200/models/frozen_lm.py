"""Frozen language-model backends that turn caption token ids into the hidden states the refiner consumes.

The reference runs a frozen pretrained LM (SlayerLab/Slayer149 GPT or the Poziomka MoE through transformers,
aurora/slayer.py:30-146, :238-432) on each caption batch, outside the trainable parameters. Backends here:

* ``slayer`` the Slayer GPT (models/slayer.py) from a local directory (config.json + model.safetensors): the
             residual stream after ``n_layer - skip_last`` blocks, as the reference's LMTextEncoder reads it.
* ``hf``     a transformers causal LM loaded from a local directory (``cfg.repo`` must be a path or a cached
             model id; there is no network on the training boxes): first ``num_layers - skip_last`` layers (the
             others are never loaded), bf16, SDPA attention, the last hidden state; MoE blocks fused
             (models/moe_infer.py). Remote code written for transformers 4 (the Poziomka BailingMoeV2 model) runs
             under transformers 5 through ``transformers5_compat`` (reference aurora/hf_compat.py:21-59).
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


def _rope_inv_freq(config, device=None):
    """Plain RoPE inverse frequencies theta^(-2i / d), i < d / 2, with d = head_dim * partial_rotary_factor; theta and
    the factor are read from the config, or from the rope_scaling / rope_parameters dicts where transformers 5 keeps
    them. Returns (inv_freq, attention scaling 1.0), the signature of transformers' RoPE init functions."""
    extra = {}
    for name in ("rope_parameters", "rope_scaling"):
        d = getattr(config, name, None)
        if isinstance(d, dict):
            extra.update(d)
    theta = getattr(config, "rope_theta", None) or extra.get("rope_theta", 10000.0)
    factor = getattr(config, "partial_rotary_factor", None) or extra.get("partial_rotary_factor", 1.0)
    head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    dim = int(head_dim * factor)
    exponents = torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim
    return 1.0 / (float(theta) ** exponents), 1.0


def transformers5_compat():
    """Let transformers-4 remote code run under transformers 5 (idempotent): the removed
    ``import_utils.is_torch_fx_available`` answers False, and RoPE init type "default" (gone from
    ``ROPE_INIT_FUNCTIONS``) is the plain rotary embedding of ``_rope_inv_freq``."""
    import transformers.modeling_rope_utils as rope_utils
    import transformers.utils.import_utils as import_utils
    if not hasattr(import_utils, "is_torch_fx_available"):
        import_utils.is_torch_fx_available = lambda: False
    if "default" not in rope_utils.ROPE_INIT_FUNCTIONS:
        rope_utils.ROPE_INIT_FUNCTIONS["default"] = lambda config, device=None, *a, **k: _rope_inv_freq(config, device)


def refresh_rope_buffers(model, device=None):
    """Models are built on the meta device and loaded from weights, so a RoPE module's non-persistent ``inv_freq``
    buffer (not in the checkpoint) may hold uninitialised memory: recompute it from the module's own init function.
    Returns the number of modules refreshed."""
    n = 0
    for mod in model.modules():
        fn = getattr(mod, "rope_init_fn", None)
        if callable(fn) and isinstance(getattr(mod, "inv_freq", None), torch.Tensor):
            dev = device if device is not None else mod.inv_freq.device
            inv, scale = fn(mod.config, dev)
            mod.inv_freq = inv
            if hasattr(mod, "original_inv_freq"):
                mod.original_inv_freq = inv
            mod.attention_scaling = scale
            n += 1
    return n


class HFFrozenLM:
    """fused_moe: the LM's mixture-of-experts blocks run as stacked experts + grouped GEMMs (models/moe_infer.py),
    optionally with int8 expert weights (quant="int8")."""

    def __init__(self, repo, skip_last=0, device=None, fused_moe=True, quant=""):
        from transformers import AutoConfig, AutoModelForCausalLM
        transformers5_compat()
        cfg = AutoConfig.from_pretrained(repo, trust_remote_code=True, local_files_only=True)
        keep = cfg.num_hidden_layers - skip_last
        model = AutoModelForCausalLM.from_pretrained(repo, dtype=torch.bfloat16, trust_remote_code=True,
                                                     local_files_only=True, attn_implementation="sdpa",
                                                     num_hidden_layers=keep)
        self.model = model.model.to(device).eval().requires_grad_(False)
        refresh_rope_buffers(self.model)
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
