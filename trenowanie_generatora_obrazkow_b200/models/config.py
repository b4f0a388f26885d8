"""Model configurations and named presets.

Field names and defaults of ``DenoiserConfig``, ``TextEncoderConfig`` and ``LMEncoderConfig`` follow the reference
(aurora/model.py:224-276) so that ``asdict(config)`` round-trips through checkpoints written by either framework
(checkpoint keys ``den_config`` / ``te_config``, reference train.py:824-827). The size tables reproduce the
reference presets (aurora/model.py:409-441) and add the shapes of this project's benchmark configurations.
"""
from dataclasses import dataclass, replace


@dataclass
class TextEncoderConfig:
    """From-scratch GQA text encoder with an MLM head tied to the embedding (reference aurora/model.py:224-238)."""
    vocab_size: int = 8192
    dim: int = 384
    depth: int = 6
    heads: int = 6
    kv_heads: int = 2
    head_dim: int = 64
    mlp_hidden: int = 1024
    max_tokens: int = 64
    pad_id: int = 0
    bos_id: int = 2
    eos_id: int = 3
    null_id: int = 4
    mask_id: int = 5


@dataclass
class LMEncoderConfig:
    """Frozen LM states -> trainable refiner (reference aurora/model.py:241-262).

    ``backend`` selects where the frozen states come from: "slayer" / "hf" name the reference's pretrained LMs
    (they need network weights); "states" means the caller passes the (B, L, lm_dim) states directly, which is what
    the synthetic benchmarks do (random N(0, 1) states of the LM's width).
    """
    kind: str = "lm"
    repo: str = "SlayerLab/Slayer149"
    tok_suffix: str = "slayer149"
    lm_dim: int = 768
    skip_last: int = 1
    dim: int = 768
    depth: int = 2
    heads: int = 12
    kv_heads: int = 4
    head_dim: int = 64
    mlp_hidden: int = 2048
    max_tokens: int = 96
    backend: str = "slayer"
    experts: int = 0
    quant: str = ""
    out_dim: int = 0


@dataclass
class DenoiserConfig:
    """adaLN-single DiT on FLUX.2 latents, one token per latent pixel (reference aurora/model.py:265-276)."""
    latent_channels: int = 128
    latent_size: int = 16
    dim: int = 640
    depth: int = 8
    heads: int = 10
    mlp_hidden: int = 1536
    text_dim: int = 384
    latent_layout: str = "flux2_pipeline"
    rope_ref: int = 0
    micro_cond: int = 0

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


def swiglu_hidden(dim: int, mult: float = 8 / 3, multiple: int = 128) -> int:
    """SwiGLU hidden width with the parameter count of a ``4 x dim`` GELU MLP, rounded up to ``multiple``."""
    return -(-int(dim * mult) // multiple) * multiple


SIZES = {
    # reference presets (aurora/model.py:409-429)
    "50m": DenoiserConfig(),
    "116m": DenoiserConfig(dim=768, depth=12, heads=12, mlp_hidden=1792),
    "253m": DenoiserConfig(dim=1024, depth=16, heads=16, mlp_hidden=2432),
    "1b": DenoiserConfig(dim=2048, depth=15, heads=32, mlp_hidden=4864),
    "1.5b": DenoiserConfig(dim=2048, depth=23, heads=32, mlp_hidden=4864),
    "2b": DenoiserConfig(dim=2048, depth=31, heads=32, mlp_hidden=4864),
    "750m": DenoiserConfig(dim=2560, depth=7, heads=20, mlp_hidden=6912),
    "750m-w2048": DenoiserConfig(dim=2048, depth=11, heads=16, mlp_hidden=5504),
    "750m-w1792": DenoiserConfig(dim=1792, depth=15, heads=14, mlp_hidden=4864),
    "750m-w1536": DenoiserConfig(dim=1536, depth=20, heads=12, mlp_hidden=4096),
    "750m-w1280": DenoiserConfig(dim=1280, depth=30, heads=10, mlp_hidden=3456),
    "1.6b": DenoiserConfig(dim=2560, depth=15, heads=20, mlp_hidden=6912),
    "2.4b": DenoiserConfig(dim=2560, depth=23, heads=20, mlp_hidden=6912),
    # the released HomeIMG 1.24B (preset 750m at depth 12, refiner 1280 x 4)
    "1.24b-homeimg": DenoiserConfig(dim=2560, depth=12, heads=20, mlp_hidden=6912, text_dim=1280),
    # benchmark shapes: hidden 2048, 24 blocks, 16 heads of 128, "MLP 4x" as a parameter-matched SwiGLU
    # (8/3 x 2048 -> 5504), text width 1024 (refiner at half the width)
    "1.24b": DenoiserConfig(dim=2048, depth=24, heads=16, mlp_hidden=swiglu_hidden(2048), text_dim=1024,
                            latent_size=32),
    # the CPU test DiT: hidden 576, 12 blocks, 9 heads, MLP 4x (SwiGLU 1536), 256 tokens
    "tiny": DenoiserConfig(dim=576, depth=12, heads=9, mlp_hidden=swiglu_hidden(576), text_dim=576, latent_size=16),
    # a few-MB model for smoke runs and multi-process CPU tests of the entry points
    "nano": DenoiserConfig(dim=128, depth=4, heads=2, mlp_hidden=384, text_dim=128, latent_size=8),
    # the MoE benchmark backbone is "1.24b" with every other MLP replaced by experts (models/moe.py)
    # the 4B OPD teacher: hidden 3072, 32 blocks, 24 heads of 128
    "teacher-4b": DenoiserConfig(dim=3072, depth=32, heads=24, mlp_hidden=swiglu_hidden(3072), text_dim=1024,
                                 latent_size=32),
}


TE_SIZES = {
    "13m": TextEncoderConfig(),
    "27m": TextEncoderConfig(dim=512, depth=8, heads=8, kv_heads=2, head_dim=64, mlp_hidden=1408),
    "slayer149": LMEncoderConfig(),
    "poziomka": LMEncoderConfig(repo="cpral/Poziomka-Baza-2026-09-05", tok_suffix="poziomka", lm_dim=2048,
                                skip_last=0, max_tokens=256, backend="hf", experts=8),
    # synthetic frozen-LM states of width 1024 (128 tokens) -> 2-block refiner (benchmark configurations)
    "states1024": LMEncoderConfig(repo="", tok_suffix="", lm_dim=1024, skip_last=0, dim=1024, depth=2, heads=16,
                                  kv_heads=4, head_dim=64, mlp_hidden=2816, max_tokens=128, backend="states"),
    "states-nano": LMEncoderConfig(repo="", tok_suffix="", lm_dim=64, skip_last=0, dim=128, depth=1, heads=2,
                                   kv_heads=1, head_dim=64, mlp_hidden=384, max_tokens=16, backend="states"),
    "states1024-64": LMEncoderConfig(repo="", tok_suffix="", lm_dim=1024, skip_last=0, dim=576, depth=2, heads=9,
                                     kv_heads=3, head_dim=64, mlp_hidden=1536, max_tokens=64, backend="states"),
}


def refiner_shape(dim: int):
    """Refiner shape for a width: heads of 64, GQA with >= 3 query heads per kv head, SwiGLU 8/3 x dim
    (reference aurora/model.py:458-462)."""
    assert dim % 64 == 0, "refiner width must be a multiple of 64 (heads of 64)"
    heads = dim // 64
    kv_heads = max(d for d in range(1, max(1, heads // 3) + 1) if heads % d == 0)
    return dict(dim=dim, heads=heads, kv_heads=kv_heads, mlp_hidden=swiglu_hidden(dim))


def make_configs(size: str, te_size: str, te_dim: int = None, te_depth: int = None, depth: int = None,
                 te_experts: int = None, te_quant: str = None):
    """(denoiser config, text encoder config) for presets; te_dim / te_depth resize an LM refiner
    (reference aurora/model.py:444-464)."""
    te_cfg = TE_SIZES[te_size]
    if te_experts:
        assert getattr(te_cfg, "backend", "") == "hf", "--te-experts only applies to MoE LM encoders"
        te_cfg = replace(te_cfg, experts=te_experts)
    if te_quant is not None:
        assert getattr(te_cfg, "backend", "") == "hf", "--te-quant only applies to MoE LM encoders"
        te_cfg = replace(te_cfg, quant=te_quant)
    if te_dim or te_depth:
        assert isinstance(te_cfg, LMEncoderConfig), "--te-dim / --te-depth only apply to LM text encoders"
        shape = refiner_shape(te_dim or te_cfg.dim)
        te_cfg = replace(te_cfg, depth=te_depth or te_cfg.depth, **shape)
    den_cfg = replace(SIZES[size], text_dim=getattr(te_cfg, "out_dim", 0) or te_cfg.dim)
    return (replace(den_cfg, depth=depth) if depth else den_cfg), te_cfg


def te_config_from_dict(d):
    """Checkpoints from before te_config existed used the released text encoder. Keys that are not config fields
    (an export's packed-LM description: lm_arch, lm_blocks, ...) are ignored."""
    cls = LMEncoderConfig if d.get("kind") == "lm" else TextEncoderConfig
    return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


def configs_from_ckpt(ck):
    return DenoiserConfig(**ck["den_config"]), te_config_from_dict(ck.get("te_config", {}))


def benchmark_configs(name: str):
    """Named benchmark configurations -> (denoiser config, text encoder config)."""
    if name == "1.24b":
        return SIZES["1.24b"], TE_SIZES["states1024"]
    if name == "tiny":
        return SIZES["tiny"], TE_SIZES["states1024-64"]
    if name == "1.24b-homeimg":
        return SIZES["1.24b-homeimg"], replace(TE_SIZES["states1024"], lm_dim=2048, max_tokens=256,
                                               depth=4, **refiner_shape(1280))
    if name == "teacher-4b":
        return SIZES["teacher-4b"], TE_SIZES["states1024"]
    raise KeyError(name)
