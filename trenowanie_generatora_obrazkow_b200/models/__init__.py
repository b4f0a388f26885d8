"""Models: DiT denoiser, text encoders / refiner, configs, MoE variant."""
from .config import (SIZES, TE_SIZES, DenoiserConfig, LMEncoderConfig, TextEncoderConfig, benchmark_configs,
                     configs_from_ckpt, make_configs, te_config_from_dict)
from .dit import Denoiser
from .text import LMTextEncoder, TextEncoder, build_text_encoder


def build_models(den_cfg=DenoiserConfig(), te_cfg=TextEncoderConfig(), device=None):
    """(text encoder, denoiser), initialised (reference aurora/model.py:476-487)."""
    te_out = getattr(te_cfg, "out_dim", 0) or te_cfg.dim
    assert den_cfg.text_dim == te_out, f"denoiser text_dim {den_cfg.text_dim} != text encoder output {te_out}"
    te = build_text_encoder(te_cfg)
    den = Denoiser(den_cfg)
    te.init_weights()
    den.init_weights()
    if device is not None:
        te.to(device)
        den.to(device)
    return te, den
