"""Checkpoint <-> self-contained export directory in the diffusers repository layout.

Behaviour of the reference (export.py:28-161, import_homeimg.py:18-67, homeimg_loader.py:13-48): the EMA weights
(or the live ones) of a training checkpoint become

    model_index.json                      pipeline class + one entry per component
    transformer/config.json               the denoiser config (dataclass fields) + the default time shift
    transformer/diffusion_pytorch_model.safetensors
    text_encoder/config.json              the text encoder / refiner config (+ "kind")
    text_encoder/diffusion_pytorch_model.safetensors
    scheduler/scheduler_config.json       Euler flow-matching schedule: shift, shift_ref, steps
    pipeline.py                           the classes model_index.json names (loaded by homeimg_loader.py)
    tokenizer/                            copied when a local tokenizer.json is given
    vae/                                  copied when a local FLUX.2 VAE directory is given

Parameter names are the reference's own (the modules keep its names), so the transformer / text-encoder
safetensors of an export load into the reference's modules and vice versa. The frozen language model is not packed:
this framework's LM backends are a random-init stand-in or a local Hugging Face directory (``LMEncoderConfig.repo``),
recorded in text_encoder/config.json. ``export_to_init`` turns an export back into an ``--init`` checkpoint (weights
as both live and EMA, validated against freshly built modules), like import_homeimg.py.
"""
import json
import os
import shutil
from dataclasses import asdict

import torch

PIPELINE_CLASS = "HomeIMGPipeline"

# The export's own code module: model_index.json names its components as ("pipeline", class), so the directory
# carries a pipeline.py defining them. Here they are this framework's classes under the exported names; the loader
# (homeimg_loader.py) imports the file under a name unique to the export.
PIPELINE_SOURCE = '''"""Code of a HomeIMG export: the classes that model_index.json names, provided by the
trenowanie_generatora_obrazkow_b200 package."""
from trenowanie_generatora_obrazkow_b200.models.dit import Denoiser as AuroraDenoiser
from trenowanie_generatora_obrazkow_b200.models.text import LMTextEncoder as AuroraLMTextEncoder
from trenowanie_generatora_obrazkow_b200.models.text import TextEncoder as AuroraTextEncoder
from trenowanie_generatora_obrazkow_b200.sampling.pipeline import HomeIMGPipeline as _Pipeline


class EulerFlowMatch(dict):
    """The Euler flow-matching schedule of scheduler/scheduler_config.json (shift, shift_ref)."""


class HomeIMGPipeline(_Pipeline):
    """Text -> image pipeline over this export directory (``HomeIMGPipeline.from_pretrained(root)``)."""
'''


def _write_json(path, obj):
    with open(path, "w") as f:
        json.dump(obj, f, indent=2)


def _lm_pack(te_cfg, lm_dir):
    """The frozen Slayer LM blocks a refiner reads (token embedding + the first n_layer - skip_last blocks, fp32)
    as ``lm.``-prefixed tensors, the text_encoder config fields that describe them, and the LM's tokenizer.json path
    (the layout of the reference's exports, export.py:28-52, so such exports load in either framework)."""
    from ..models.frozen_lm import LM_NULL, LM_PAD
    from ..models.slayer import load_gpt
    gpt, tok_json = load_gpt(lm_dir)
    g = gpt.cfg
    if not (g.pos == "rope" and g.ffn == "swiglu" and g.norm == "rmsnorm"):
        raise ValueError("only rope / swiglu / rmsnorm Slayer LMs can be packed into an export")
    n = g.n_layer - te_cfg.skip_last
    tensors = {}
    for k, v in gpt.state_dict().items():
        if k == "tok.weight" or (k.startswith("blocks.") and int(k.split(".")[1]) < n):
            tensors["lm." + k] = v.detach().float().contiguous()
    fields = dict(kind="lm", lm_arch="slayer", vocab_size=g.vocab, lm_blocks=n, lm_dim=g.n_embd, lm_heads=g.n_head,
                  lm_ffn_mult=g.ffn_mult, lm_norm_eps=g.norm_eps, lm_rope_theta=g.rope_theta,
                  lm_value_residual=bool(g.value_residual), lm_qk_norm=bool(g.qk_norm), pad_id=LM_PAD, null_id=LM_NULL)
    return tensors, fields, tok_json if os.path.exists(tok_json) else None


def packed_lm(te_json, tensors, device=None):
    """A SlayerFrozenLM rebuilt from an export's packed ``lm.`` tensors (None when the export packs none)."""
    if te_json.get("lm_arch") != "slayer" or not any(k.startswith("lm.") for k in tensors):
        return None
    from ..models.frozen_lm import SlayerFrozenLM
    from ..models.slayer import GPT, GPTConfig
    cfg = GPTConfig(vocab=te_json["vocab_size"], n_layer=te_json["lm_blocks"], n_embd=te_json["lm_dim"],
                    n_head=te_json["lm_heads"], norm_eps=te_json["lm_norm_eps"], rope_theta=te_json["lm_rope_theta"],
                    ffn_mult=te_json["lm_ffn_mult"], value_residual=te_json["lm_value_residual"],
                    qk_norm=te_json["lm_qk_norm"])
    gpt = GPT(cfg)
    lm_sd = {k[3:]: v for k, v in tensors.items() if k.startswith("lm.")}
    missing, _ = gpt.load_state_dict(lm_sd, strict=False)
    if any(m.startswith(("tok.", "blocks.")) for m in missing):
        raise ValueError(f"packed LM is incomplete: {missing[:4]}")
    return SlayerFrozenLM(None, skip_last=0, device=device, model=gpt, dtype=torch.float32)


def export_checkpoint(ck, out_dir, use_ema=True, time_shift=None, time_shift_ref=None, vae_dir=None,
                      tokenizer_json=None, lm_dir=None):
    """Write the export of checkpoint dict ``ck`` (a loaded latest.pt / snap / merged file) into ``out_dir``.
    lm_dir: a local Slayer LM directory whose used blocks are packed into text_encoder/ (LM-encoder checkpoints),
    making the export self-contained."""
    from safetensors.torch import save_file

    from ..models import build_models, configs_from_ckpt
    from . import checkpoint as C
    den_cfg, te_cfg = configs_from_ckpt(ck)
    te, den = build_models(den_cfg, te_cfg)
    C.load_weights(ck, te, den)
    used_ema = bool(use_ema and ck.get("ema"))
    if used_ema:
        C.load_weights(ck, te, den, use_ema=True)
    targs = ck.get("args", {}) or {}
    shift = float(time_shift if time_shift is not None else targs.get("t_shift", 1.0))
    shift_ref = float(time_shift_ref if time_shift_ref is not None else (targs.get("t_shift_ref", 0) or 0))
    for sub in ("transformer", "text_encoder", "scheduler"):
        os.makedirs(os.path.join(out_dir, sub), exist_ok=True)
    save_file({k: v.detach().contiguous() for k, v in den.state_dict().items()},
              os.path.join(out_dir, "transformer", "diffusion_pytorch_model.safetensors"))
    te_tensors = {k: v.detach().contiguous() for k, v in te.state_dict().items()}
    lm_fields = {}
    if lm_dir:
        if type(te_cfg).__name__ != "LMEncoderConfig":
            raise ValueError("--lm-dir packs a frozen LM: the checkpoint's text encoder is not an LM encoder")
        lm_tensors, lm_fields, lm_tok = _lm_pack(te_cfg, lm_dir)
        te_tensors.update(lm_tensors)
        if tokenizer_json is None and lm_tok is not None:
            tokenizer_json = lm_tok
    save_file(te_tensors, os.path.join(out_dir, "text_encoder", "diffusion_pytorch_model.safetensors"))
    _write_json(os.path.join(out_dir, "transformer", "config.json"),
                dict(_class_name="AuroraDenoiser", **asdict(den_cfg), time_shift=shift, time_shift_ref=shift_ref))
    te_kind = type(te_cfg).__name__
    _write_json(os.path.join(out_dir, "text_encoder", "config.json"),
                dict(_class_name="AuroraLMTextEncoder" if te_kind == "LMEncoderConfig" else "AuroraTextEncoder",
                     **{**asdict(te_cfg), **lm_fields}))
    _write_json(os.path.join(out_dir, "scheduler", "scheduler_config.json"),
                dict(_class_name="EulerFlowMatch", shift=shift, shift_ref=shift_ref, num_train_timesteps=1000))
    index = dict(_class_name=PIPELINE_CLASS, transformer=["pipeline", "AuroraDenoiser"],
                 text_encoder=["pipeline", "AuroraLMTextEncoder" if te_kind == "LMEncoderConfig"
                               else "AuroraTextEncoder"],
                 scheduler=["pipeline", "EulerFlowMatch"], step=ck.get("step"),
                 weights="EMA" if used_ema else "live")
    if tokenizer_json:
        os.makedirs(os.path.join(out_dir, "tokenizer"), exist_ok=True)
        shutil.copy(tokenizer_json, os.path.join(out_dir, "tokenizer", "tokenizer.json"))
        index["tokenizer"] = ["transformers", "PreTrainedTokenizerFast"]
    if vae_dir:
        shutil.copytree(vae_dir, os.path.join(out_dir, "vae"), dirs_exist_ok=True)
        index["vae"] = ["diffusers", "AutoencoderKLFlux2"]
    with open(os.path.join(out_dir, "pipeline.py"), "w") as f:
        f.write(PIPELINE_SOURCE)
    _write_json(os.path.join(out_dir, "model_index.json"), index)
    return index


def load_export(src):
    """(te, den, den_cfg, te_cfg, transformer config dict) from an export directory."""
    from safetensors.torch import load_file

    from ..models import DenoiserConfig, build_models, te_config_from_dict
    with open(os.path.join(src, "transformer", "config.json")) as f:
        tcfg = json.load(f)
    den_cfg = DenoiserConfig(**{k: v for k, v in tcfg.items() if k in DenoiserConfig.__dataclass_fields__})
    with open(os.path.join(src, "text_encoder", "config.json")) as f:
        te_cfg = te_config_from_dict({k: v for k, v in json.load(f).items() if not k.startswith("_")})
    te, den = build_models(den_cfg, te_cfg)
    den.load_state_dict(load_file(os.path.join(src, "transformer", "diffusion_pytorch_model.safetensors")))
    te_tensors = load_file(os.path.join(src, "text_encoder", "diffusion_pytorch_model.safetensors"))
    te.load_state_dict({k: v for k, v in te_tensors.items() if not k.startswith("lm.")})
    return te, den, den_cfg, te_cfg, tcfg


def export_to_init(src, out_path):
    """An export -> a checkpoint usable as ``train.py --init`` (weights also as the EMA list; no optimizer state)."""
    from . import checkpoint as C
    te, den, den_cfg, te_cfg, tcfg = load_export(src)
    ck = dict(step=0, samples=0, den_config=asdict(den_cfg), te_config=asdict(te_cfg), te=C._sd(te), den=C._sd(den),
              opts=None, ema=C.ema_list(te, den, None), args=dict(t_shift=tcfg.get("time_shift", 1.0),
                                                                 t_shift_ref=tcfg.get("time_shift_ref", 0.0)),
              outer=None, repa_proj=None, imported_from=os.path.abspath(src))
    C.atomic_save(ck, out_path)
    return ck
