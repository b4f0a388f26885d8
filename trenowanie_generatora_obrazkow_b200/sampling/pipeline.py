"""Text -> image pipeline over an export directory: the ``HomeIMGPipeline`` that ``model_index.json`` names
(reference aurora/hf_pipeline.py:1-858, whose pipeline is a diffusers DiffusionPipeline twin of the training
modules). diffusers is not a dependency here: the pipeline is a plain class with the same steps and arguments.

  pipe = HomeIMGPipeline.from_pretrained("exports/homeimg", device="cuda")
  out = pipe(["a red fox in the snow"], height=1024, width=1024, num_inference_steps=50, guidance_scale=3.0)
  out.latents   # (B, 128, 64, 64) normalised FLUX.2 latents
  out.images    # (B, 1024, 1024, 3) uint8, when the export carries a VAE and diffusers is importable

Steps: tokenise (tokenizer/tokenizer.json: [BOS] ids [EOS] PAD rows for the from-scratch encoder, [BOS] ids
LM_PAD rows for a frozen-LM encoder), text encoder (frozen LM states -> refiner for LM encoders), CFG Euler
flow-matching loop with the scheduler's time shift (the fused CFG + Euler kernel on CUDA), VAE decode.
"""
import json
import os
from dataclasses import dataclass, replace

import numpy as np
import torch

from ..models.text import LMTextEncoder
from .euler import sample


@dataclass
class PipelineOutput:
    latents: torch.Tensor
    images: np.ndarray = None


class HomeIMGPipeline:
    def __init__(self, te, den, scheduler=None, tokenizer=None, frozen_lm=None, vae_dir=None, device="cuda",
                 max_tokens=None):
        self.te, self.den = te.to(device).eval(), den.to(device).eval()
        self.scheduler = scheduler or {}
        self.tokenizer, self.frozen_lm, self.vae_dir = tokenizer, frozen_lm, vae_dir
        self.device = torch.device(device)
        self.lm = isinstance(te, LMTextEncoder)
        self.max_tokens = max_tokens or getattr(te.config, "max_tokens", 128)
        self._decoder = None

    @classmethod
    def from_pretrained(cls, path, device="cuda", frozen_lm=None):
        """Load an export directory (utils/export.py layout). ``frozen_lm``: states provider for a frozen-LM text
        encoder (default: the LM backend recorded in text_encoder/config.json, if its weights are local)."""
        from ..models.frozen_lm import build_frozen_lm
        from ..utils.export import load_export
        te, den, den_cfg, te_cfg, tcfg = load_export(path)
        sched = {}
        sp = os.path.join(path, "scheduler", "scheduler_config.json")
        if os.path.exists(sp):
            with open(sp) as f:
                sched = json.load(f)
        sched.setdefault("shift", tcfg.get("time_shift", 1.0))
        sched.setdefault("shift_ref", tcfg.get("time_shift_ref", 0.0))
        tok = None
        tp = os.path.join(path, "tokenizer", "tokenizer.json")
        if os.path.exists(tp):
            from tokenizers import Tokenizer
            tok = Tokenizer.from_file(tp)
        if frozen_lm is None and isinstance(te, LMTextEncoder):  # the frozen LM blocks packed into the export
            from safetensors.torch import load_file

            from ..utils.export import packed_lm
            with open(os.path.join(path, "text_encoder", "config.json")) as f:
                te_json = json.load(f)
            if te_json.get("lm_arch"):
                frozen_lm = packed_lm(te_json, load_file(os.path.join(path, "text_encoder",
                                                                      "diffusion_pytorch_model.safetensors")), device)
        if frozen_lm is None and isinstance(te, LMTextEncoder) and getattr(te_cfg, "backend", "states") != "states":
            try:
                frozen_lm = build_frozen_lm(te_cfg, torch.device(device))
            except Exception:
                frozen_lm = None  # prompts then need lm_states passed in
        vae = os.path.join(path, "vae")
        return cls(te, den, sched, tok, frozen_lm, vae if os.path.isdir(vae) else None, device,
                   getattr(te_cfg, "max_tokens", None))

    # ---- text
    def tokenize(self, prompts):
        """Caption rows as the training shards hold them."""
        from ..models.frozen_lm import LM_PAD
        assert self.tokenizer is not None, "this export has no tokenizer/tokenizer.json: pass ids or lm_states"
        L = self.max_tokens
        if self.lm:
            rows = torch.full((len(prompts), L), LM_PAD, dtype=torch.long)
            enc = self.tokenizer.encode_batch([" ".join(p.split()) for p in prompts], add_special_tokens=False)
            bos = self.tokenizer.token_to_id("<|endoftext|>") or 0
            for j, e in enumerate(enc):
                ids = e.ids[: L - 1]
                rows[j, 0] = bos
                rows[j, 1:1 + len(ids)] = torch.tensor(ids)
            return rows
        from ..data.shards import BOS_ID, EOS_ID, PAD_ID
        rows = torch.full((len(prompts), L), PAD_ID, dtype=torch.long)
        enc = self.tokenizer.encode_batch([" " + " ".join(p.split()) for p in prompts], add_special_tokens=False)
        for j, e in enumerate(enc):
            ids = e.ids[: L - 2]
            rows[j, 0], rows[j, 1 + len(ids)] = BOS_ID, EOS_ID
            rows[j, 1:1 + len(ids)] = torch.tensor(ids)
        return rows

    def _text_args(self, prompts, ids, lm_states, valid):
        from ..models.frozen_lm import LM_PAD
        if lm_states is not None:
            return dict(lm_states=lm_states.to(self.device), valid=None if valid is None else valid.to(self.device))
        if ids is None:
            ids = self.tokenize(prompts)
        ids = ids.to(self.device)
        if not self.lm:
            return dict(ids=ids)
        assert self.frozen_lm is not None, "frozen-LM text encoder without a local LM: pass lm_states"
        return dict(lm_states=self.frozen_lm.states(ids), valid=ids.ne(LM_PAD))

    # ---- image
    def decode(self, latents):
        if self.vae_dir is None:
            return None
        if self._decoder is None:
            from .vae import LatentDecoder
            self._decoder = LatentDecoder(self.vae_dir, self.device)
        return self._decoder.decode(latents)

    @torch.no_grad()
    def __call__(self, prompt=None, ids=None, lm_states=None, valid=None, height=1024, width=None,
                 num_inference_steps=None, guidance_scale=3.0, shift=None, seed=0, batch=16, output_type="np"):
        width = width or height
        assert height == width and height % 16 == 0, "square images, a multiple of 16 px"
        if isinstance(prompt, str):
            prompt = [prompt]
        side = height // 16
        if self.den.config.latent_size != side:  # RoPE tables follow the latent grid
            self.den = self._resized(side)
        if shift is None:
            ref = self.scheduler.get("shift_ref") or 0
            shift = height / ref if ref else self.scheduler.get("shift", 1.0)
        steps = num_inference_steps or self.scheduler.get("num_inference_steps", 50)
        kw = self._text_args(prompt, ids, lm_states, valid)
        z = sample(self.te, self.den, steps=steps, cfg=guidance_scale, seed=seed, shift=shift, latent_size=side,
                   batch=batch, ids=kw.get("ids"), lm_states=kw.get("lm_states"), valid=kw.get("valid"))
        images = self.decode(z) if output_type != "latent" else None
        return PipelineOutput(latents=z, images=images)

    def _resized(self, side):
        from ..models import build_models
        den_cfg = replace(self.den.config, latent_size=side)
        _, den = build_models(den_cfg, self.te.config)
        den.load_state_dict(self.den.state_dict(), strict=False)
        return den.to(self.device).eval()
