"""Rectified-flow (flow-matching) objective.

Reference: FlowModel train.py:191-227 and the sampling of t / noise / caption dropout train.py:906-935,
train_pp.py:1901-1904.
  t  = sigmoid(N(0, 1)), shifted t -> s t / (1 + (s - 1) t)
  z_t = (1 - t) x0 + t eps ;  target = eps - x0 ;  loss = MSE(v.float(), target)
  cfg_drop of the captions are replaced by the null prompt (learned null vector for LM encoders).
Auxiliary losses: MLM on the from-scratch text encoder (reference train.py:216-227), REPA (train.py:199-215).
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import fused as Fz

from ..models.text import MASK_ID, LMTextEncoder


def shift_t(t, shift):
    return t if shift == 1.0 else shift * t / (1 + (shift - 1) * t)


def sample_t(n, device, shift=1.0, generator=None):
    """Logit-normal timesteps with the SD3 resolution shift."""
    return shift_t(torch.sigmoid(torch.randn(n, device=device, generator=generator)), shift)


def make_mlm(ids, prob, generator=None):
    """15% [MASK] on ids > MASK_ID -> (masked ids, labels with -100 elsewhere)."""
    maskable = ids > MASK_ID
    m = (torch.rand(ids.shape, device=ids.device, generator=generator) < prob) & maskable
    return ids.masked_fill(m, MASK_ID), ids.masked_fill(~m, -100)


class FlowModel(nn.Module):
    """Text encoder + denoiser in one module (one gradient bucket set, one checkpoint)."""

    def __init__(self, te, den, mlm_weight=0.0, repa_proj=None, repa_layer=0, repa_weight=0.0, moe_aux_weight=0.0):
        super().__init__()
        self.te, self.den, self.mlm_weight = te, den, mlm_weight
        self.moe_aux_weight = moe_aux_weight
        self.repa_proj, self.repa_layer, self.repa_weight = repa_proj, repa_layer, repa_weight

    def encode_text(self, ids=None, lm_states=None, valid=None, is_null=None):
        if isinstance(self.te, LMTextEncoder):
            return self.te(ids, lm_states=lm_states, valid=valid, is_null=is_null)
        return self.te(ids)

    def forward(self, x0, t, eps, ids=None, lm_states=None, valid=None, is_null=None, mlm_ids=None, mlm_labels=None,
                repa_target=None, cond=None, rope=None):
        """Returns (loss, fm, mlm or None, repa or None); x0 / eps (B, C, H, W) fp32, t (B,)."""
        text, text_valid = self.encode_text(ids, lm_states, valid, is_null)
        loss_repa = None
        repa = repa_target is not None and self.repa_proj is not None
        if x0.is_cuda and hasattr(self.den, "forward_tokens"):
            # one kernel writes the token-major input the patch-in GEMM reads and the token-major target the
            # token-major velocity is compared with (no latent-layout transposes on either side)
            z_tok, target = Fz.fm_inputs(x0, eps, t)
            out = self.den.forward_tokens(z_tok, x0.shape[2:], t, text, text_valid, cond=cond, rope=rope,
                                          hidden_at=self.repa_layer if repa else 0)
        else:
            tt = t.view(-1, 1, 1, 1)
            z_t = (1 - tt) * x0 + tt * eps
            target = eps - x0
            out = self.den(z_t, t, text, text_valid, cond=cond, rope=rope, hidden_at=self.repa_layer if repa else 0)
        if repa:
            v, h = out
            pred = self.repa_proj(h[: repa_target.shape[0]].float())
            loss_repa = -F.cosine_similarity(pred.float(), repa_target, dim=-1).mean()
        else:
            v = out
        loss_fm = F.mse_loss(v.float(), target)
        loss = loss_fm
        if self.moe_aux_weight > 0:
            from ..models.moe import moe_aux_loss
            aux = moe_aux_loss(self.den)
            if aux is not None:
                loss = loss + self.moe_aux_weight * aux
        if loss_repa is not None:
            loss = loss + self.repa_weight * loss_repa
            loss_repa = loss_repa.detach()
        if mlm_ids is None:
            return loss, loss_fm.detach(), None, loss_repa
        h, _ = self.te(mlm_ids)
        logits = h.float() @ self.te.token_embedding.weight.float().T  # MLM head tied to the embedding
        loss_mlm = F.cross_entropy(logits.flatten(0, 1), mlm_labels.flatten(), ignore_index=-100)
        return loss + self.mlm_weight * loss_mlm, loss_fm.detach(), loss_mlm.detach(), loss_repa


def drop_captions(is_null, valid, p, generator=None):
    """Classifier-free-guidance dropout for LM-state inputs: a fraction p of the rows become null prompts
    (valid = first token only)."""
    B = valid.shape[0]
    drop = torch.rand(B, device=valid.device, generator=generator) < p
    is_null = drop if is_null is None else (is_null | drop)
    valid = valid.clone()
    valid[drop] = False
    valid[drop, 0] = True
    return is_null, valid
