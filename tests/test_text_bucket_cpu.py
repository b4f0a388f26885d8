"""Caption trimming and length-sorted micro-batches: trimming the padded tail of the text changes nothing in the
loss (pads are masked out), and length sorting groups similar lengths."""
import torch

from trenowanie_generatora_obrazkow_b200.models import DenoiserConfig, LMEncoderConfig
from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_PAD
from trenowanie_generatora_obrazkow_b200.train.trainer import TrainConfig, Trainer, length_sorted, trim_ids

DEN = DenoiserConfig(dim=64, depth=2, heads=1, mlp_hidden=128, text_dim=64, latent_channels=16, latent_size=4)
TE = LMEncoderConfig(lm_dim=32, dim=64, depth=1, heads=1, kv_heads=1, head_dim=64, mlp_hidden=128, max_tokens=32,
                     backend="states")


def test_trim_and_sort_helpers():
    ids = torch.full((4, 40), LM_PAD)
    for r, n in enumerate([3, 20, 9, 1]):
        ids[r, :n] = 5
    assert trim_ids(ids, 8).shape[1] == 24 and trim_ids(ids, 64).shape[1] == 40
    parts = length_sorted(ids, 2, torch.Generator().manual_seed(0))
    assert sorted(parts[0].tolist()) == [0, 3] and sorted(parts[1].tolist()) == [1, 2]


def _loss(bucket):
    torch.manual_seed(0)
    cfg = TrainConfig(global_batch=4, micro_batch=2, steps=1, cfg_drop=0.0, text_bucket=bucket, optimizer="adamw")
    tr = Trainer(DEN, TE, cfg, "cpu")
    g = torch.Generator().manual_seed(3)
    states = torch.randn(4, 32, 32, generator=g)
    valid = torch.zeros(4, 32, dtype=torch.bool)
    for r, n in enumerate([5, 9, 3, 12]):
        valid[r, :n] = True
    batch = dict(x0=torch.randn(4, 16, 4, 4, generator=g), lm_states=states, valid=valid)
    return float(tr.step(batch))


def test_text_bucket_keeps_the_loss():
    assert abs(_loss(0) - _loss(8)) < 1e-5
