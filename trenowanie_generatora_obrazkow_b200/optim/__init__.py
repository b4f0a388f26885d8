"""Optimizers: Muon (batched Newton-Schulz on the tcgen05 GEMM), AdamW grouping, LR schedule, EMA."""
from .groups import EMA, build_optimizers, lr_mult, set_lr, split_params
from .muon import Muon, muon_splits
from .newton_schulz import zeropower, zeropower_reference
