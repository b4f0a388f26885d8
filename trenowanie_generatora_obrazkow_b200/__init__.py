"""HomeIMG-B200: a Blackwell-native (sm_100a) rectified-flow DiT training and sampling framework.

Subpackages: ``models`` (DiT denoiser, text refiner, configs), ``ops`` (sm_100a kernels and their fp32 PyTorch
oracles), ``optim`` (Muon, AdamW groups, EMA, LR schedule), ``parallel`` (DDP gradient reduction, sharded Muon,
1F1B pipeline, expert parallelism, peer-memory communication), ``train`` (flow-matching trainers, OPD), ``data``
(shard store, train stream, synthetic FLUX.2-shaped data), ``sampling`` (Euler/CFG sampler, export), ``utils``.
"""
__version__ = "0.1.0"
