"""Training: flow-matching objective, trainers (DDP / DiLoCo / pipeline), on-policy distillation."""
