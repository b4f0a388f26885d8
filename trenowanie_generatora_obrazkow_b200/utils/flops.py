"""Training FLOP accounting and peak table (reference train.py:344-370 and train_pp.py:1697-1714).

Analytic count per training sample: 6 x (matrix parameters touched per token) x tokens for the linear layers plus
the attention products (self: 4 T^2 d per layer forward; cross: 4 T L d), times 3 for forward + backward.
"""

# dense bf16 tensor peak in TFLOP/s (fp32 accumulate)
PEAK_TFLOPS = {"B200": 2250.0, "H100": 989.0, "A100": 312.0, "5090": 209.5, "5080": 112.6, "4090": 165.2,
               "3090 Ti": 153.0, "3090": 71.0}


def peak_tflops(name):
    for key in sorted(PEAK_TFLOPS, key=len, reverse=True):
        if key in name:
            return PEAK_TFLOPS[key]
    return 0.0


def train_flops_per_sample(den_cfg, te_cfg, tokens, text_len=None):
    d, L = den_cfg.dim, den_cfg.depth
    text_len = text_len or getattr(te_cfg, "max_tokens", 64)
    per_block = 3 * d * d + d * d + d * d + 2 * d * den_cfg.text_dim + d * d + 3 * d * den_cfg.mlp_hidden
    lin = 2 * per_block * L * tokens + 2 * (den_cfg.latent_channels * d * 2) * tokens
    kv = 2 * 2 * d * den_cfg.text_dim * text_len * L  # cross kv projection runs on text tokens
    lin = lin - 2 * 2 * d * den_cfg.text_dim * L * tokens + kv
    attn = L * (4 * tokens * tokens * d + 4 * tokens * text_len * d)
    te_dim = te_cfg.dim
    te_lin = 2 * text_len * te_cfg.depth * (te_dim * (te_cfg.heads + 2 * te_cfg.kv_heads) * te_cfg.head_dim
                                           + te_cfg.heads * te_cfg.head_dim * te_dim + 3 * te_dim * te_cfg.mlp_hidden)
    return 3 * (lin + attn + te_lin)
