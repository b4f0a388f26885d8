"""Checkpoint merging that emulates a learning-rate decay after constant-LR training.

WSM (Warmup-Stable-Merge, arXiv:2507.17634, Theorem 3.1): merging checkpoints theta_0..theta_k with
    c_0 = 1 - w_1,  c_j = w_j - w_{j+1},  c_k = w_k
equals having scaled the updates between them by the non-increasing decay coefficients w_1..w_k.
QAM (quadratic-accurate merging, arXiv:2609.35168): the coefficients of prod_j (1 - w_j + w_j t), which match the
decayed run to second order. Decay shapes: linear ("mean"), 1 - sqrt, cosine, over the window's progress.
(Reference: merge.py:34-77.)
"""
import math

DECAYS = {
    "mean": lambda p: 1 - p,
    "1-sqrt": lambda p: 1 - math.sqrt(p),
    "cosine": lambda p: 0.5 * (1 + math.cos(math.pi * p)),
}


def decay_profile(scheme, k):
    """Update strengths of the k intervals between k + 1 checkpoints."""
    return [DECAYS[scheme](i / (k + 1)) for i in range(1, k + 1)]


def merge_coefficients(scheme, n_ckpts, method="wsm"):
    """Non-negative weights (sum 1) for checkpoints ordered old -> new."""
    k = n_ckpts - 1
    if k <= 0:
        return [1.0]
    w = decay_profile(scheme, k)
    if method == "wsm":
        c = [1 - w[0]] + [w[j] - w[j + 1] for j in range(k - 1)] + [w[-1]]
    elif method == "qam":
        c = [1.0]
        for wj in w:  # multiply the polynomial by (1 - wj + wj t)
            nxt = [0.0] * (len(c) + 1)
            for i, ci in enumerate(c):
                nxt[i] += (1 - wj) * ci
                nxt[i + 1] += wj * ci
            c = nxt
    else:
        raise ValueError(f"unknown merge method {method!r}")
    assert all(x >= -1e-9 for x in c) and abs(sum(c) - 1) < 1e-6
    return c
