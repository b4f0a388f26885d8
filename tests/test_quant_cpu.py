"""Frozen quantized projections (models/quant.py): output error of int8 / fp8 group-wise weights and of W8A8
against the bf16-free fp32 linear, and module-wide replacement."""
import pytest
import torch

from trenowanie_generatora_obrazkow_b200.models.quant import QLinear, W8A8Linear, quantize


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_group_quantized_linear_errors():
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 192)
    x = torch.randn(64, 512)
    ref = lin(x)
    assert _rel(QLinear(lin, "int8")(x), ref) < 0.01
    assert _rel(QLinear(lin, "fp8")(x), ref) < 0.04
    q = QLinear(lin, "int8")
    assert q.w.dtype == torch.int8 and q.w.numel() == lin.weight.numel() and q.s.numel() == 192 * 4


def test_w8a8_linear():
    torch.manual_seed(0)
    lin = torch.nn.Linear(256, 96)
    x = torch.randn(40, 256)
    try:
        y = W8A8Linear(lin)(x)
    except RuntimeError as e:  # no int8 GEMM on this backend
        pytest.skip(str(e))
    assert _rel(y, lin(x)) < 0.02


def test_quantize_replaces_linears():
    m = torch.nn.Sequential(torch.nn.Linear(64, 64), torch.nn.ReLU(), torch.nn.Sequential(torch.nn.Linear(64, 32)))
    quantize(m, "int8")
    assert isinstance(m[0], QLinear) and isinstance(m[2][0], QLinear)
    assert m(torch.randn(3, 64)).shape == (3, 32)
