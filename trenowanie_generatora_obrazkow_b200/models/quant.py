"""Frozen quantized projections for teacher models (reference aurora/klein.py:45-107).

* ``QLinear``: 8-bit weights with one scale per group of ``group`` consecutive inputs of an output row, symmetric
  int8 (max |w| / 127) or fp8 e4m3 (max |w| / 448, e4m3's largest normal value); dequantised to the activation dtype
  and multiplied with the framework's GEMM (``ops.fused.linear``: the tcgen05 kernel on CUDA). Halves the weight
  memory of a frozen teacher; the arithmetic stays bf16.
* ``W8A8Linear``: per-output-channel int8 weights, dynamic per-token int8 activations, int32 accumulation. On CUDA
  the activations are quantised by one kernel and multiplied by the tcgen05 ``kind::i8`` GEMM with both scales
  applied in its epilogue (``ext().quantize_rows_i8``, ``ext().gemm_i8``); elsewhere ``torch._int_mm``. Used for
  frozen teachers only; the training path never quantises.
* ``quantize(module, kind)``: replaces every ``nn.Linear`` below ``module`` in place (kind "int8", "fp8" or
  "w8a8"; w8a8 only where both feature counts are multiples of 8, as the int8 GEMM requires).
"""
import torch
import torch.nn as nn

from ..ops import fused as Fz


class QLinear(nn.Module):
    def __init__(self, lin: nn.Linear, kind: str = "int8", group: int = 128):
        super().__init__()
        assert kind in ("int8", "fp8"), kind
        w = lin.weight.detach().float()
        out, inp = w.shape
        g = group if inp % group == 0 else inp
        wg = w.view(out, inp // g, g)
        top = 127.0 if kind == "int8" else 448.0
        scale = wg.abs().amax(-1, keepdim=True).clamp_min(1e-12) / top
        if kind == "int8":
            q = torch.round(wg / scale).clamp_(-127, 127).to(torch.int8)
        else:
            q = (wg / scale).to(torch.float8_e4m3fn)
        self.register_buffer("w", q)
        self.register_buffer("s", scale.to(torch.bfloat16))
        self.bias = lin.bias
        self.kind, self.shape = kind, (out, inp)

    def dequantized(self, dtype):
        return (self.w.to(dtype) * self.s.to(dtype)).view(self.shape)

    def forward(self, x):
        w = self.dequantized(x.dtype if x.is_floating_point() else torch.bfloat16)
        y = Fz.linear(x, w) if x.is_cuda else torch.nn.functional.linear(x, w)
        return y + self.bias if self.bias is not None else y


class W8A8Linear(nn.Module):
    def __init__(self, lin: nn.Linear):
        super().__init__()
        w = lin.weight.detach().float()
        scale = w.abs().amax(1).clamp_min(1e-12) / 127
        self.register_buffer("scale", scale)
        # [in, out] view of the row-major [out, in] int8 matrix (the layout the int8 GEMM takes for its B operand)
        self.register_buffer("weight_t", torch.round(w / scale[:, None]).clamp_(-127, 127).to(torch.int8).contiguous().T)
        self.bias = lin.bias

    def forward(self, x):
        k, n = self.weight_t.shape
        if x.is_cuda and k % 16 == 0 and n % 8 == 0:
            from ..ops._ext import err_buf, ext
            rows = x.reshape(-1, k).to(torch.bfloat16).contiguous()
            q, a_scale = ext().quantize_rows_i8(rows)
            out = torch.empty(rows.shape[0], n, device=x.device, dtype=torch.bfloat16)
            ext().gemm_i8(q, self.weight_t.T, out, a_scale, self.scale, err_buf(x.device))
            if self.bias is not None:
                out = out + self.bias.to(out.dtype)
            return out.to(x.dtype).reshape(*x.shape[:-1], n)
        rows = x.reshape(-1, x.shape[-1]).float()
        a_scale = rows.abs().amax(1, keepdim=True).clamp_min(1e-12) / 127
        q = torch.round(rows / a_scale).clamp_(-127, 127).to(torch.int8)
        pad = max(24, -(-q.shape[0] // 8) * 8) - q.shape[0]  # the int8 GEMM wants > 16 rows, a multiple of 8
        if pad:
            q = torch.nn.functional.pad(q, (0, 0, 0, pad))
        acc = torch._int_mm(q, self.weight_t)[:rows.shape[0]]
        out = acc.float() * a_scale * self.scale
        if self.bias is not None:
            out = out + self.bias.float()
        return out.to(x.dtype).reshape(*x.shape[:-1], -1)


def quantize(module: nn.Module, kind: str) -> nn.Module:
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear):
            if kind == "w8a8":
                if child.in_features % 8 == 0 and child.out_features % 8 == 0:
                    setattr(module, name, W8A8Linear(child))
            else:
                setattr(module, name, QLinear(child, kind))
        else:
            quantize(child, kind)
    return module
