"""Dense int8 linear layers: drop-in for moelab's QLinear (moelab/denseq.py:60-104).

The model's non-expert nn.Linear layers (attention projections, shared MLPs, the output head) stored
as int8 with one fp16 scale per group of input columns, in the store's format (quant.py
`quantize(w, 8, gs)`). Decode batches (up to 8 tokens) run the B200 int8 GEMV
(`moeb200_dense_int8_gemv`, one pass over the weights); larger batches dequantise row blocks with
`moeb200_dense_int8_dequant` (the exact values of moelab's `dequantize`) and multiply them with
F.linear, as the reference's prefill branch does (denseq.py:92-100). There is no CPU fallback: the
tensors must be on a CUDA device.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import format as Fmt
from . import ops

GEMV_MAX_TOKENS = 8


class B200QLinear(nn.Module):
    """nn.Linear with int8 group-quantised weights (weights only; the product is computed in float)."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor, group_size: int, bias: torch.Tensor | None, out_dtype):
        super().__init__()
        self.register_buffer("q", q.contiguous(), persistent=False)
        self.register_buffer("s", s.contiguous(), persistent=False)
        self.bias = None if bias is None else nn.Parameter(bias, requires_grad=False)
        self.group_size = group_size
        self.in_features, self.out_features = q.shape[1], q.shape[0]
        self.out_dtype = out_dtype
        self.gemv = group_size % 16 == 0 and self.in_features % 16 == 0

    @classmethod
    def from_linear(cls, lin: nn.Linear, device, group_size: int = 64) -> "B200QLinear":
        """Quantise an nn.Linear like moelab's QLinear.from_linear (absmax scales, gs64 by default)."""
        w = lin.weight.data
        gs = Fmt.pick_group_size(w.shape[1], group_size)
        q, s = ops.quantize(w.to(device).contiguous(), 8, gs, "absmax")
        bias = None if lin.bias is None else lin.bias.data.to(device)
        return cls(q, s, gs, bias, w.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        n = x2.shape[0]
        bias = None if self.bias is None else self.bias.to(x.dtype)
        if self.gemv and n <= GEMV_MAX_TOKENS and x.dtype in (torch.float16, torch.bfloat16):
            y = ops.dense_int8_gemv(self.q, self.s, self.group_size, x2.contiguous(), bias)
            return y.reshape(*lead, self.out_features)
        # several tokens (prefill): dequantise row blocks (bounded temporary memory) and multiply
        parts = []
        step = max(1, (64 * 2**20) // (self.in_features * x.element_size()))
        for o in range(0, self.out_features, step):
            w = ops.dense_int8_dequant(self.q[o: o + step], self.s[o: o + step], self.group_size, x.dtype)
            parts.append(F.linear(x2, w))
        y = torch.cat(parts, dim=-1) if len(parts) > 1 else parts[0]
        if bias is not None:
            y = y + bias
        return y.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, int8 gs{self.group_size} (B200)"


def quantize_dense(model: nn.Module, device, names: list[str], group_size: int = 64) -> int:
    """Replace the named nn.Linear modules of `model` by B200QLinear (the `dense_int8` load option).
    Returns the number of layers replaced."""
    n = 0
    for name in names:
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        lin = getattr(parent, child)
        if isinstance(lin, nn.Linear):
            setattr(parent, child, B200QLinear.from_linear(lin, device, group_size))
            n += 1
    return n
