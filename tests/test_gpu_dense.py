"""Dense int8 layers (the B200 QLinear) on the GPU, through the C ABI: the dequantiser byte-exact
against moelab's dequantize arithmetic, the decode GEMV against the oracle, and the module's two
paths (GEMV for <= 8 tokens, dequantise + F.linear beyond)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn

from moeb200 import _lib, ops
from moeb200.dense import B200QLinear
from oracle import moe_oracle as O

from gpu_util import act_np

pytestmark = pytest.mark.gpu

DT = {"fp16": (torch.float16, "float16"), "bf16": (torch.bfloat16, "bfloat16")}


def _qs(Oo, K, gs, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn(Oo, K, generator=g, device=dev) * 0.02
    q, s = ops.quantize(w, 8, gs, "absmax")
    return q, s


@pytest.mark.parametrize("act", ["fp16", "bf16"])
@pytest.mark.parametrize("Oo,K,gs", [(256, 512, 64), (100, 768, 32), (64, 1024, 128)])
def test_dequant_matches_moelab_arithmetic(cuda_dev, act, Oo, K, gs):
    dt, dn = DT[act]
    q, s = _qs(Oo, K, gs, cuda_dev, Oo + K)
    w = ops.dense_int8_dequant(q, s, gs, dt)
    # moelab/quant.py:191-205 in torch: q.to(dtype) * scales.to(dtype) per group
    ref = (q.to(dt).reshape(Oo, K // gs, gs) * s.to(dt).unsqueeze(-1)).reshape(Oo, K)
    assert torch.equal(w.view(torch.int16), ref.view(torch.int16))
    assert np.array_equal(act_np(w), O.dense_int8_dequant(q.cpu().numpy(), s.cpu().numpy(), dn))


@pytest.mark.parametrize("act", ["fp16", "bf16"])
@pytest.mark.parametrize("T", [1, 3, 8])
@pytest.mark.parametrize("Oo,K,gs,bias", [(2048, 2048, 64, False), (1000, 768, 32, True), (50304, 2048, 64, False)])
def test_gemv_matches_oracle(cuda_dev, act, T, Oo, K, gs, bias):
    dt, dn = DT[act]
    q, s = _qs(Oo, K, gs, cuda_dev, 7 * T + Oo)
    g = torch.Generator(device=cuda_dev).manual_seed(T)
    x = torch.randn(T, K, generator=g, device=cuda_dev).to(dt)
    b = (torch.randn(Oo, generator=g, device=cuda_dev) * 0.1).to(dt) if bias else None
    y = ops.dense_int8_gemv(q, s, gs, x, b)
    ref = O.dense_int8_linear(act_np(x), q.cpu().numpy(), s.cpu().numpy(), None if b is None else act_np(b), dn)
    err = np.abs(act_np(y) - ref).max() / np.abs(ref).max()
    assert err < 1e-2, err  # fp32 sums in a different order + one rounding to the activation dtype


@pytest.mark.parametrize("act", ["fp16", "bf16"])
@pytest.mark.parametrize("T", [1, 8, 9, 64])
def test_module_paths(cuda_dev, act, T):
    dt, dn = DT[act]
    torch.manual_seed(T)
    lin = nn.Linear(1024, 1536, bias=True).to(cuda_dev).to(dt)
    ql = B200QLinear.from_linear(lin, cuda_dev)
    x = torch.randn(T, 1024, device=cuda_dev).to(dt)
    y = ql(x)
    assert y.shape == (T, 1536) and y.dtype == dt
    # the reference module's arithmetic: dequantise then F.linear (prefill) / the GEMV (decode)
    w = ops.dense_int8_dequant(ql.q, ql.s, ql.group_size, dt)
    ref = torch.nn.functional.linear(x, w) + ql.bias.to(dt)
    err = ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err < 1e-2, err
    if T > 8:  # the prefill path is the reference's own arithmetic: identical
        assert torch.equal(y, ref)


def test_gemv_rejects_bad_arguments(cuda_dev):
    q, s = _qs(64, 256, 64, cuda_dev, 1)
    x = torch.randn(9, 256, device=cuda_dev).half()
    with pytest.raises(_lib.MoeB200Error):
        ops.dense_int8_gemv(q, s, 64, x)  # more than 8 tokens
    q8, s8 = _qs(64, 256, 8, cuda_dev, 2)
    with pytest.raises(_lib.MoeB200Error):
        ops.dense_int8_gemv(q8, s8, 8, x[:1])  # group of 8 columns: GEMV needs multiples of 16
