"""The device quantiser (moeb200_quantize) byte-exact against the oracle quantiser and the
reference's golden integers and scales, and device-built records byte-identical to host-built ones."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from moeb200 import format as Fmt
from moeb200 import ops
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("method", ["absmax", "mse"])
def test_quantize_matches_reference_goldens(cuda_dev, golden, bits, method):
    w = torch.from_numpy(golden["quant/w"]).to(cuda_dev)
    q, s = ops.quantize(w, bits, 64, method)
    assert np.array_equal(q.cpu().numpy(), golden[f"quant/q{bits}_{method}"])
    assert np.array_equal(s.cpu().numpy().view(np.uint16), golden[f"quant/s{bits}_{method}"].view(np.uint16))


def test_quantize_negative_scales_match_reference(cuda_dev, golden):
    w = torch.from_numpy(golden["quant/wt"]).to(cuda_dev)
    q, s = ops.quantize(w, 4, 64, "mse")
    assert np.array_equal(q.cpu().numpy(), golden["quant/q4_mse_tail"])
    assert np.array_equal(s.cpu().numpy().view(np.uint16), golden["quant/s4_mse_tail"].view(np.uint16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bits,method,gs", [(4, "mse", 64), (4, "absmax", 32), (8, "mse", 64), (8, "absmax", 128),
                                            (4, "mse", 96), (4, "mse", 256), (8, "mse", 16)])
def test_quantize_matches_oracle(cuda_dev, dtype, bits, method, gs):
    g = torch.Generator(device=cuda_dev).manual_seed(bits * 100 + gs)
    K = 768 if gs != 256 else 1024
    w = torch.randn(130, K, generator=g, device=cuda_dev) * 0.02
    w[torch.rand(130, K, generator=g, device=cuda_dev) < 0.01] *= 20.0  # heavy tails: signed candidates
    w[3, :gs] = 0.0  # an all-zero group: the fp16(1e-7) scale
    w = w.to(dtype)
    q, s = ops.quantize(w, bits, gs, method)
    qo, so = O.quantize(w.float().cpu().numpy(), bits, gs, method)
    assert np.array_equal(q.cpu().numpy().view(np.uint8), qo.view(np.uint8))
    assert np.array_equal(s.cpu().numpy().view(np.uint16), so.view(np.uint16))


@pytest.mark.parametrize("prec", ["int4", "int8"])
def test_device_records_equal_host_records(cuda_dev, prec):
    lay = Fmt.record_layout(prec, 512, 256)
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    gu = torch.randn(512, 512, generator=g, device=cuda_dev) * 0.02
    dn = torch.randn(512, 256, generator=g, device=cuda_dev) * 0.02
    dev_rec = Fmt.encode_record(lay, gu, dn)
    host = O.encode_record(lay, gu.cpu().numpy(), dn.cpu().numpy())
    assert np.array_equal(dev_rec.cpu().numpy(), host)


@pytest.mark.parametrize("prec", ["int8", "int4"])
def test_device_records_match_reference_goldens(cuda_dev, golden, golden_meta, prec):
    lay = golden_meta["layouts"][f"{prec}_128_64"]
    blob = Fmt.encode_record(lay, torch.from_numpy(golden["rec/gu"]).to(cuda_dev),
                             torch.from_numpy(golden["rec/dn"]).to(cuda_dev))
    assert np.array_equal(blob.cpu().numpy(), golden[f"rec/{prec}"])
