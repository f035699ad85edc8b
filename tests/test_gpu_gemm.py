"""The tcgen05 grouped-GEMM (prefill) path vs the oracle, through the C ABI (needs a B200)."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from moeb200 import ops
from moeb200.runtime import B200Runtime
from oracle import moe_oracle as O

from gpu_util import TOL, act_np, layer_records

pytestmark = pytest.mark.gpu

ACTS = {"fp16": torch.float16, "bf16": torch.bfloat16}

CASES = [
    # (name, H, I, E, k, T, precs, policy, act, renorm, bias[, group size])
    ("small_int4_bf16", 256, 128, 8, 2, 40, ["int4"], dict(mode="lo"), "bf16", False, False),
    ("small_fp16_fp16", 256, 128, 8, 2, 40, ["fp16"], dict(mode="hi"), "fp16", False, False),
    ("small_int8_bf16", 256, 128, 8, 2, 40, ["int8"], dict(mode="lo"), "bf16", False, False),
    ("qwen3_30b_c2_T2048", 2048, 768, 128, 8, 2048, ["int4"], dict(mode="lo"), "bf16", True, True),
    ("olmoe_T512_mix", 2048, 1024, 64, 8, 512, ["fp16", "int4"], dict(mode="hobbit", t1=0.6), "fp16", False, False),
    ("qwen3next_T1024_int8_int4", 2048, 512, 512, 10, 1024, ["int8", "int4"], dict(mode="hobbit", t1=0.6), "bf16",
     True, True),
    # float records in the other 16-bit type and in fp32 (converted by the dequant warps)
    ("bf16_records_fp16_acts", 512, 256, 8, 2, 96, ["bf16"], dict(mode="hi"), "fp16", False, False),
    ("fp32_records_bf16_acts", 512, 256, 8, 2, 96, ["fp32"], dict(mode="hi"), "bf16", False, False),
    ("fp16_fp32_mix_fp16", 256, 128, 8, 2, 64, ["fp16", "fp32"], dict(mode="hobbit", t1=0.6), "fp16", False, False),
    # int4 rows of 704 bytes (a half raw unit at the end of every row of the down matrix)
    ("int4_I1408_bf16", 512, 1408, 8, 2, 80, ["int4"], dict(mode="lo"), "bf16", False, False),
    # groups smaller than a k-block: a scale per 8-column chunk
    ("int4_gs32_fp16", 512, 256, 8, 2, 80, ["int4"], dict(mode="lo"), "fp16", False, False, 32),
    ("int8_gs16_bf16", 512, 256, 8, 2, 80, ["int8"], dict(mode="lo"), "bf16", False, False, 16),
    ("int8_gs128_int4_fp16", 1024, 512, 16, 4, 200, ["int8", "int4"], dict(mode="hobbit", t1=0.6), "fp16", True,
     False, 128),
    # items of more than 128 pairs: the weight tile feeds two token halves (two B stages, two MMAs)
    ("fp16_items_of_200", 512, 256, 4, 2, 400, ["fp16"], dict(mode="hi"), "fp16", False, False),
    ("int8_items_of_256_bf16", 512, 256, 4, 2, 512, ["int8"], dict(mode="lo"), "bf16", False, False),
    ("int4_items_130_to_250", 1024, 256, 6, 3, 400, ["int4"], dict(mode="lo"), "fp16", False, False),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_gemm_path_matches_oracle(cuda_dev, case):
    name, H, I, E, k, T, precs, pol, act, renorm, bias = case[:11]
    gs = case[11] if len(case) > 11 else 64
    dt = ACTS[act]
    lays, recs = layer_records(precs, H, I, E, seed=zlib.crc32(name.encode()) % 1000, device=cuda_dev,
                               std=0.02 if H > 256 else 0.05, group_size=gs)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec(**pol), layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    g = torch.Generator(device=cuda_dev).manual_seed(7)
    x = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    wr = (torch.randn(E, H, generator=g, device=cuda_dev) * 0.02).to(dt)
    b = torch.randn(E, generator=g, device=cuda_dev) if bias else None
    _, wv, idx, _, _ = ops.router(x, wr, k, renorm, b, want_probs=False)
    ops.set_path("gemm")
    try:
        out = rt.run_layer(0, x, idx, wv, torch.nn.SiLU())
        torch.cuda.synchronize()
    finally:
        ops.set_path("auto")
    lvl, skip = rt.levels(0, wv)
    P = len(precs)
    lv = np.zeros((T, k), np.int64) if lvl is None else lvl.cpu().numpy().astype(np.int64)
    sk = None if skip is None else skip.cpu().numpy().astype(bool)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), P))(lv)
    recs_np = [[bb.cpu().numpy() for bb in recs[p]] for p in precs]
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, sk, recs_np, [lays[p] for p in precs], E)
    err = O.max_rel_err(act_np(out), ref)
    assert err < TOL, (name, err)
    # the same layer through the GEMV path agrees too
    ops.set_path("gemv")
    try:
        out2 = rt.run_layer(0, x, idx, wv, torch.nn.SiLU())
    finally:
        ops.set_path("auto")
    assert O.max_rel_err(act_np(out2), ref) < TOL
