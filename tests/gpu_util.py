"""Helpers shared by the GPU parity tests: seeded records on the device, oracle views of them."""

from __future__ import annotations

import numpy as np
import torch

from moeb200 import format as F
from oracle import moe_oracle as O

TOL = 1e-2  # max |got - ref| / max |ref| for layer outputs (fp32 accumulation), per the spec


def act_np(x: torch.Tensor) -> np.ndarray:
    """Activations as the float32 values the kernels see."""
    return x.float().cpu().numpy()


def make_records(prec: str, H: int, I: int, n: int, seed: int, device, std: float = 0.02, scale: str | None = None):
    """n records of one precision built on the device from N(0, std) weights.
    Returns (layout, [uint8 CUDA tensors], [uint8 numpy copies])."""
    lay = F.record_layout(prec, H, I, scale=scale)
    g = torch.Generator(device=device).manual_seed(seed)
    blobs = []
    for _ in range(n):
        gu = torch.randn(2 * I, H, generator=g, device=device) * std
        dn = torch.randn(H, I, generator=g, device=device) * std
        blobs.append(F.encode_record(lay, gu, dn))
    return lay, blobs, [b.cpu().numpy() for b in blobs]


def layer_records(precs, H, I, E, seed, device, std=0.02, group_size=64):
    """Per precision, E records of the SAME float experts (like a store with several precisions)."""
    lays = {p: F.record_layout(p, H, I, group_size=group_size) for p in precs}
    g = torch.Generator(device=device).manual_seed(seed)
    recs = {p: [] for p in precs}
    for _ in range(E):
        gu = torch.randn(2 * I, H, generator=g, device=device) * std
        dn = torch.randn(H, I, generator=g, device=device) * std
        for p in precs:
            recs[p].append(F.encode_record(lays[p], gu, dn))
    return lays, recs


def emulate_router_logits(h: np.ndarray, wr: np.ndarray, dtype: str) -> np.ndarray:
    """Bit-exact emulation of the router-logit kernel's fp32 arithmetic: lane l of a warp takes the
    columns l*8 + 256*i + j (i over H/256, j over 8) in that order with fused multiply-adds (the
    product of two 16-bit values is exact in fp64, and one fp64 add of it to an fp32 partial
    rounded once to fp32 is the FMA), then an xor butterfly over offsets 16, 8, 4, 2, 1, then one
    rounding to the model dtype."""
    from oracle import moe_oracle as O

    T, H = h.shape
    E = wr.shape[0]
    hf = h.astype(np.float64).reshape(T, 1, H // 256, 32, 8)
    wf = wr.astype(np.float64).reshape(1, E, H // 256, 32, 8)
    acc = np.zeros((T, E, 32), np.float32)
    for i in range(H // 256):
        for j in range(8):
            prod = hf[:, :, i, :, j] * wf[:, :, i, :, j]  # (T, E, 32), exact
            acc = (acc.astype(np.float64) + prod).astype(np.float32)
    for o in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, :, np.arange(32) ^ o]).astype(np.float32)
    return O.round_to(acc[:, :, 0], dtype)
