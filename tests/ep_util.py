"""Test helpers for expert parallelism: a torch mirror of the exchange-row format and CPU versions
of the four device steps (pack, unpack, owned-expert partial sums, combine) so the collective
data flow of moeb200.ep runs on gloo ranks without a GPU. The partial sums come from the oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as O


def row_bytes(H: int, k: int, dtype: torch.dtype) -> int:
    es = 4 if dtype == torch.float32 else 2
    b = H * es + 14 * k
    return (b + 15) // 16 * 16


def pack_rows(x, idx, w, level, skip) -> torch.Tensor:
    """[T, row_bytes] uint8: x row | idx int64 | w f32 | level u8 | skip u8 | zero pad."""
    T, H = x.shape
    k = idx.shape[1]
    rb = row_bytes(H, k, x.dtype)
    lv = level if level is not None else torch.zeros(T, k, dtype=torch.uint8, device=x.device)
    sk = skip if skip is not None else torch.zeros(T, k, dtype=torch.uint8, device=x.device)
    parts = [x.contiguous().view(torch.uint8).reshape(T, -1), idx.contiguous().view(torch.uint8).reshape(T, -1),
             w.contiguous().view(torch.uint8).reshape(T, -1), lv.reshape(T, k), sk.reshape(T, k)]
    row = torch.cat(parts, dim=1)
    pad = rb - row.shape[1]
    if pad:
        row = torch.cat([row, torch.zeros(T, pad, dtype=torch.uint8, device=x.device)], dim=1)
    return row.contiguous()


def unpack_rows(rows, H, k, dtype):
    n = rows.shape[0]
    es = 4 if dtype == torch.float32 else 2
    o = 0
    x = rows[:, o:o + H * es].contiguous().view(dtype).reshape(n, H)
    o += H * es
    idx = rows[:, o:o + 8 * k].contiguous().view(torch.int64).reshape(n, k)
    o += 8 * k
    w = rows[:, o:o + 4 * k].contiguous().view(torch.float32).reshape(n, k)
    o += 4 * k
    level = rows[:, o:o + k].contiguous()
    skip = rows[:, o + k:o + 2 * k].contiguous()
    return x, idx, w, level, skip


class CpuRuntime:
    """What ExpertParallel needs of a runtime, for CPU ranks: the expert count and, per slot, the
    records of the experts this rank owns (numpy uint8 blobs)."""

    def __init__(self, num_experts: int, layouts: list, records: list, n_prec: int):
        self.num_experts = num_experts
        self.layouts = layouts
        self.records = records  # records[slot][e] (None where this rank does not hold it)
        self.n_prec = n_prec
        self.capture_hook = None

    def levels(self, layer, w):
        return None, None


class CpuOps:
    """CPU stand-ins of moeb200.ep.CudaOps (same arguments, same results up to fp32 sum order)."""

    def row_bytes(self, H, k, dtype):
        return row_bytes(H, k, dtype)

    def pack(self, x, idx, w, level, skip, rows):
        rows.copy_(pack_rows(x, idx, w, level, skip))
        return rows

    def unpack(self, rows, H, k, dtype, x, idx, w, level, skip):
        xs, ids, ws, lv, sk = unpack_rows(rows, H, k, dtype)
        x.copy_(xs)
        idx.copy_(ids)
        w.copy_(ws)
        if level is not None:
            level.copy_(lv)
        if skip is not None:
            skip.copy_(sk)

    def local(self, runtime, layer, e_lo, e_hi, x, idx, w, level, skip, part):
        idx_n = idx.numpy()
        sk = skip.numpy().astype(bool) | (idx_n < e_lo) | (idx_n >= e_hi)
        slot = np.vectorize(lambda v: O.level_to_slot(int(v), runtime.n_prec))(level.numpy().astype(np.int64))
        y = O.moe_layer(x.float().numpy(), idx_n, w.numpy(), slot, sk, runtime.records, runtime.layouts,
                        runtime.num_experts)
        part.copy_(torch.from_numpy(y))
        return part

    def vote(self, idx, level, skip, num_experts, hi_vote):
        _, lv = O.expert_vote(idx.numpy(), level.numpy(), None if skip is None else skip.numpy().astype(bool),
                              num_experts, hi_vote)
        level.copy_(torch.from_numpy(lv))
        return level

    def combine(self, parts, out, add=False):
        acc = torch.zeros(parts.shape[1:], dtype=torch.float32)
        for g in range(parts.shape[0]):
            acc += parts[g]
        if add:
            acc = out.float() + acc
        out.copy_(acc.to(out.dtype))
        return out
