"""Expert parallelism for the B200 MoE layer over NCCL (no moelab counterpart: moelab runs on one GPU).

Experts are split in contiguous blocks over the G ranks of a process group: rank r owns
experts [r*E//G, (r+1)*E//G) and holds only their records. Every rank routes its own T tokens
(router weights are replicated). One MoE layer is then three steps on the current stream, with no
host synchronisation, so the whole decode step stays capturable in one CUDA graph:

  dispatch  every rank packs each token's hidden row with its routing (top-k indices, weights,
            precision levels, skip flags) into one exchange row; one all_gather gives every rank
            all G*T rows, which are unpacked into the arrays the expert kernels read.
  experts   the owned experts over the G*T gathered tokens (pairs routed elsewhere are dropped);
            the down phase reduces straight into an fp32 partial-sum buffer [G*T, H].
  combine   one all_to_all_single sends rows [g*T, (g+1)*T) of the partial sums to rank g; each
            rank adds the G partials of its tokens in rank order 0..G-1 and casts once.

Every rank must call with the same T (a rank with fewer tokens pads with rows whose skip flags are
set). The collectives are NCCL over NVLink/NVSwitch on a GPU box; the same code runs on gloo with
CPU tensors when an ``ops`` object providing CPU versions of the four kernels is passed (tests).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn


def partition(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous expert block [lo, hi) owned by `rank` of `world` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if num_experts < world:
        raise ValueError(f"{num_experts} experts cannot be split over {world} ranks")
    return rank * num_experts // world, (rank + 1) * num_experts // world


def owner(expert: int, num_experts: int, world: int) -> int:
    """Rank owning `expert` under `partition` (inverse of the block split)."""
    if not 0 <= expert < num_experts:
        raise ValueError(f"expert {expert} outside [0, {num_experts})")
    r = (expert * world) // num_experts
    while partition(num_experts, world, r)[1] <= expert:
        r += 1
    while partition(num_experts, world, r)[0] > expert:
        r -= 1
    return r


class CudaOps:
    """The four device steps of an expert-parallel layer, on libmoeb200 kernels."""

    def row_bytes(self, H: int, k: int, dtype: torch.dtype) -> int:
        from . import ops

        return ops.ep_row_bytes(H, k, dtype)

    def pack(self, x, idx, w, level, skip, rows):
        from . import ops

        return ops.ep_pack(x, idx, w, level, skip, rows)

    def unpack(self, rows, H, k, dtype, x, idx, w, level, skip):
        from . import ops

        ops.ep_unpack(rows, H, k, dtype, x, idx, w, level, skip)

    def local(self, runtime, layer, e_lo, e_hi, x, idx, w, level, skip, part):
        from . import ops

        runtime._table(layer)
        return ops.experts_forward_part(runtime._ctables[layer], e_lo, e_hi, x, idx, w, level, skip, part=part,
                                        miss=runtime.miss)

    def combine(self, parts, out, add=False):
        from . import ops

        return ops.combine_parts(parts, out, add)


@dataclass
class _Bufs:
    rows: torch.Tensor
    rows_all: torch.Tensor
    x_all: torch.Tensor
    idx_all: torch.Tensor
    w_all: torch.Tensor
    level_all: torch.Tensor
    skip_all: torch.Tensor
    part: torch.Tensor
    recv: torch.Tensor


class ExpertParallel:
    """One rank of an expert-parallel MoE layer group.

    runtime: a B200Runtime holding the records of the experts this rank owns (`self.e_lo` ..
    `self.e_hi`); other experts' records are not needed on this rank.
    """

    def __init__(self, runtime, group=None, ops=None):
        self.runtime = runtime
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_lo, self.e_hi = partition(runtime.num_experts, self.world, self.rank)
        self.ops = ops if ops is not None else CudaOps()
        self._bufs: dict[tuple, _Bufs] = {}

    def owns(self, expert: int) -> bool:
        return self.e_lo <= expert < self.e_hi

    def _buffers(self, T: int, H: int, k: int, dtype: torch.dtype, device) -> _Bufs:
        key = (T, H, k, dtype, str(device))
        b = self._bufs.get(key)
        if b is None:
            G = self.world
            rb = self.ops.row_bytes(H, k, dtype)
            n = G * T
            b = _Bufs(rows=torch.empty(T, rb, dtype=torch.uint8, device=device),
                      rows_all=torch.empty(n, rb, dtype=torch.uint8, device=device),
                      x_all=torch.empty(n, H, dtype=dtype, device=device),
                      idx_all=torch.empty(n, k, dtype=torch.int64, device=device),
                      w_all=torch.empty(n, k, dtype=torch.float32, device=device),
                      level_all=torch.empty(n, k, dtype=torch.uint8, device=device),
                      skip_all=torch.empty(n, k, dtype=torch.uint8, device=device),
                      part=torch.empty(n, H, dtype=torch.float32, device=device),
                      recv=torch.empty(n, H, dtype=torch.float32, device=device))
            self._bufs[key] = b
        return b

    @torch.no_grad()
    def run_layer(self, layer: int, x: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                  level: torch.Tensor | None = None, skip: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """out[T,H] = this rank's tokens through the MoE layer whose experts are spread over the group."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T, H = x2.shape
        idx = top_k_index.reshape(T, -1)
        if idx.dtype != torch.int64:
            idx = idx.long()
        idx = idx.contiguous()
        k = idx.shape[1]
        w = top_k_weights.reshape(T, k).float().contiguous()
        if level is None and skip is None:
            level, skip = self.runtime.levels(layer, w)
        b = self._buffers(T, H, k, x2.dtype, x2.device)
        self.ops.pack(x2, idx, w, level, skip, b.rows)
        dist.all_gather_into_tensor(b.rows_all, b.rows, group=self.group)
        self.ops.unpack(b.rows_all, H, k, x2.dtype, b.x_all, b.idx_all, b.w_all, b.level_all, b.skip_all)
        self.ops.local(self.runtime, layer, self.e_lo, self.e_hi, b.x_all, b.idx_all, b.w_all, b.level_all,
                       b.skip_all, b.part)
        dist.all_to_all_single(b.recv, b.part, group=self.group)
        if out is None:
            out = torch.empty_like(x2)
        self.ops.combine(b.recv.view(self.world, T, H), out.view(T, H))
        return out.view_as(x)


class B200EPExperts(nn.Module):
    """Drop-in for moelab's OffloadedExperts (moelab/runtime.py:1094-1112) whose experts are spread
    over an expert-parallel group: same forward contract, every rank calls it with its own tokens."""

    def __init__(self, ep: ExpertParallel, layer: int, act_fn: nn.Module, num_experts: int):
        super().__init__()
        from .runtime import require_silu

        require_silu(act_fn)
        self.ep = ep
        self.runtime = ep.runtime
        self.layer = layer
        self.act_fn = act_fn
        self.num_experts = num_experts

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        hook = self.runtime.capture_hook
        if hook is not None:
            return hook(self, hidden_states, top_k_index, top_k_weights)
        return self.ep.run_layer(self.layer, hidden_states, top_k_index, top_k_weights)

    def extra_repr(self) -> str:
        return (f"moe_layer={self.layer}, experts={self.num_experts}, owned=[{self.ep.e_lo}, {self.ep.e_hi}), "
                f"ranks={self.ep.world}")
