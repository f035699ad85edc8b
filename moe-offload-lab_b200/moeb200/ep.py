"""Expert parallelism for the B200 MoE layer (no moelab counterpart: moelab runs on one GPU).

Experts are split in contiguous blocks over the G ranks of a process group: rank r owns
experts [r*E//G, (r+1)*E//G) and holds only their records. Every rank routes its own T tokens
(router weights are replicated). One MoE layer is then three steps on the current stream, with no
host synchronisation, so the whole decode step stays capturable in one CUDA graph:

  dispatch  every rank packs each token's hidden row with its routing (top-k indices, weights,
            precision levels, skip flags) into one exchange row; every rank receives all G*T rows
            and unpacks them into the arrays the expert kernels read.
  experts   the owned experts over the G*T gathered tokens (pairs routed elsewhere are dropped);
            the down phase reduces straight into an fp32 partial-sum buffer [G*T, H].
  combine   rank g receives rows [g*T, (g+1)*T) of every rank's partial sums, adds the G partials
            of its tokens in rank order 0..G-1 and casts once.

Two exchanges implement dispatch and combine:
  "nccl" (default): all_gather_into_tensor + all_to_all_single through torch.distributed (also runs
        on gloo with CPU tensors when an ``ops`` object with CPU versions of the kernels is passed:
        tests);
  "p2p": every rank's exchange rows and partial sums live in buffers its peers map
        with CUDA IPC; flag words (release/acquire at system scope, bounded waits) order them, the
        gather kernel reads the peers' rows over NVLink and unpacks them, the combine kernel reads
        the peers' partial rows of this rank's tokens and adds them in rank order -- no collective
        call, five kernels per layer, all capturable in a CUDA graph. On 2 B200s it measured ~5 %
        slower than NCCL for decode-sized layers (its system-scope signal / wait kernels cost more
        per layer than NCCL's small collectives), so it is opt-in.
Every rank must call with the same T (a rank with fewer tokens pads with rows whose skip flags are
set).

Cold experts (records held in pinned host memory, uploaded when routed) work under the "nccl"
exchange: attach a ColdExperts of this rank's runtime as `ExpertParallel.cold`; each rank then reads
the gathered routing back, uploads only the routed cold records of its own block and runs its
block's pairs as a resident pass and an uploaded pass.
"""

from __future__ import annotations

from dataclasses import dataclass

import ctypes as C

import torch
import torch.distributed as dist
import torch.nn as nn


class PeerFailure(RuntimeError):
    """A collective of the expert-parallel exchange did not complete: a peer raised and left, exited,
    or stalled past the process group's timeout. The group is unusable afterwards: every later call
    on the same ExpertParallel raises this at once instead of entering another collective."""


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

    def vote(self, idx, level, skip, num_experts, hi_vote):
        from . import ops

        return ops.levels_vote(idx, level, skip, num_experts, hi_vote)


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


class PeerExchange:
    """This rank's exchange buffers (packed rows [T, row_bytes], fp32 partial sums [G*T, H], flags
    int32 [2][G]) allocated with moeb200_peer_alloc, the peers' buffers mapped with CUDA IPC, and the
    moeb200_peer_group that points the exchange kernels at all of them. Creating one is a collective
    (the IPC handles travel through the process group)."""

    def __init__(self, group, world: int, rank: int, T: int, H: int, k: int, dtype: torch.dtype, device):
        from . import _lib
        from . import ops as O

        L = _lib.lib()
        self.world, self.rank, self.T, self.H, self.k = world, rank, T, H, k
        self.row_bytes = O.ep_row_bytes(H, k, dtype)
        sizes = {"rows": T * self.row_bytes, "parts": world * T * H * 4, "flags": 2 * world * 4}
        self.local: dict[str, int] = {}
        handles = {}
        for name, nbytes in sizes.items():
            ptr, h = C.c_void_p(), (C.c_char * 64)()
            _lib.check(L.moeb200_peer_alloc(nbytes, C.byref(ptr), h))
            self.local[name] = ptr.value
            handles[name] = bytes(h)
        allh: list = [None] * world
        dist.all_gather_object(allh, handles, group=group)
        self.opened: list[int] = []
        mapped = {name: [0] * world for name in sizes}
        for s in range(world):
            for name in sizes:
                if s == rank:
                    mapped[name][s] = self.local[name]
                    continue
                ptr = C.c_void_p()
                _lib.check(L.moeb200_peer_open(allh[s][name], C.byref(ptr)))
                mapped[name][s] = ptr.value
                self.opened.append(ptr.value)
        self.tabs = {name: torch.tensor(mapped[name], dtype=torch.int64, device=device) for name in sizes}
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        g = _lib.PeerGroup()
        g.G, g.rank, g.T, g.H, g.k = world, rank, T, H, k
        g.rows, g.parts, g.flags = (self.tabs["rows"].data_ptr(), self.tabs["parts"].data_ptr(),
                                    self.tabs["flags"].data_ptr())
        g.epoch, g.status = self.epoch.data_ptr(), self.status.data_ptr()
        self.group_c = g
        self.group = group

    def close(self) -> None:
        """Unmap the peers' buffers, wait for every rank to do the same, free this rank's buffers."""
        from . import _lib

        L = _lib.lib()
        torch.cuda.synchronize()
        for ptr in self.opened:
            L.moeb200_peer_close(C.c_void_p(ptr))
        self.opened = []
        dist.barrier(group=self.group)
        for ptr in self.local.values():
            L.moeb200_peer_free(C.c_void_p(ptr))
        self.local = {}


class ExpertParallel:
    """One rank of an expert-parallel MoE layer group.

    runtime: a B200Runtime holding the records of the experts this rank owns (`self.e_lo` ..
    `self.e_hi`); other experts' records are not needed on this rank.
    exchange: "nccl" (collectives, the default) or "p2p" (peer memory over NVLink, CUDA tensors only).
    """

    def __init__(self, runtime, group=None, ops=None, exchange: str | None = None):
        self.runtime = runtime
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_lo, self.e_hi = partition(runtime.num_experts, self.world, self.rank)
        self.ops = ops if ops is not None else CudaOps()
        if exchange is None:
            exchange = "nccl"
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', not {exchange!r}")
        self.exchange = exchange
        self._bufs: dict[tuple, _Bufs] = {}
        self._peers: dict[tuple, PeerExchange] = {}
        self.failed: str | None = None  # the first failed collective, once one failed
        self.cold = None  # optional ColdExperts of this rank's runtime ("nccl" exchange)
        # phase timing: when a list, every run_layer appends (pack + all_gather + unpack, experts,
        # all_to_all, combine) CUDA event pairs recorded on the current stream (eager calls only)
        self.timing: list | None = None

    def _collective(self, phase: str, fn, *args) -> None:
        """Run one collective of the exchange; a failure (peer error, exit or timeout) marks the group
        failed and raises PeerFailure naming the phase."""
        try:
            fn(*args, group=self.group)
        except Exception as exc:
            self.failed = f"{phase} on rank {self.rank}: {exc}"
            raise PeerFailure(self.failed) from exc

    def close(self) -> None:
        for px in self._peers.values():
            px.close()
        self._peers = {}

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
        votes = hasattr(self.runtime, "votes") and self.runtime.votes(layer)
        if level is None and skip is None:
            # per-pair levels here; a per-expert vote is taken over every rank's tokens after the gather
            level, skip = self.runtime.levels(layer, w, vote=False) if votes else self.runtime.levels(layer, w)
        elif votes and level is None:
            votes = False  # no levels to vote on
        if self.failed is not None:
            raise PeerFailure(f"the exchange group failed earlier ({self.failed})")
        b = self._buffers(T, H, k, x2.dtype, x2.device)
        if out is None:
            out = torch.empty_like(x2)
        if self.exchange == "p2p":
            if self.cold is not None:
                raise ValueError("cold experts under expert parallelism need the 'nccl' exchange")
            self._run_p2p(layer, x2, idx, w, level, skip, b, out.view(T, H), votes)
            return out.view_as(x)
        ev = self._events(5) if self.timing is not None else None
        if ev:
            ev[0].record()
        self.ops.pack(x2, idx, w, level, skip, b.rows)
        self._collective("dispatch all_gather", dist.all_gather_into_tensor, b.rows_all, b.rows)
        self.ops.unpack(b.rows_all, H, k, x2.dtype, b.x_all, b.idx_all, b.w_all, b.level_all, b.skip_all)
        if votes and self.world * T > 1:
            self.ops.vote(b.idx_all, b.level_all, b.skip_all, self.runtime.num_experts, self.runtime.policy.hi_vote)
        if ev:
            ev[1].record()
        if self.cold is not None:
            self.cold.run_part(layer, self.e_lo, self.e_hi, b.x_all, b.idx_all, b.w_all, b.level_all, b.skip_all,
                               b.part)
        else:
            self.ops.local(self.runtime, layer, self.e_lo, self.e_hi, b.x_all, b.idx_all, b.w_all, b.level_all,
                           b.skip_all, b.part)
        if ev:
            ev[2].record()
        self._collective("combine all_to_all", dist.all_to_all_single, b.recv, b.part)
        if ev:
            ev[3].record()
        self.ops.combine(b.recv.view(self.world, T, H), out.view(T, H))
        if ev:
            ev[4].record()
            self.timing.append(ev)
        return out.view_as(x)

    @staticmethod
    def _events(n: int) -> list:
        return [torch.cuda.Event(enable_timing=True) for _ in range(n)]

    def phase_ms(self) -> dict:
        """Per-phase milliseconds summed over the calls recorded in `timing` (synchronises):
        dispatch = pack + all_gather + unpack (+ vote), experts, combine_exchange = the all_to_all of
        the partial sums, combine = the rank-order add and cast."""
        torch.cuda.synchronize()
        tot = {"dispatch": 0.0, "experts": 0.0, "combine_exchange": 0.0, "combine": 0.0}
        for ev in self.timing or []:
            tot["dispatch"] += ev[0].elapsed_time(ev[1])
            tot["experts"] += ev[1].elapsed_time(ev[2])
            tot["combine_exchange"] += ev[2].elapsed_time(ev[3])
            tot["combine"] += ev[3].elapsed_time(ev[4])
        return tot

    def _run_p2p(self, layer, x2, idx, w, level, skip, b: _Bufs, out, votes: bool = False) -> None:
        from . import _lib
        from . import ops as O

        T, H = x2.shape
        k = idx.shape[1]
        key = (T, H, k, x2.dtype, str(x2.device))
        px = self._peers.get(key)
        if px is None:
            px = PeerExchange(self.group, self.world, self.rank, T, H, k, x2.dtype, x2.device)
            self._peers[key] = px
        L = _lib.lib()
        st = O._stream(x2.device)
        act = O._act(x2.dtype)
        g = C.byref(px.group_c)
        _lib.check(L.moeb200_ep_pack(O._ptr(x2), O._ptr(idx), O._ptr(w), O._ptr(level), O._ptr(skip), T, H, k, act,
                                     C.c_void_p(px.local["rows"]), st))
        _lib.check(L.moeb200_ep_signal(g, 0, st))
        _lib.check(L.moeb200_ep_gather(g, act, O._ptr(b.x_all), O._ptr(b.idx_all), O._ptr(b.w_all),
                                       O._ptr(b.level_all), O._ptr(b.skip_all), st))
        if votes and self.world * T > 1:
            O.levels_vote(b.idx_all, b.level_all, b.skip_all, self.runtime.num_experts, self.runtime.policy.hi_vote)
        rt = self.runtime
        rt._table(layer)
        n = self.world * T
        nbytes = L.moeb200_experts_workspace(C.byref(rt._ctables[layer]), n, k)
        ws = O.workspace(nbytes, x2.device, slot=0)
        _lib.check(L.moeb200_experts_forward_part(C.byref(rt._ctables[layer]), self.e_lo, self.e_hi, O._ptr(b.x_all),
                                                  act, n, O._ptr(b.idx_all), O._ptr(b.w_all), k, O._ptr(b.level_all),
                                                  O._ptr(b.skip_all), C.c_void_p(px.local["parts"]),
                                                  O._ptr(rt.miss), O._ptr(ws), ws.numel(), st))
        _lib.check(L.moeb200_ep_signal(g, 1, st))
        _lib.check(L.moeb200_ep_combine_peers(g, act, O._ptr(out), 0, st))

    def status(self) -> int:
        """Largest status word of this rank's peer exchanges (0 = every wait ended); synchronises."""
        torch.cuda.synchronize()
        return max([int(px.status.item()) for px in self._peers.values()] or [0])


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
