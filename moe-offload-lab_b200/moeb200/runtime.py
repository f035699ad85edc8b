"""Drop-in MoE-layer modules for transformers models, backed by libmoeb200.

``B200Experts`` replaces the module moelab swaps into each MoE block (``OffloadedExperts``,
moelab/runtime.py:1094-1112): same constructor inputs (runtime, layer, act_fn, num_experts), same
call ``forward(hidden_states [T,H], top_k_index [T,k] int64, top_k_weights [T,k] f32) -> [T,H]``,
same ``runtime.capture_hook`` so a segmented CUDA-graph decoder can cut around it.
``B200Router`` replaces the block's ``gate`` (the transformers TopKRouter) with the fused router
kernel and the same return contract ``(probs, weights, indices)``.

``B200Runtime`` holds what moelab's MoERuntime holds for resident experts: for every layer a device
table of record addresses per precision (moelab/fullgraph.py:43-98 DeviceTable), the precision
policy, and the scratch of the kernels. Every call stays on the device: no routing read-back, no
host synchronisation, so a whole decode step can be captured in one CUDA graph.
"""

from __future__ import annotations

import ctypes as C

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, ops
from .format import record_layout, to_c
from .ops import PolicySpec


def require_silu(act_fn) -> None:
    """The kernels compute silu(gate) * up, which is the OLMoE / Qwen3 expert; anything else is
    refused (the reference would fall back to torch; this build has no fallback)."""
    ok = act_fn is F.silu or type(act_fn).__name__ in ("SiLU", "SiLUActivation")
    if not ok:
        raise _lib.MoeB200Error(_lib.ERR_UNSUPPORTED, f"activation {act_fn!r} is not SiLU")


def level_to_slot(level: int, n_prec: int) -> int:
    """moelab/policy.py:188-192 (precisions listed most precise first)."""
    if n_prec >= 3:
        return min(level, n_prec - 1)
    return 0 if level == 0 else n_prec - 1


def aligned_copy(blob: torch.Tensor, align: int = 4096) -> torch.Tensor:
    """blob itself when its address is a multiple of align, else a copy at such an address (a view
    into a slightly larger buffer, which the view keeps alive)."""
    if blob.data_ptr() % align == 0:
        return blob
    n = blob.numel()
    buf = torch.empty(n + align, dtype=torch.uint8, device=blob.device)
    off = (-buf.data_ptr()) % align
    out = buf[off:off + n]
    out.copy_(blob.reshape(-1))
    return out


def aligned_empty(shape, device, align: int = 4096) -> torch.Tensor:
    """An uninitialised uint8 device tensor whose data starts at a multiple of align."""
    n = 1
    for d in shape:
        n *= d
    buf = torch.empty(n + align, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % align
    return buf[off:off + n].view(shape)


class B200Runtime:
    """Resident expert records of every MoE layer plus the policy, for the B200 kernels.

    precisions: store precisions, most precise first (e.g. ["fp16", "int4"]).
    layouts: {precision: moelab layout dict} (format.record_layout).
    """

    def __init__(self, precisions: list[str], layouts: dict, num_experts: int, device,
                 policy: PolicySpec | None = None, layers=()):
        if not 1 <= len(precisions) <= 4:
            raise ValueError("1 to 4 precisions")
        self.precisions = list(precisions)
        self.layouts = dict(layouts)
        self.num_experts = num_experts
        self.device = torch.device(device)
        self.policy = policy or PolicySpec("hi")
        self.capture_hook = None
        self._tables: dict[int, torch.Tensor] = {}
        self._ctables: dict[int, _lib.ExpertTable] = {}
        self._records: dict[tuple[int, int, str], torch.Tensor] = {}
        self._lays_c = [to_c(self.layouts[p]) for p in self.precisions]
        # lowest device address a record of this runtime can have (records and slots are 4096-byte
        # aligned): the base of the fused decode kernel's tensor maps
        self._tma_base = 0
        for layer in layers:
            self._table(layer)
        self.miss = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def n_prec(self) -> int:
        return len(self.precisions)

    def _table(self, layer: int) -> torch.Tensor:
        t = self._tables.get(layer)
        if t is None:
            t = torch.zeros(self.n_prec, self.num_experts, dtype=torch.int64, device=self.device)
            self._tables[layer] = t
            ct = _lib.ExpertTable()
            ct.n_prec = self.n_prec
            ct.num_experts = self.num_experts
            for i, L in enumerate(self._lays_c):
                ct.layout[i] = L
            ct.table = t.data_ptr()
            ct.tma_base = self._tma_base
            self._ctables[layer] = ct
        return t

    def note_region(self, addr: int) -> None:
        """Register device memory that records may occupy (4096-byte aligned), e.g. upload slots."""
        if addr % 4096:
            raise ValueError("record regions must be 4096-byte aligned")
        if self._tma_base == 0 or addr < self._tma_base:
            self._tma_base = addr
            for ct in self._ctables.values():
                ct.tma_base = addr

    def add_record(self, layer: int, expert: int, prec: str, blob: torch.Tensor) -> None:
        """Make a resident record visible to the kernels (blob: uint8 CUDA tensor, kept alive). A
        record that is not 4096-byte aligned is copied into an aligned buffer first."""
        if blob.device != self.device or blob.dtype != torch.uint8:
            raise ValueError("records must be uint8 tensors on the runtime's device")
        blob = aligned_copy(blob)
        self.note_region(blob.data_ptr())
        p = self.precisions.index(prec)
        self._records[(layer, expert, prec)] = blob
        self._table(layer)[p, expert] = blob.data_ptr()

    def record(self, layer: int, expert: int, prec: str) -> torch.Tensor:
        """The resident record blob of (layer, expert, precision)."""
        return self._records[(layer, expert, prec)]

    def remove_record(self, layer: int, expert: int, prec: str) -> None:
        p = self.precisions.index(prec)
        self._records.pop((layer, expert, prec), None)
        self._table(layer)[p, expert] = 0

    def votes(self, layer: int) -> bool:
        """Whether this layer's levels go through the per-expert vote (policy.hi_vote set, a rule that
        depends on the router weights, layer not protected)."""
        pol = self.policy
        return pol.hi_vote is not None and pol.mode not in ("hi", "lo") and layer not in pol.protect_layers

    def levels(self, layer: int, top_k_weights: torch.Tensor, top_k_index: torch.Tensor | None = None,
               vote: bool = True):
        """(level, skip) [T,k] of the policy; with ``policy.hi_vote`` set and more than one token, every
        kept pair takes its expert's vote (moelab/runtime.py:476-488), which needs top_k_index
        (vote=False: per-pair levels only, for callers that vote over more tokens themselves)."""
        pol = self.policy
        if pol.mode == "hi" and not pol.protect_layers:
            return None, None
        level, skip = ops.levels(top_k_weights.float().contiguous(), pol.to_c(layer))
        if vote and self.votes(layer) and top_k_weights.shape[0] > 1:
            if top_k_index is None:
                raise ValueError("the per-expert vote needs the routed expert indices")
            ops.levels_vote(top_k_index.long().contiguous(), level, skip, self.num_experts, pol.hi_vote)
        return level, skip

    @torch.no_grad()
    def run_layer(self, layer: int, x: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                  act_fn=None, out: torch.Tensor | None = None, level: torch.Tensor | None = None,
                  skip: torch.Tensor | None = None) -> torch.Tensor:
        """out[T,H] = weighted SwiGLU expert sum over the routed pairs (moelab/runtime.py:522-770,
        resident-expert path)."""
        if act_fn is not None:
            require_silu(act_fn)
        if level is None and skip is None:
            level, skip = self.levels(layer, top_k_weights.reshape(-1, top_k_index.shape[-1]),
                                      top_k_index.reshape(-1, top_k_index.shape[-1]))
        self._table(layer)
        x2 = x.reshape(-1, x.shape[-1])
        idx = top_k_index.reshape(x2.shape[0], -1)
        if idx.dtype != torch.int64:
            idx = idx.long()
        w = top_k_weights.reshape(idx.shape)
        if w.dtype != torch.float32:
            w = w.float()
        o = ops.experts_forward(self._ctables[layer], x2.contiguous(), idx.contiguous(), w.contiguous(), level, skip,
                                out=None if out is None else out.reshape(x2.shape), miss=self.miss)
        return o.view_as(x) if out is None else out


class B200Experts(nn.Module):
    """Drop-in for moelab's OffloadedExperts (moelab/runtime.py:1094-1112)."""

    def __init__(self, runtime: B200Runtime, layer: int, act_fn: nn.Module, num_experts: int):
        super().__init__()
        require_silu(act_fn)
        self.runtime = runtime
        self.layer = layer
        self.act_fn = act_fn
        self.num_experts = num_experts

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor) -> torch.Tensor:
        hook = self.runtime.capture_hook
        if hook is not None:
            return hook(self, hidden_states, top_k_index, top_k_weights)
        return self.runtime.run_layer(self.layer, hidden_states, top_k_index, top_k_weights, self.act_fn)

    def extra_repr(self) -> str:
        return f"moe_layer={self.layer}, experts={self.num_experts}, precisions={self.runtime.precisions}"


class B200Router(nn.Module):
    """Drop-in for the transformers TopKRouter (olmoe/modeling_olmoe.py:341-359): same attributes
    (top_k, num_experts, norm_topk_prob, hidden_dim, weight) and the same return contract
    (router probabilities [T,E] f32, top-k weights [T,k] f32, top-k indices [T,k] int64).
    ``bias`` adds a per-expert fp32 offset to the logits (the synthetic skew of the build's configs)."""

    def __init__(self, weight: torch.Tensor, top_k: int, norm_topk_prob: bool, bias: torch.Tensor | None = None):
        super().__init__()
        self.top_k = top_k
        self.num_experts, self.hidden_dim = weight.shape
        self.norm_topk_prob = norm_topk_prob
        self.weight = nn.Parameter(weight.detach(), requires_grad=False)
        self.register_buffer("bias", None if bias is None else bias.detach().float().contiguous())

    @classmethod
    def from_module(cls, gate: nn.Module) -> "B200Router":
        return cls(gate.weight, gate.top_k, bool(getattr(gate, "norm_topk_prob", False)))

    @torch.no_grad()
    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        wr = self.weight if self.weight.dtype == h.dtype else self.weight.to(h.dtype)
        probs, w, idx, _, _ = ops.router(h.contiguous(), wr.contiguous(), self.top_k, self.norm_topk_prob, self.bias)
        return probs, w, idx


class B200MoeBlock(nn.Module):
    """A whole Qwen3-Next sparse MoE block (transformers qwen3_next/modeling_qwen3_next.py:783-801:
    router, routed experts, sigmoid-gated shared expert) on the B200 kernels, with the shared expert
    folded into the routed launches: the router gives every token one more pair (expert E,
    sigmoid(x . shared_expert_gate)), and expert E of the runtime's table holds the shared MLP's
    record. No moelab counterpart: moelab leaves the shared expert to transformers."""

    def __init__(self, runtime: "B200Runtime", layer: int, router_weight: torch.Tensor, shared_gate: torch.Tensor,
                 top_k: int, norm_topk_prob: bool, shared_level: int = 0):
        super().__init__()
        self.runtime = runtime
        self.layer = layer
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.num_experts, self.hidden_dim = router_weight.shape
        self.shared_level = shared_level
        w = torch.cat([router_weight.detach(), shared_gate.detach().reshape(1, -1).to(router_weight.dtype)])
        self.register_buffer("router_ext", w.contiguous())

    @torch.no_grad()
    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        h = hidden_states.reshape(-1, self.hidden_dim).contiguous()
        rt = self.runtime
        wr = self.router_ext if self.router_ext.dtype == h.dtype else self.router_ext.to(h.dtype)
        pol = rt.policy
        want_levels = not (pol.mode == "hi" and not pol.protect_layers)
        _, w, idx, level, skip = ops.router(h, wr, self.top_k, self.norm_topk_prob, None,
                                            pol.to_c(self.layer) if want_levels else None, want_probs=False,
                                            shared_level=self.shared_level)
        if want_levels and rt.votes(self.layer) and h.shape[0] > 1:
            ops.levels_vote(idx, level, skip, self.num_experts + 1, pol.hi_vote)
        hook = rt.capture_hook
        if hook is not None:
            out = hook(self, h, idx, w)
        else:
            rt._table(self.layer)
            out = ops.experts_forward(rt._ctables[self.layer], h, idx, w, level, skip, miss=rt.miss)
        return out.reshape(shape)

    def extra_repr(self) -> str:
        return (f"moe_layer={self.layer}, experts={self.num_experts} + shared (folded), "
                f"precisions={self.runtime.precisions}")


def iter_moe_blocks(model: nn.Module):
    """(layer index, MoE block) for blocks holding 3-D experts and a router `gate` (as
    moelab/loader.py:53-65 finds them)."""
    li = 0
    for _, mod in model.named_modules():
        ex = getattr(mod, "experts", None)
        gate = getattr(mod, "gate", None)
        if ex is not None and gate is not None and hasattr(ex, "gate_up_proj") and hasattr(ex, "down_proj"):
            yield li, mod
            li += 1


def _shared_mlp(blk: nn.Module, inter: int):
    """(gate_up [2I, H], down [H, I]) of a block's shared expert when it can be folded (a SwiGLU MLP
    with the routed experts' intermediate size and a one-row sigmoid gate), else None."""
    se, sg = getattr(blk, "shared_expert", None), getattr(blk, "shared_expert_gate", None)
    if se is None or sg is None or not all(hasattr(se, n) for n in ("gate_proj", "up_proj", "down_proj")):
        return None
    if se.gate_proj.weight.shape[0] != inter or sg.weight.shape[0] != 1:
        return None
    require_silu(se.act_fn)
    return torch.cat([se.gate_proj.weight, se.up_proj.weight]), se.down_proj.weight


def install(model: nn.Module, precisions: list[str], policy: PolicySpec | None = None, group_size: int = 64,
            device=None, swap_router: bool = True, fold_shared: bool = False) -> B200Runtime:
    """Quantise every MoE block's experts into moelab records on the device, make them resident,
    and swap ``experts`` (and optionally ``gate``) for the B200 modules (moelab/loader.py:211-223).

    fold_shared: blocks with a Qwen3-Next shared expert of the routed experts' size are replaced
    whole by B200MoeBlock, the shared MLP quantised like the routed experts (every precision) and
    held as expert E; its pair always takes the most precise record (level 0)."""
    blocks = list(iter_moe_blocks(model))
    if not blocks:
        raise ValueError("no MoE block with 3-D experts found")
    ex0 = blocks[0][1].experts
    E, two_i, H = ex0.gate_up_proj.shape
    I = two_i // 2
    dev = torch.device(device) if device is not None else ex0.gate_up_proj.device
    fold = fold_shared and all(_shared_mlp(b, I) is not None for _, b in blocks)
    if fold_shared and not fold:
        raise ValueError("fold_shared: a block has no shared expert of the routed experts' size to fold")
    lays = {p: record_layout(p, H, I, group_size) for p in precisions}
    rt = B200Runtime(precisions, lays, E + (1 if fold else 0), dev, policy, layers=range(len(blocks)))
    from .format import encode_record

    parents = {id(m): (parent, name) for parent in model.modules() for name, m in parent.named_children()}
    for li, blk in blocks:
        ex = blk.experts
        require_silu(ex.act_fn)
        for e in range(E):
            gu = ex.gate_up_proj[e].detach().to(dev, torch.float32)
            dn = ex.down_proj[e].detach().to(dev, torch.float32)
            for p in precisions:
                rt.add_record(li, e, p, encode_record(lays[p], gu, dn))
        if fold:
            gu, dn = _shared_mlp(blk, I)
            for p in precisions:
                rt.add_record(li, E, p, encode_record(lays[p], gu.detach().to(dev, torch.float32),
                                                      dn.detach().to(dev, torch.float32)))
            new = B200MoeBlock(rt, li, blk.gate.weight.to(dev), blk.shared_expert_gate.weight.to(dev), blk.gate.top_k,
                               bool(getattr(blk.gate, "norm_topk_prob", False)))
            parent, name = parents[id(blk)]
            setattr(parent, name, new)
            continue
        blk.experts = B200Experts(rt, li, ex.act_fn, E)
        if swap_router:
            blk.gate = B200Router.from_module(blk.gate).to(dev)
    return rt
