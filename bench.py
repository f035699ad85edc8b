#!/usr/bin/env python
"""Benchmark of the B200 MoE-layer hot path (one JSON line on rank 0).

Default workload (config 1 of the build's configs): a 16-layer OLMoE-1B-7B-shaped MoE stack in
decode: H=2048, 64 SwiGLU experts of I=1024, top-8, softmax without renormalisation, router
weights and experts N(0, 0.02), every expert resident in HBM both as fp16 and as int4 gs64 (mse
scales), per-(token, expert) precision by the threshold rule (fp16 if the router probability is
>= 0.1, else int4), activations fp16, T tokens per step (default 64; 1/8/32 are swept too).
A step is the hot path of all 16 layers for T tokens: router -> precision mask -> dispatch ->
grouped gate/up GEMV -> grouped down GEMV + weighted combine, with a residual add between layers
standing in for the dense part (out of scope). Weights are random (no checkpoint), inputs seeded.

value: tokens/s with inputs resident in HBM, the step replayed as one CUDA graph.
e2e:   tokens/s through the public modules (B200Router + B200Experts per layer), copying the step's
       input from pinned host memory and reading its output back every step.
--impl reference: the reference's CPU expert path (materialise to fp32 + expert_ffn + weighted
       index_add, moelab/runtime.py:681-702) restated by the oracle, on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "moe-offload-lab_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/s"
CFG1 = dict(name="c1", layers=16, H=2048, I=1024, E=64, k=8, renorm=False, precs=["fp16", "int4"],
            policy=dict(mode="threshold", thr=0.1), act="fp16", bias=False, T=64)
# single-layer configurations reported beside the headline (BASELINE.json configs 0 and 2)
CFG0 = dict(name="c0", layers=1, H=2048, I=1024, E=64, k=8, renorm=False, precs=["int4"],
            policy=dict(mode="lo"), act="fp16", bias=False, T=1)
CFG2 = dict(name="c2", layers=1, H=2048, I=768, E=128, k=8, renorm=True, precs=["int4"],
            policy=dict(mode="lo"), act="bf16", bias=True, T=2048)
# config 3: Qwen3-Next-shaped layers, one protected (int8) and one int4, each with the sigmoid-gated
# shared expert (same precision as its layer); decode T=1 and prefill T=4096
CFG3 = dict(name="c3", layers=2, H=2048, I=512, E=512, k=10, renorm=True, precs=["int8", "int4"],
            layer_precs=[["int8"], ["int4"]], policy=dict(mode="lo", protect_layers=frozenset({0})), act="bf16",
            bias=False, shared=True, T=1)
CFG3P = dict(CFG3, name="c3p", T=4096)
# config 4: batched decode on the Qwen3-Next layer shape, Zipf(1.1) expert popularity as a router
# bias, fp16/int4 by router prob >= 0.05, 40 % of the experts (seeded choice) held in pinned host
# memory and uploaded every step on a copy stream (no record stays cached across steps)
CFG4 = dict(name="c4", layers=1, H=2048, I=512, E=512, k=10, renorm=True, precs=["fp16", "int4"],
            policy=dict(mode="threshold", thr=0.05), act="bf16", bias="zipf", T=256, cold_frac=0.4)
CONFIGS = {"c0": CFG0, "c1": CFG1, "c2": CFG2, "c3": CFG3, "c3p": CFG3P, "c4": CFG4}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--sweep", default="1,8,32", help="extra batch sizes reported beside the headline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling only)")
    ap.add_argument("--config", default="c1", choices=["c0", "c1", "c2", "c3", "c3p", "c4"],
                    help="workload of --ncu mode")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: one warm-up step, then one device step inside cudaProfilerStart/Stop")
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "gemm", "decode", "ws"])
    ap.add_argument("--exchange", default="nccl", choices=["p2p", "nccl"],
                    help="expert-parallel dispatch/combine (N > 1): peer memory over NVLink or NCCL collectives")
    ap.add_argument("--policy", default=None, choices=["hi", "lo"],
                    help="--ncu mode: every pair at the most precise (hi) or least precise (lo) record")
    ap.add_argument("--ep-extra", default="c3,c3p,c4",
                    help="configurations also run expert-parallel when --gpus > 1 (c3: T=1/GPU decode; c3p: "
                         "4096 tokens split over the ranks; c4: 256 tokens/GPU with cold uploads)")
    ap.add_argument("--extra", default="c0,c2,c3,c3p,c4,dense",
                    help="single-layer configs (and the dense int8 GEMV) measured beside the headline")
    return ap.parse_args()


# ---- distributed plumbing ---------------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- clocks ------------------------------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampled every 100 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        busy = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- workload ---------------------------------------------------------------------------------------------------
class Stack:
    """The 16-layer MoE stack of config 1 with every record resident on the device."""

    def __init__(self, cfg: dict, dev: torch.device, seed: int = 0, ep: bool = False, exchange: str = "p2p",
                 shared_mode: str = "fused"):
        import moeb200
        from moeb200 import format as F
        from moeb200 import ops

        self.cfg = cfg
        self.dev = dev
        L, H, I, E = cfg["layers"], cfg["H"], cfg["I"], cfg["E"]
        self.act = {"fp16": torch.float16, "bf16": torch.bfloat16}[cfg["act"]]
        self.lays = {p: F.record_layout(p, H, I) for p in cfg["precs"]}
        self.policy = ops.PolicySpec(**cfg["policy"])
        # Qwen3-Next shared expert folded into the routed launches as expert E (one more pair per
        # token from the router), or run beside them (its own gate / gate-up / down / finalize)
        self.shared_fused = bool(cfg.get("shared")) and not ep and shared_mode == "fused"
        self.rt = moeb200.B200Runtime(cfg["precs"], self.lays, E + (1 if self.shared_fused else 0), dev, self.policy,
                                      layers=range(L))
        # expert parallelism when launched on several ranks: this rank holds only its expert block
        self.ep = None
        self.world = 1
        if ep:
            import torch.distributed as dist

            from moeb200.ep import ExpertParallel

            self.world = dist.get_world_size()
            self.ep = ExpertParallel(self.rt, exchange=exchange)
        self.e_lo, self.e_hi = (self.ep.e_lo, self.ep.e_hi) if self.ep else (0, E)
        # expert-parallel runs: rank 0 also keeps layer 0 with ALL experts on one GPU, the reference
        # the EP layer output is checked against (built from the same seeded draws)
        self.rt_full0 = None
        if self.ep is not None and self.ep.rank == 0:
            self.rt_full0 = moeb200.B200Runtime(cfg["precs"], self.lays, E, dev, self.policy, layers=[0])
        g = torch.Generator(device=dev).manual_seed(seed)
        self.wr = []
        if cfg.get("bias") == "zipf":  # log(rank^-1.1) over a seeded permutation of the experts
            perm = torch.randperm(E, generator=g, device=dev)
            self.bias = torch.empty(E, device=dev)
            self.bias[perm] = -1.1 * torch.log(torch.arange(1, E + 1, device=dev, dtype=torch.float32))
        else:
            self.bias = (torch.randn(E, generator=g, device=dev) if cfg.get("bias") else None)
        self.shared = []  # per layer (record, layout, wg) of the shared expert, if the config has one
        self.wr_ext, self.shared_level = [], []  # fused shared expert: router rows + gate row, its level
        for li in range(L):
            self.wr.append((torch.randn(E, H, generator=g, device=dev) * 0.02).to(self.act))
            lprecs = cfg["layer_precs"][li] if cfg.get("layer_precs") else cfg["precs"]
            for e in range(E):
                gu = torch.randn(2 * I, H, generator=g, device=dev) * 0.02
                dn = torch.randn(H, I, generator=g, device=dev) * 0.02
                if li == 0 and self.rt_full0 is not None:
                    for p in lprecs:
                        self.rt_full0.add_record(0, e, p, F.encode_record(self.lays[p], gu, dn))
                if not self.e_lo <= e < self.e_hi:
                    continue
                for p in lprecs:
                    self.rt.add_record(li, e, p, F.encode_record(self.lays[p], gu, dn))
            if cfg.get("shared"):
                gu = torch.randn(2 * I, H, generator=g, device=dev) * 0.02
                dn = torch.randn(H, I, generator=g, device=dev) * 0.02
                wg = (torch.randn(H, generator=g, device=dev) * 0.02).to(self.act)
                lay = self.lays[lprecs[0]]
                rec = F.encode_record(lay, gu, dn)
                self.shared.append((rec, lay, F.to_c(lay), wg))
                if self.shared_fused:
                    slot = cfg["precs"].index(lprecs[0])
                    self.rt.add_record(li, E, lprecs[0], rec)
                    self.wr_ext.append(torch.cat([self.wr[li], wg[None, :]]).contiguous())
                    # the level whose precision slot holds the shared record (moelab/policy.py:188-192)
                    P = len(cfg["precs"])
                    self.shared_level.append(slot if P >= 3 else (0 if slot == 0 else 2))
        self.routers = [moeb200.B200Router(w, cfg["k"], cfg["renorm"], self.bias) for w in self.wr]
        if self.ep:
            from moeb200.ep import B200EPExperts

            self.experts = [B200EPExperts(self.ep, li, torch.nn.SiLU(), E) for li in range(L)]
        else:
            self.experts = [moeb200.B200Experts(self.rt, li, torch.nn.SiLU(), E) for li in range(L)]
        self.record_bytes = {p: self.lays[p]["record_bytes"] for p in cfg["precs"]}

    # device-resident step: fused router (+ mask) -> experts, residual between layers
    def make_device_step(self, T: int):
        from moeb200 import ops

        cfg, dev = self.cfg, self.dev
        L, k, H = cfg["layers"], cfg["k"], cfg["H"]
        kk = k + (1 if self.shared_fused else 0)  # the fused shared expert is one more pair per token
        self.bufs = [dict(w=torch.empty(T, kk, device=dev), idx=torch.empty(T, kk, dtype=torch.int64, device=dev),
                          level=torch.empty(T, kk, dtype=torch.uint8, device=dev),
                          skip=torch.empty(T, kk, dtype=torch.uint8, device=dev)) for _ in range(L)]
        self.xs = [torch.empty(T, H, dtype=self.act, device=dev) for _ in range(L + 1)]
        self.outs = [torch.empty(T, H, dtype=self.act, device=dev) for _ in range(L)]
        pols = [self.policy.to_c(li) for li in range(L)]
        tables = [self.rt._ctables[li] for li in range(L)]
        miss = self.rt.miss

        ep = self.ep
        fused = self.shared_fused
        shared = [] if fused else self.shared

        def step():
            for li in range(L):
                b = self.bufs[li]
                x = self.xs[li]
                if fused:
                    ops.router(x, self.wr_ext[li], k, cfg["renorm"], self.bias, pols[li], want_probs=False, out=b,
                               shared_level=self.shared_level[li])
                else:
                    ops.router(x, self.wr[li], k, cfg["renorm"], self.bias, pols[li], want_probs=False, out=b)
                if ep is not None:
                    ep.run_layer(li, x, b["idx"], b["w"], b["level"], b["skip"], out=self.outs[li])
                else:
                    ops.experts_forward(tables[li], x, b["idx"], b["w"], b["level"], b["skip"], out=self.outs[li],
                                        miss=miss)
                if shared:
                    rec, _, lay_c, wg = shared[li]
                    ops.shared_expert(lay_c, rec, wg, x, out=self.outs[li], add=True)
                torch.add(x, self.outs[li], out=self.xs[li + 1])
        return step

    def launches_per_step(self) -> int:
        # per layer: router logits, router top-k (+ levels), dispatch (one fused kernel when the
        # layer's pairs fit one 1024-pair block, else count, scan, scatter), gate/up GEMV, down GEMV,
        # finalize; expert parallel: + pack, unpack, combine, no finalize; shared expert run beside
        # the routed ones: gate kernel, gate/up, down, finalize (folded in: no launch of its own)
        T = self.xs[0].shape[0] * self.world
        kk = self.cfg["k"] + (1 if self.shared_fused else 0)
        disp = 1 if T * kk <= 1024 else 3
        base = 2 + disp + 2 + (3 if self.ep else 1)
        return self.cfg["layers"] * (base + (4 if self.shared and not self.shared_fused else 0))

    def gathered_routing(self, li: int):
        """idx, level, skip of every rank's tokens for layer li (numpy), outside any timed region."""
        b = self.bufs[li]
        if self.ep is None:
            return b["idx"].cpu().numpy(), b["level"].cpu().numpy(), b["skip"].cpu().numpy().astype(bool)
        import torch.distributed as dist

        outs = []
        for name in ("idx", "level", "skip"):
            t = b[name]
            full = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(full, t.contiguous())
            outs.append(full.cpu().numpy())
        return outs[0], outs[1], outs[2].astype(bool)

    def ep_layer0_error(self) -> float | None:
        """Expert-parallel parity of the last device step's layer 0: every rank's input rows, routing
        and EP output are gathered; rank 0 runs the same tokens and routing through the single-GPU
        layer over all experts and returns max |EP - single| / max |single| (None on other ranks).
        The two differ only in the fp32 summation order of the expert contributions."""
        import torch.distributed as dist

        from moeb200 import ops

        b = self.bufs[0]
        got = {}
        for name, t in (("x", self.xs[0]), ("out", self.outs[0]), ("idx", b["idx"]), ("w", b["w"]),
                        ("level", b["level"]), ("skip", b["skip"])):
            full = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(full, t.contiguous())
            got[name] = full
        err = None
        if self.rt_full0 is not None:
            rt = self.rt_full0
            ref = ops.experts_forward(rt._ctables[0], got["x"], got["idx"], got["w"], got["level"], got["skip"],
                                      miss=rt.miss)
            if self.shared:
                rec, _, lay_c, wg = self.shared[0]
                ops.shared_expert(lay_c, rec, wg, got["x"], out=ref, add=True)
            err = float((got["out"].float() - ref.float()).abs().max() / ref.float().abs().max().clamp_min(1e-30))
        dist.barrier()
        return err

    def e2e_step(self, x_host: torch.Tensor, x_dev: torch.Tensor, y_host: torch.Tensor):
        x_dev.copy_(x_host, non_blocking=True)
        x = x_dev
        for li in range(self.cfg["layers"]):
            _, w, idx = self.routers[li](x)
            x = x + self.experts[li](x, idx, w)
        y_host.copy_(x, non_blocking=True)

    def routing_bytes(self) -> dict:
        """Algorithmic bytes of the last device step per layer: distinct (expert, precision)
        records used, split into the gate/up and down matrices, plus activations."""
        from moeb200.format import field_offsets

        cfg = self.cfg
        P = len(cfg["precs"])
        out = {"up": 0, "down": 0, "records": 0, "pairs": 0, "up_layers": [], "down_layers": []}
        gu_bytes, dn_bytes = {}, {}
        for p in cfg["precs"]:
            lay = self.lays[p]
            f = {n: (s, d) for n, s, d, _ in lay["fields"]}
            el = {"float16": 2, "bfloat16": 2, "float32": 4, "int8": 1, "uint8": 1}

            def nb(name):
                s, d = f[name]
                return int(np.prod(s)) * el[d]

            if "gate_up" in f:
                gu_bytes[p], dn_bytes[p] = nb("gate_up"), nb("down")
            else:
                gu_bytes[p] = nb("gate_up.q") + nb("gate_up.s")
                dn_bytes[p] = nb("down.q") + nb("down.s")
        T, H, I = self.xs[0].shape[0] * self.world, cfg["H"], cfg["I"]
        for li in range(cfg["layers"]):
            idx, lvl, skip = self.gathered_routing(li)
            used = set()
            for t in range(idx.shape[0]):
                for j in range(idx.shape[1]):
                    if skip[t, j] or not self.e_lo <= int(idx[t, j]) < self.e_hi:
                        continue
                    lv = int(lvl[t, j])
                    slot = min(lv, P - 1) if P >= 3 else (0 if lv == 0 else P - 1)
                    used.add((int(idx[t, j]), slot))
                    out["pairs"] += 1
            pairs_l = out["pairs"] - sum(out.get("_pairs_prev", [0]))
            out.setdefault("_pairs_prev", []).append(pairs_l)
            up_l = sum(gu_bytes[cfg["precs"][s]] for (_, s) in used)
            dn_l = sum(dn_bytes[cfg["precs"][s]] for (_, s) in used)
            out["up"] += up_l
            out["down"] += dn_l
            # one gate/up launch: its records + the layer's token rows + the h rows it writes
            out["up_layers"].append(up_l + T * H * 2 + pairs_l * I * 2)
            out["down_layers"].append(dn_l + pairs_l * I * 2 + T * H * 4)
            out["records"] += len(used)
        for rec, lay, _, _ in self.shared:
            p = lay["precision"]
            out["up"] += gu_bytes[p]
            out["down"] += dn_bytes[p]
            out["records"] += 1
            out["shared_pairs"] = out.get("shared_pairs", 0) + T
        out.pop("_pairs_prev", None)
        n_pairs = out["pairs"] + out.get("shared_pairs", 0)
        out["up_total"] = out["up"] + cfg["layers"] * T * H * 2 + n_pairs * I * 2
        out["down_total"] = out["down"] + n_pairs * I * 2 + cfg["layers"] * T * H * 4
        return out


_L2_FLUSH: dict = {}


def l2_flush(dev) -> None:
    """Evict the 126 MB L2: write a 256 MB buffer (outside any timed interval)."""
    buf = _L2_FLUSH.get(str(dev))
    if buf is None:
        buf = _L2_FLUSH[str(dev)] = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    buf.zero_()


def time_graph(step, K: int, W: int, world: int, flush_l2: bool = False):
    """Captures step in a CUDA graph and returns (graph, ms per replay). flush_l2: evict L2 before
    every timed replay and time each replay on its own (workloads smaller than L2)."""
    for _ in range(W):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        step()
    for _ in range(max(3, W)):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if flush_l2:
        dev = torch.device("cuda", torch.cuda.current_device())
        evs = []
        for _ in range(K):
            l2_flush(dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        barrier(world)
        return g, sum(a.elapsed_time(b) for a, b in evs) / K
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = a.elapsed_time(b) / K
    return g, ms


def path_used() -> int:
    """Expert path of this thread's last experts_forward call: 1 GEMV, 2 GEMM, 3 fused decode, 4 warp-streamed GEMV."""
    from moeb200 import _lib

    return int(_lib.lib().moeb200_path_used())


def phase_times(step, reps: int = 5, flush_l2: bool = False):
    """Summed duration (ms) per step of the gate/up and of the down expert kernels, from CUDA events
    that libmoeb200 records on the launching stream around its phases (eager replay of the step;
    flush_l2: L2 evicted before every step)."""
    import ctypes as C

    from moeb200 import _lib

    lib = _lib.lib()
    step()
    torch.cuda.synchronize()
    dev = torch.device("cuda", torch.cuda.current_device())
    _lib.check(lib.moeb200_trace_begin())
    for _ in range(reps):
        if flush_l2:
            l2_flush(dev)
        step()
    up, dn, n = C.c_float(), C.c_float(), C.c_int32()
    _lib.check(lib.moeb200_trace_end(C.byref(up), C.byref(dn), C.byref(n)))
    return up.value / reps, dn.value / reps


def ep_phase_split(stack, step, reps: int, world: int) -> dict:
    """Expert-parallel layers: milliseconds per layer of dispatch (pack + all_gather + unpack),
    experts, the partial-sum all_to_all and the combine, from CUDA events of eager steps (host launch
    gaps included), max over ranks."""
    stack.ep.timing = []
    for _ in range(reps):
        step()
    ph = stack.ep.phase_ms()
    n = max(1, len(stack.ep.timing))
    stack.ep.timing = None
    out = {}
    for key in ("dispatch", "experts", "combine_exchange", "combine"):
        out[key] = max_over_ranks(ph[key] / n, world)
    out["timing"] = "eager steps, CUDA events per phase, per layer, max over ranks"
    return out


def measure_single(cfg: dict, dev, steps: int, warmup: int, world: int, peaks: dict, T: int | None = None,
                   exchange: str = "nccl") -> dict:
    """Tokens/s of one MoE layer of `cfg` (CUDA-graph replay, inputs resident) and the roofline of
    its expert kernels: HBM bytes for decode, tensor flops for prefill (tcgen05 path). With world > 1
    the layer runs expert-parallel (T tokens per rank) and the line carries the per-phase split and
    layer 0's parity against the single-GPU layer."""
    ep = world > 1
    stack = Stack(cfg, dev, seed=1, ep=ep, exchange=exchange)
    T = cfg["T"] if T is None else T
    L = cfg["layers"]
    step = stack.make_device_step(T)
    stack.xs[0].copy_(torch.randn(T, cfg["H"], device=dev).to(stack.act))
    # one layer's records may fit the 126 MB L2: evict it before every timed replay
    g, ms = time_graph(step, steps, warmup, world, flush_l2=True)
    del g
    ms = max_over_ranks(ms, world)
    if ep:
        err = stack.ep_layer0_error()
        phases = ep_phase_split(stack, step, 3, world)
        out = {"workload": cfg["name"], "T_per_gpu": T, "n_gpus": world, "layers": L,
               "tokens_per_s": T * world / (ms / 1e3), "ms_per_step": ms, "ms_per_layer": ms / L,
               "parallelism": f"ep{world} (NCCL all_gather + all_to_all)", "ep_max_rel_err": err,
               "ep_phase_ms_per_layer": phases,
               "layer_precisions": [lp[0] for lp in cfg["layer_precs"]] if cfg.get("layer_precs") else cfg["precs"],
               "shared_expert": "run beside the routed experts on every rank for its own tokens"
               if cfg.get("shared") else False,
               "l2": "evicted (256 MB write) before every timed replay"}
        stack.ep.close()
        del stack
        torch.cuda.empty_cache()
        return out
    rb = stack.routing_bytes()
    up_ms, dn_ms = phase_times(step, flush_l2=True)
    pairs = rb["pairs"] + rb.get("shared_pairs", 0)
    out = {"workload": cfg["name"], "T": T, "layers": L, "tokens_per_s": T * world / (ms / 1e3), "ms_per_step": ms,
           "ms_per_layer": ms / L, "experts_ms": up_ms + dn_ms, "records": rb["records"], "pairs": pairs,
           "layer_precisions": [lp[0] for lp in cfg["layer_precs"]] if cfg.get("layer_precs") else cfg["precs"],
           "shared_expert": ("folded into the routed launches (expert E, one more pair per token)"
                             if stack.shared_fused else bool(cfg.get("shared"))),
           "l2": "evicted (256 MB write) before every timed replay and every traced call"}
    prefill = T * cfg["k"] >= 40 * cfg["E"]  # the automatic path's GEMM switch (40 pairs per expert)
    if prefill:
        flops = 6.0 * cfg["H"] * cfg["I"] * pairs
        tf = flops / ((up_ms + dn_ms) / 1e3) / 1e12
        peak = peaks.get("bf16_tflops", 1590.0)
        out["roofline"] = {"bound": "tensor", "kernel": "tcgen05 grouped GEMM (up + down)", "achieved": tf,
                           "peak": peak, "unit": "TFLOP/s", "frac": tf / peak, "flops_per_step": flops,
                           "up_ms": up_ms, "down_ms": dn_ms}
    else:
        byts = rb["up_total"] + rb["down_total"]
        gbs = byts / ((up_ms + dn_ms) / 1e3) / 1e9
        peak = peaks.get("hbm_gbs", 6650.0)
        kname = {3: "fused decode kernel (one launch)", 4: "warp-streamed grouped GEMV (up + down)"}.get(
            path_used(), "grouped GEMV (up + down)")
        out["roofline"] = {"bound": "hbm", "kernel": kname, "achieved": gbs, "peak": peak,
                           "unit": "GB/s", "frac": gbs / peak, "bytes_per_step": byts, "up_ms": up_ms,
                           "down_ms": dn_ms}
    del stack
    torch.cuda.empty_cache()
    return out


def h2d_peak_gbs(dev, nbytes: int = 256 << 20) -> float:
    """Pinned host -> device copy bandwidth of this box (one large cudaMemcpyAsync, best of 3)."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) / 1e3) / 1e9)
    return best


def measure_dense(dev, steps: int, warmup: int, peaks: dict) -> dict:
    """The dense int8 GEMV (B200QLinear decode path) on the OLMoE output head shape: 50304 x 2048
    int8 gs64, one token, fp16 -- the largest dense layer read per decoded token (103 MB)."""
    from moeb200 import ops

    O, K, gs = 50304, 2048, 64
    g = torch.Generator(device=dev).manual_seed(3)
    w = torch.randn(O, K, generator=g, device=dev) * 0.02
    q, s = ops.quantize(w, 8, gs, "absmax")
    del w
    x = torch.randn(1, K, generator=g, device=dev).half()
    y = torch.empty(1, O, dtype=torch.float16, device=dev)

    def step():
        ops.dense_int8_gemv(q, s, gs, x, out=y)

    gr, ms = time_graph(step, steps, warmup, 1)
    del gr
    nbytes = q.numel() + s.numel() * 2 + K * 2 + O * 2
    gbs = nbytes / (ms / 1e3) / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    return {"workload": "dense int8 GEMV, OLMoE output head 50304x2048 gs64, T=1, fp16", "ms_per_call": ms,
            "bytes_per_call": nbytes, "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                                   "frac": gbs / peak},
            "timing": "CUDA graph replay of one call (weights 103 MB > L2), CUDA events"}


def measure_cold(cfg: dict, dev, steps: int, warmup: int, world: int = 1) -> dict:
    """Config 4: every step routes T tokens, uploads the routed cold records from pinned host memory
    on a copy stream while the resident pairs run, then runs the uploaded pairs. Eager steps (one
    routing read-back per layer, as the reference), CUDA events around the steps. With world > 1 the
    layer runs expert-parallel (T tokens per rank, NCCL exchange): each rank holds and uploads only the
    cold records of its own expert block, from the gathered routing of every rank."""
    from moeb200 import ops
    from moeb200.cold import ColdExperts

    ep = world > 1
    stack = Stack(cfg, dev, seed=2, ep=ep, exchange="nccl")
    E, T, k = cfg["E"], cfg["T"], cfg["k"]
    g = torch.Generator().manual_seed(4)
    cold_set = sorted(torch.randperm(E, generator=g)[: int(round(cfg["cold_frac"] * E))].tolist())
    owned = [e for e in cold_set if stack.e_lo <= e < stack.e_hi]
    cold = ColdExperts(stack.rt, {p: max(1, len(owned)) for p in cfg["precs"]})
    for e in owned:
        for p in cfg["precs"]:
            cold.add_cold(0, e, p, stack.rt._records[(0, e, p)].cpu())
    if ep:
        stack.ep.cold = cold
    torch.cuda.empty_cache()
    b = dict(w=torch.empty(T, k, device=dev), idx=torch.empty(T, k, dtype=torch.int64, device=dev),
             level=torch.empty(T, k, dtype=torch.uint8, device=dev), skip=torch.empty(T, k, dtype=torch.uint8, device=dev))
    x = torch.randn(T, cfg["H"], device=dev).to(stack.act)
    out = torch.empty_like(x)
    pol = stack.policy.to_c(0)

    def step():
        cold.reset()  # nothing stays cached: the cold records are uploaded again every step
        ops.router(x, stack.wr[0], k, cfg["renorm"], stack.bias, pol, want_probs=False, out=b)
        if ep:
            stack.ep.run_layer(0, x, b["idx"], b["w"], b["level"], b["skip"], out=out)
        else:
            cold.run_layer(0, x, b["idx"], b["w"], b["level"], b["skip"], out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    up0, by0 = cold.uploads, cold.uploaded_bytes
    a, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    e_.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(e_) / steps, world)
    ups = (cold.uploads - up0) / steps
    byts = (cold.uploaded_bytes - by0) / steps
    peak = h2d_peak_gbs(dev)
    gbs = byts / (ms / 1e3) / 1e9  # this rank's upload rate (every GPU has its own host link)
    res = {"workload": "c4", "T": T, "tokens_per_s": T * world / (ms / 1e3), "ms_per_step": ms,
           "cold_experts": len(cold_set), "uploads_per_step": ups, "upload_bytes_per_step": byts,
           "miss": int(stack.rt.miss.item()),
           "roofline": {"bound": "h2d", "kernel": "cold-record uploads (cudaMemcpyAsync on a copy stream)",
                        "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                        "peak_kind": "measured pinned H2D copy, 256 MiB"},
           "timing": "eager steps (routing read back per layer), CUDA events" + (", max over ranks" if ep else "")}
    if ep:
        res.update({"T_per_gpu": T, "n_gpus": world, "cold_experts_this_rank": len(owned),
                    "parallelism": f"ep{world} (NCCL all_gather + all_to_all; each rank uploads its own block's "
                                   "routed cold records)",
                    "uploads_per_step_rank0": ups, "upload_bytes_per_step_rank0": byts})
        res.pop("uploads_per_step")
        res.pop("upload_bytes_per_step")
        stack.ep.close()
    del stack, cold
    torch.cuda.empty_cache()
    return res


# ---- CPU baseline (oracle restatement of the reference's CPU expert path) ---------------------------------------
def cpu_layer_sample(stack: Stack, T: int, layer: int = 0):
    """One layer of the workload on the host cores: returns (seconds, sample description)."""
    from oracle import moe_oracle as O

    cfg = stack.cfg
    P = len(cfg["precs"])
    b = stack.bufs[layer]
    x = stack.xs[layer].float().cpu().numpy()
    idx = b["idx"].cpu().numpy()
    w = b["w"].cpu().numpy()
    lvl = b["level"].cpu().numpy().astype(np.int64)
    skip = b["skip"].cpu().numpy().astype(bool)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), P))(lvl)
    recs = [[stack.rt._records[(layer, e, p)].cpu().numpy() for e in range(cfg["E"])] for p in cfg["precs"]]
    lays = [stack.lays[p] for p in cfg["precs"]]
    t0 = time.perf_counter()
    O.moe_layer(x, idx, w, slot, skip, recs, lays, cfg["E"])
    dt = time.perf_counter() - t0
    return dt, f"layer {layer} of the step at T={T} (all its routed pairs), scaled x{cfg['layers']} layers"


def headline_config(T: int, world: int, exchange: str) -> dict:
    """The `config` object of the headline line, shared by both arms (same workload, same keys)."""
    return {"workload": f"c1 OLMoE-1B-7B 16-layer MoE stack decode, T={T}/GPU, "
                        "fp16/int4 by router prob >= 0.1, all experts resident",
            "global_batch": T * world, "layers": CFG1["layers"], "experts": CFG1["E"], "top_k": CFG1["k"],
            "hidden": CFG1["H"], "inter": CFG1["I"],
            "parallelism": (f"ep{world} (experts in contiguous blocks; dispatch/combine " + (
                "through peer memory over NVLink: CUDA IPC buffers, flag handshakes)"
                if exchange == "p2p" else "by NCCL all_gather + all_to_all)")) if world > 1 else "1gpu",
            "l2": "no flush: each step streams the routed records of 16 layers, GBs (> 126 MB L2)",
            "dense_part": "attention stood in by a residual add between layers (out of scope)",
            "timing": "CUDA graph replay of the whole step, CUDA events, max over ranks"}


def _encode_oracle(args):
    """Worker of the reference arm's record pool: one record with the oracle's numpy quantiser."""
    from oracle import moe_oracle as O

    lay, gu, dn = args
    return O.encode_record(lay, gu, dn)


def reference_arm(args, world, rank):
    """--impl reference: the reference's CPU expert path (moelab/runtime.py:681-702: materialise each
    routed record to fp32, expert_ffn, weighted index_add) on the host cores, rank 0 only.

    The reference (moelab) is a Python project without packaging metadata, so it cannot be installed
    on the GPU box; its CPU path runs here as the oracle's numpy restatement (kind "port"), pinned
    to the reference's own outputs by the golden tests. Nothing of this build's CUDA library runs:
    the weights are drawn with the same seeded torch generator as the headline's layer 0, records
    are quantised by the oracle (a process pool on the host cores), routing and masks by the oracle.
    Each timed step is ONE MoE layer of the workload (all T*k routed pairs of layer 0): ms_per_step is
    that measured layer, and value = T / (16 x ms_per_step), the metric of the 16 identical layers."""
    if rank != 0:
        return
    import multiprocessing as mp

    from oracle import moe_oracle as O

    cfg = CFG1
    H, I, E, k, T = cfg["H"], cfg["I"], cfg["E"], cfg["k"], args.batch
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    g = torch.Generator(device=dev).manual_seed(0)
    lays = [O.record_layout(p, H, I) for p in cfg["precs"]]
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).half().float().cpu().numpy()
    jobs = []
    for e in range(E):
        gu = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).cpu().numpy()
        dn = (torch.randn(H, I, generator=g, device=dev) * 0.02).cpu().numpy()
        jobs += [(lay, gu, dn) for lay in lays]
    cores = os.cpu_count() or 1
    t_build = time.perf_counter()
    with mp.get_context("spawn").Pool(min(cores, 32)) as pool:
        blobs = pool.map(_encode_oracle, jobs, chunksize=1)
    t_build = time.perf_counter() - t_build
    recs = [[blobs[e * len(lays) + s_] for e in range(E)] for s_ in range(len(lays))]
    torch.manual_seed(1234)
    x = torch.randn(T, H, device=dev).half().float().cpu().numpy()
    probs, w, idx, _ = O.router(x, wr, k, cfg["renorm"], "float16")
    lvl, skip = O.threshold_levels(w, cfg["policy"]["thr"])
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), len(lays)))(lvl.astype(np.int64))
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.moe_layer(x, idx, w, slot, skip, recs, lays, E)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    step_s = float(np.mean(times))
    v = T / (cfg["layers"] * step_s)
    sample = (f"each step: layer 0 of the workload (all {T * k} routed pairs of T={T}, records materialised "
              f"to fp32 per call, numpy on the host cores); value = T / ({cfg['layers']} x measured step)")
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "layers_per_step": 1, "ms_per_layer": step_s * 1e3,
            "config": headline_config(T, world, args.exchange),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "setup_s": {"record_quantisation": t_build}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_kind = "measured" if "hbm_gbs" in peaks else "fallback"
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config] if args.ncu else CFG1)
    if args.layers:
        cfg["layers"] = args.layers
    if args.ncu and args.policy:
        cfg["policy"] = dict(mode=args.policy)
    from moeb200 import ops as _ops

    _ops.set_path(args.path)
    stack = Stack(cfg, dev, seed=0, ep=world > 1, exchange=args.exchange)
    T = args.batch if not args.ncu or args.config == "c1" else cfg["T"]
    if args.ncu:
        step = stack.make_device_step(T)
        stack.xs[0].copy_(torch.randn(T, cfg["H"], device=dev).to(stack.act))
        step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        rb = stack.routing_bytes()
        print(json.dumps({"ncu_step_done": True, "layers": cfg["layers"], "T": T,
                          "up_alg_bytes_per_layer": rb["up_layers"], "down_alg_bytes_per_layer": rb["down_layers"]}))
        return
    H = CFG1["H"]
    torch.manual_seed(1234 + rank)
    x0 = torch.randn(T, H, device=dev).to(stack.act)

    # headline: device-resident step replayed as a CUDA graph
    step = stack.make_device_step(T)
    stack.xs[0].copy_(x0)
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    graph, ms = time_graph(step, args.steps, args.warmup, world)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world)
    value = T * world / (ms / 1e3)
    rb = stack.routing_bytes()
    miss = int(stack.rt.miss.item())
    del graph
    # expert-parallel runs: the last replay's layer 0 against the single-GPU layer (outside timing)
    ep_err = stack.ep_layer0_error() if world > 1 else None
    # expert-parallel runs: per-phase split of the headline layers (eager steps, outside the timed region)
    ep_phases = ep_phase_split(stack, step, 2, world) if world > 1 else None

    # roofline of the dominant kernel (gate/up GEMV) from CUDA events on its stream
    try:
        up_ms, dn_ms = phase_times(step)
        up_ms, dn_ms = up_ms / cfg["layers"], dn_ms / cfg["layers"]  # one call per layer
    except Exception as exc:  # the measurement hook failed: report no roofline rather than guess
        print(f"phase timing unavailable: {exc}", file=sys.stderr)
        up_ms = dn_ms = float("nan")
    L = cfg["layers"]
    fused = path_used() == 3
    if fused:
        # one launch per layer does gate/up, down, the combine and the cast: its bytes are both phases'
        up_bytes_launch = (rb["up_total"] + rb["down_total"]) / L
        dn_bytes_launch = 0.0
        up_ms, dn_ms = up_ms + dn_ms, 0.0
    else:
        up_bytes_launch = rb["up_total"] / L
        dn_bytes_launch = rb["down_total"] / L
    up_gbs = up_bytes_launch / (up_ms / 1e3) / 1e9
    dn_gbs = dn_bytes_launch / (dn_ms / 1e3) / 1e9 if dn_ms > 0 else None
    # DRAM bytes (read + write) of one launch of the dominant kernel: the committed ncu capture of
    # this workload's layer 0 (a 2-layer stack), scaled from that launch's algorithmic bytes to this
    # run's average launch (DRAM traffic follows the records a layer routes to)
    traffic, traffic_src = None, None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists() and world == 1 and T == CFG1["T"]:
        rec = json.loads(tf.read_text()).get("decode_c1_T64" if fused else "gemv_up_c1_T64")
        if rec:
            traffic = rec["dram_bytes"] * up_bytes_launch / rec["alg_bytes"]
            traffic_src = (rec["source"] + f"; captured launch: {rec['dram_bytes']} DRAM bytes for {rec['alg_bytes']} "
                           "algorithmic bytes, scaled to this run's average launch")

    # sweep of other decode batches (device-resident value only)
    sweep = {}
    for Ts in [int(s) for s in args.sweep.split(",") if s.strip()]:
        st = stack.make_device_step(Ts)
        stack.xs[0].copy_(torch.randn(Ts, H, device=dev).to(stack.act))
        g2, ms2 = time_graph(st, max(5, args.steps // 2), 3, world)
        del g2
        ms2 = max_over_ranks(ms2, world)
        rb2 = stack.routing_bytes()
        sweep[str(Ts)] = {"tokens_per_s": Ts * world / (ms2 / 1e3), "ms_per_step": ms2,
                          "record_gbs": (rb2["up"] + rb2["down"]) / (ms2 / 1e3) / 1e9}

    # end to end through the public modules, host copies inside the timed region
    x_host = x0.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x0)
    for _ in range(args.warmup):
        stack.e2e_step(x_host, x_dev, y_host)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        stack.e2e_step(x_host, x_dev, y_host)
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
    e2e = T * world / (e2e_ms / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        stack.make_device_step(T)
        stack.xs[0].copy_(x0)
        st = stack.make_device_step(T)
        stack.xs[0].copy_(x0)
        st()
        torch.cuda.synchronize()
        dt, sample = cpu_layer_sample(stack, T, layer=0)
        cpu = {"value": T / (dt * L), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": sample}

    extra = {}
    if world > 1:
        for name in [c for c in args.ep_extra.split(",") if c]:
            cfgx = CONFIGS[name]
            if cfgx.get("cold_frac"):
                extra[name] = measure_cold(cfgx, dev, max(5, args.steps // 2), 3, world)
            elif name == "c3p":  # prefill: the 4096 tokens split over the ranks (strong scaling)
                extra[name] = measure_single(cfgx, dev, max(5, args.steps // 2), 3, world, peaks,
                                             T=max(1, cfgx["T"] // world))
                extra[name]["scaling"] = "strong (4096 tokens in total)"
            else:
                extra[name] = measure_single(cfgx, dev, max(5, args.steps // 2), 3, world, peaks)
    for name in [c for c in args.extra.split(",") if c and world == 1]:
        if name == "dense":
            extra[name] = measure_dense(dev, max(20, args.steps), 5, peaks)
            continue
        cfgx = CONFIGS[name]
        if cfgx.get("cold_frac"):
            extra[name] = measure_cold(cfgx, dev, max(5, args.steps // 2), 3)
        else:
            extra[name] = measure_single(cfgx, dev, max(5, args.steps // 2), 3, world, peaks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 activations, fp16+int4 gs64 records, f32 accumulation",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) random-init experts and routers)",
            "config": headline_config(T, world, args.exchange),
            "int4_fp16_record_gbs": (rb["up"] + rb["down"]) / (ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": ("fused decode kernel (gate/up + SwiGLU + down + combine + cast, "
                                                    "one launch per layer)") if fused else
                         "gemv up (gate/up dequant GEMV + SwiGLU)",
                         "achieved": up_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": up_gbs / hbm_peak,
                         "peak_kind": peak_kind, "traffic": traffic, "traffic_source": traffic_src,
                         "bytes_per_launch": up_bytes_launch,
                         "launch_ms": up_ms, "down_achieved": dn_gbs, "down_launch_ms": dn_ms},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e_ms},
            "cpu_baseline": cpu,
            "gpu_launches": stack.launches_per_step() * args.steps,
            "clocks": clk,
            "sweep": sweep,
            "missing_pairs": miss,
            "ep_max_rel_err": ep_err,
            "ep_phase_ms_per_layer": ep_phases,
            "extra_configs": extra,
            "records_per_step": rb["records"], "pairs_per_step": rb["pairs"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        if stack.ep is not None:
            stack.ep.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
