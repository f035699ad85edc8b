"""Generate the golden vectors that pin the oracle to the reference.

Run in the build container, where the reference (moelab) is importable from its read-only
checkout and transformers is installed:

    MOELAB_ROOT=<path to the moelab checkout> python tests/golden/make_golden.py

Everything here is computed by the reference's own code: moelab.quant.quantize,
moelab.store.record_layout / encode_record / materialize, moelab.runtime.expert_ffn and
MoERuntime._decide_general, moelab.policy.PrecisionPolicy, and the installed transformers
routers. Inputs are seeded; large inputs are not stored but regenerated from their torch seed
by the tests and checked against the SHA-256 recorded here.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, os.environ.get("MOELAB_ROOT", "/root/reference"))

from moelab.policy import PrecisionPolicy, level_to_precision  # noqa: E402
from moelab.quant import quantize  # noqa: E402
from moelab.runtime import MoERuntime, RunStats, expert_ffn  # noqa: E402
from moelab.store import encode_record, materialize, record_layout  # noqa: E402

out: dict[str, np.ndarray] = {}
meta: dict = {"layouts": {}, "hashes": {}, "cases": {}}


def sha(a) -> str:
    a = a.numpy() if isinstance(a, torch.Tensor) else a
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


# -- A. quantiser ---------------------------------------------------------------------------------
torch.manual_seed(0)
w = torch.randn(96, 256)
out["quant/w"] = w.numpy()
for bits in (4, 8):
    for method in ("absmax", "mse"):
        q, s = quantize(w, bits, 64, method)
        out[f"quant/q{bits}_{method}"] = q.numpy()
        out[f"quant/s{bits}_{method}"] = s.numpy()
# heavy-tailed groups: exercises the signed "max / -8" mse candidate (negative scales)
g = torch.Generator().manual_seed(5)
wt = torch.randn(64, 128, generator=g) * 0.02
wt[torch.rand(64, 128, generator=g) < 0.02] *= 25.0
out["quant/wt"] = wt.numpy()
q, s = quantize(wt, 4, 64, "mse")
out["quant/q4_mse_tail"], out["quant/s4_mse_tail"] = q.numpy(), s.numpy()

# -- B. records ------------------------------------------------------------------------------------
torch.manual_seed(1)
H, I = 128, 64
gu, dn = torch.randn(2 * I, H), torch.randn(H, I)
out["rec/gu"], out["rec/dn"] = gu.numpy(), dn.numpy()
for prec in ("fp32", "fp16", "bf16", "int8", "int4"):
    lay = record_layout(prec, H, I)
    meta["layouts"][f"{prec}_{H}_{I}"] = lay
    blob = encode_record(lay, gu, dn)
    out[f"rec/{prec}"] = blob
    g2, d2 = materialize(lay, torch.from_numpy(blob), torch.float32)
    out[f"rec/{prec}_gu_f32"], out[f"rec/{prec}_dn_f32"] = g2.numpy(), d2.numpy()
for (h, i) in ((2048, 1024), (2048, 768), (2048, 512)):
    for prec in ("int4", "int8", "fp16"):
        meta["layouts"][f"{prec}_{h}_{i}"] = record_layout(prec, h, i)

# -- C. grouped expert sums (tests/test_kernels.py:31-50 shapes and seeds) -------------------------
for (H, I) in ((64, 32), (96, 48), (512, 256), (256, 128)):
    for prec in ("int4", "int8", "fp16", "fp32"):
        torch.manual_seed(H + I)
        lay = record_layout(prec, H, I)
        recs = [torch.from_numpy(encode_record(lay, torch.randn(2 * I, H) * 0.1, torch.randn(H, I) * 0.1))
                for _ in range(3)]
        ws = [0.5, 0.3, 0.2]
        x = torch.randn(1, H)
        ref = torch.zeros(1, H)
        for b, wt_ in zip(recs, ws):
            g_, d_ = materialize(lay, b, torch.float32)
            gg, uu = F.linear(x, g_).chunk(2, -1)
            ref += wt_ * F.linear(F.silu(gg) * uu, d_)
        key = f"grp/{prec}_{H}_{I}"
        meta["cases"][key] = {"H": H, "I": I, "prec": prec, "seed": H + I, "ws": ws,
                              "recs_sha": [sha(b) for b in recs], "x_sha": sha(x)}
        out[key + "/ref"] = ref.numpy()
        if H <= 96:
            for j, b in enumerate(recs):
                out[f"{key}/rec{j}"] = b.numpy()
            out[key + "/x"] = x.numpy()

# -- D. HOBBIT levels ---------------------------------------------------------------------------------
g = torch.Generator().manual_seed(0)
wh = torch.rand(64, 8, generator=g) ** 3
out["hob/w"] = wh.numpy()
pols = {
    "t06": PrecisionPolicy("hobbit", t1=0.6),
    "t03_t209": PrecisionPolicy("hobbit", t1=0.3, t2=0.9),
    "t05_mid08": PrecisionPolicy("hobbit", t1=0.5, t_mid=0.8),
    "t04_mid07_t209": PrecisionPolicy("hobbit", t1=0.4, t_mid=0.7, t2=0.9),
    "hi": PrecisionPolicy("hi"),
    "lo": PrecisionPolicy("lo"),
}
for name, pol in pols.items():
    lvl, skip = pol.levels(0, wh)
    out[f"hob/{name}/lvl"] = lvl.numpy()
    out[f"hob/{name}/skip"] = skip.numpy()
out["hob/s"] = PrecisionPolicy("hobbit").unimportance(wh).numpy()
meta["hobbit"] = {"t06": [0.6, None, None], "t03_t209": [0.3, None, 0.9], "t05_mid08": [0.5, 0.8, None],
                  "t04_mid07_t209": [0.4, 0.7, 0.9]}

# -- E. dispatch: MoERuntime._decide_general on a stub runtime ------------------------------------------


class _Usage:
    def record(self, *a):
        pass


class _Store:
    precisions = ["fp16", "int8", "int4"]


class _Stub:
    pass


for case, (T, k, E, seed, pol) in {
    "d1": (37, 4, 16, 3, PrecisionPolicy("hobbit", t1=0.5, t_mid=0.8)),
    "d2": (64, 8, 64, 4, PrecisionPolicy("hobbit", t1=0.6, t2=0.9)),
    "d3": (1, 8, 64, 5, PrecisionPolicy("hobbit", t1=0.6)),
}.items():
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g)
    p = logits.softmax(-1)
    wv, idx = torch.topk(p, k, dim=-1)
    stub = _Stub()
    stub.stats, stub.store, stub.policy, stub.usage = RunStats(), _Store(), pol, _Usage()
    reqs, tok_cpu, tok_dev, w_dev, w_sorted = MoERuntime._decide_general(stub, 0, idx, wv, T, k, "cpu", None)
    lvl, skip = pol.levels(0, wv)
    flat_pos = torch.cat([torch.arange(T * k)[~skip.reshape(-1)]])
    keep = (~skip).reshape(-1)
    order = torch.argsort(idx.reshape(-1)[keep], stable=True)
    out[f"dsp/{case}/idx"] = idx.numpy()
    out[f"dsp/{case}/w"] = wv.numpy()
    out[f"dsp/{case}/lvl"] = lvl.numpy()
    out[f"dsp/{case}/skip"] = skip.numpy()
    out[f"dsp/{case}/tok"] = tok_cpu.numpy()
    out[f"dsp/{case}/w_sorted"] = w_sorted.numpy()
    out[f"dsp/{case}/experts"] = np.array([r.expert for r in reqs], np.int64)
    out[f"dsp/{case}/starts"] = np.array([r.sl.start for r in reqs], np.int64)
    out[f"dsp/{case}/stops"] = np.array([r.sl.stop for r in reqs], np.int64)
    out[f"dsp/{case}/vote_prec"] = np.array([["fp16", "int8", "int4"].index(r.prec) for r in reqs], np.int64)
    meta["cases"][f"dsp/{case}"] = {"T": T, "k": k, "E": E}

# -- F. routers (installed transformers) --------------------------------------------------------------
from transformers import OlmoeConfig, Qwen3MoeConfig  # noqa: E402
from transformers.models.olmoe.modeling_olmoe import OlmoeTopKRouter  # noqa: E402
from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeTopKRouter  # noqa: E402

for case, (cls, cfgcls, E, k, renorm, dt) in {
    "olmoe_f32": (OlmoeTopKRouter, OlmoeConfig, 16, 4, False, torch.float32),
    "qwen3_f32": (Qwen3MoeTopKRouter, Qwen3MoeConfig, 32, 8, True, torch.float32),
    "olmoe_bf16": (OlmoeTopKRouter, OlmoeConfig, 16, 4, False, torch.bfloat16),
}.items():
    cfg = cfgcls(hidden_size=64, num_experts=E, num_experts_per_tok=k, norm_topk_prob=renorm)
    r = cls(cfg)
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        r.weight.copy_(torch.randn(E, 64, generator=g) * 0.2)
    r = r.to(dt)
    h = torch.randn(24, 64, generator=g).to(dt)
    with torch.no_grad():
        probs, wts, ids = r(h)
    out[f"rt/{case}/h"] = h.float().numpy()
    out[f"rt/{case}/wr"] = r.weight.detach().float().numpy()
    out[f"rt/{case}/probs"] = probs.float().numpy()
    out[f"rt/{case}/w"] = wts.float().numpy()
    out[f"rt/{case}/idx"] = ids.numpy()
    meta["cases"][f"rt/{case}"] = {"E": E, "k": k, "renorm": renorm, "dtype": str(dt).split(".")[-1]}

# -- G. one small MoE layer through the reference's CPU expert path ------------------------------------
torch.manual_seed(11)
T, H, I, E, k = 5, 128, 64, 8, 3
precs = ["fp16", "int4"]
lays = {p: record_layout(p, H, I) for p in precs}
recs = {p: [] for p in precs}
for e in range(E):
    gu_, dn_ = torch.randn(2 * I, H) * 0.05, torch.randn(H, I) * 0.05
    for p in precs:
        recs[p].append(torch.from_numpy(encode_record(lays[p], gu_, dn_)))
x = torch.randn(T, H)
logits = torch.randn(T, E)
wv, idx = torch.topk(logits.softmax(-1), k, dim=-1)
lvl, skip = PrecisionPolicy("hobbit", t1=0.5).levels(0, wv)
ref = torch.zeros(T, H)
for t in range(T):
    for j in range(k):
        if skip[t, j]:
            continue
        p = level_to_precision(int(lvl[t, j]), precs)
        g_, d_ = materialize(lays[p], recs[p][int(idx[t, j])], torch.float32)
        ref[t] += float(wv[t, j]) * expert_ffn(x[t:t + 1], g_, d_, F.silu)[0]
out["layer/x"], out["layer/idx"], out["layer/w"] = x.numpy(), idx.numpy(), wv.numpy()
out["layer/lvl"], out["layer/ref"] = lvl.numpy(), ref.numpy()
for p in precs:
    out[f"layer/{p}"] = np.stack([b.numpy() for b in recs[p]])
meta["cases"]["layer"] = {"T": T, "H": H, "I": I, "E": E, "k": k, "precs": precs}

# -- dense int8 layers (moelab/denseq.py QLinear, CPU path: dequantize + F.linear) -----------------
from moelab.denseq import QLinear  # noqa: E402
from moelab.quant import dequantize  # noqa: E402

torch.manual_seed(13)
lin = torch.nn.Linear(256, 96, bias=True)
ql = QLinear.from_linear(lin, "cpu", 64)
out["dense/w"] = lin.weight.data.numpy()
out["dense/q"], out["dense/s"] = ql.q.numpy(), ql.s.numpy()
out["dense/bias"] = ql.bias.data.numpy()
for name, dt in (("fp16", torch.float16), ("bf16", torch.bfloat16)):
    out[f"dense/w_{name}"] = dequantize(ql.q, ql.s, 8, dt).view(torch.int16).numpy()
xd = torch.randn(3, 256)
out["dense/x"] = xd.numpy()
out["dense/y_f32"] = ql(xd).detach().numpy()
meta["cases"]["dense"] = {"O": 96, "K": 256, "gs": ql.group_size}

np.savez_compressed(HERE / "golden.npz", **out)
(HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1))
print("wrote", HERE / "golden.npz", sum(v.nbytes for v in out.values()) // 1024, "KiB raw")
