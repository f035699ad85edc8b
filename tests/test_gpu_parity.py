"""CUDA path vs the oracle, through the C ABI (needs a B200)."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import moeb200
from moeb200 import _lib
from moeb200 import format as F
from moeb200 import ops
from moeb200.runtime import B200Runtime
from oracle import moe_oracle as O

from gpu_util import TOL, act_np, emulate_router_logits, layer_records, make_records

pytestmark = pytest.mark.gpu

ACTS = {"fp16": torch.float16, "bf16": torch.bfloat16}


# -- grouped expert sums: the reference kernel API (moelab/kernels.py:747-891) --------------------------
SHAPES = [(64, 32), (512, 256), (256, 128), (2048, 1024), (2048, 768), (2048, 512), (96, 48)]


@pytest.mark.parametrize("act", ["fp16", "bf16"])
@pytest.mark.parametrize("prec", ["int4", "int8", "fp16", "bf16", "fp32"])
@pytest.mark.parametrize("H,I", SHAPES)
def test_grouped_ffn_matches_oracle(cuda_dev, act, prec, H, I):
    dt = ACTS[act]
    if prec == "int4" and (H, I) == (96, 48):
        # group size 48 cannot hold whole 32-column int4 chunks: refused loudly
        lay, blobs, _ = make_records(prec, H, I, 2, 1, cuda_dev)
        x = torch.randn(1, H, device=cuda_dev).to(dt)
        with pytest.raises(moeb200.MoeB200Error):
            moeb200.grouped_ffn_int4(x, [(F.views(lay, b), 1.0) for b in blobs], lay["group_sizes"],
                                     torch.zeros(1, H, dtype=dt, device=cuda_dev))
        return
    lay, blobs, nps = make_records(prec, H, I, 4, H + I, cuda_dev, std=0.1 if H <= 512 else 0.02)
    ws = [0.5, 0.3, 0.0, 0.2]  # a zero weight is a no-op
    torch.manual_seed(H * I)
    x = torch.randn(1, H, device=cuda_dev).to(dt)
    ents = [(F.views(lay, b), w) for b, w in zip(blobs, ws)]
    ref = O.grouped_ffn(act_np(x), nps, lay, ws)
    out = torch.zeros(1, H, dtype=dt, device=cuda_dev)
    if prec == "int4":
        moeb200.grouped_ffn_int4(x, ents, lay["group_sizes"], out)
    elif prec == "int8":
        moeb200.grouped_ffn_int8(x, ents, lay, out)
    else:
        moeb200.grouped_ffn_float(x, ents, out)
    err = O.max_rel_err(act_np(out), ref)
    assert err < TOL, (prec, act, H, I, err)
    # add-into-out semantics (tests/test_kernels.py:42 pre-fills out with 0.5)
    out2 = torch.full((1, H), 0.5, dtype=dt, device=cuda_dev)
    if prec == "int4":
        moeb200.grouped_ffn_int4(x, ents, lay["group_sizes"], out2)
    elif prec == "int8":
        moeb200.grouped_ffn_int8(x, ents, lay, out2)
    else:
        moeb200.grouped_ffn_float(x, ents, out2)
    # out2 = round(0.5 + acc) vs 0.5 + round(acc): two roundings apart, each at most half an ulp
    # of its own magnitude (|acc| and |0.5 + acc|)
    expect = torch.full((1, H), 0.5, device=cuda_dev) + out.float()
    u = 2.0 ** -8 if dt == torch.bfloat16 else 2.0 ** -11
    tol = u * (out.float().abs() + expect.abs()) + 1e-6
    assert bool(((out2.float() - expect).abs() <= tol).all()), ((out2.float() - expect).abs() - tol).max()


def test_expert_ffn_int4_single(cuda_dev):
    lay, blobs, nps = make_records("int4", 2048, 1024, 1, 3, cuda_dev)
    x = torch.randn(1, 2048, device=cuda_dev).half()
    y = moeb200.expert_ffn_int4(x, F.views(lay, blobs[0]), lay["group_sizes"], torch.nn.SiLU())
    ref = O.grouped_ffn(act_np(x), nps, lay, [1.0])
    assert O.max_rel_err(act_np(y), ref) < TOL


# -- router -------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("act", ["fp16", "bf16"])
@pytest.mark.parametrize("T,E,k,renorm,bias", [(1, 64, 8, False, False), (37, 64, 8, False, False),
                                               (64, 128, 8, True, True), (5, 512, 10, True, True),
                                               (300, 512, 10, True, False),
                                               # prefill tiles (8 experts x 8 tokens per warp), full and ragged
                                               (2048, 128, 8, True, True), (600, 500, 10, True, False)])
def test_router_matches_oracle(cuda_dev, act, T, E, k, renorm, bias):
    dt = ACTS[act]
    H = 2048
    g = torch.Generator(device=cuda_dev).manual_seed(T * 7 + E)
    h = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    wr = (torch.randn(E, H, generator=g, device=cuda_dev) * 0.02).to(dt)
    b = torch.randn(E, generator=g, device=cuda_dev) if bias else None
    logits = torch.empty(T, E, device=cuda_dev)
    probs, w, idx, _, _ = ops.router(h, wr, k, renorm, b, logits=logits)
    dtn = {"fp16": "float16", "bf16": "bfloat16"}[act]
    hn, wn = act_np(h), act_np(wr)
    o_round, exact = O.router_logits_exact(hn, wn, dtn)
    gl = logits.cpu().numpy()
    # 1) the kernel computes exactly the documented fp32 order (bit-exact emulation)
    emu = emulate_router_logits(hn, wn, dtn)
    bad = np.argwhere(gl != emu)
    assert bad.size == 0, [(int(t), int(e), float(gl[t, e]), float(emu[t, e]), float(exact[t, e]))
                           for t, e in bad[:5]]
    # 2) that order differs from the correctly rounded logit only where the exact value lies within
    #    the order's worst-case error (69 roundings of at most 2^-24 of the partial magnitudes) of a
    #    rounding midpoint of the model dtype
    mism = gl != o_round
    if mism.any():
        absdot = np.abs(hn).astype(np.float64) @ np.abs(wn).astype(np.float64).T
        bound = 69 * 2.0 ** -24 * absdot
        mid = (gl.astype(np.float64) + o_round.astype(np.float64)) / 2
        assert np.all(np.abs(exact - mid)[mism] <= bound[mism]), "logit off by more than accumulation order"
    assert mism.mean() < 1e-2, mism.mean()
    # 2) softmax / top-k / renorm on the kernel's own logits: selection bit-exact (ties -> lower index)
    lb = gl + (b.cpu().numpy()[None, :] if b is not None else 0)
    o_probs, o_w, o_idx = O.topk_from_logits(lb.astype(np.float32), k, renorm)
    g_probs, g_w, g_idx = probs.cpu().numpy(), w.cpu().numpy(), idx.cpu().numpy()
    assert np.array_equal(g_idx, o_idx)
    assert np.allclose(g_w, o_w, rtol=1e-5, atol=1e-8)
    assert np.allclose(g_probs, o_probs, rtol=1e-5, atol=1e-9)


# -- levels -------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("spec", [dict(mode="hobbit", t1=0.6), dict(mode="hobbit", t1=0.3, t2=0.9),
                                  dict(mode="hobbit", t1=0.5, t_mid=0.8), dict(mode="threshold", thr=0.1),
                                  dict(mode="hi"), dict(mode="lo")])
def test_levels_bit_exact(cuda_dev, spec):
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    w = torch.rand(257, 8, generator=g, device=cuda_dev) ** 3
    pol = ops.PolicySpec(**spec)
    lvl, skip = ops.levels(w, pol.to_c())
    wn = w.cpu().numpy()
    if spec["mode"] == "threshold":
        o_l, o_s = O.threshold_levels(wn, spec["thr"])
    else:
        mode = {"hi": O.MODE_HI, "lo": O.MODE_LO, "hobbit": O.MODE_HOBBIT}[spec["mode"]]
        o_l, o_s = O.hobbit_levels(wn, mode, spec.get("t1", 0.6), spec.get("t_mid"), spec.get("t2"))
    assert np.array_equal(lvl.cpu().numpy(), o_l)
    assert np.array_equal(skip.cpu().numpy().astype(bool), o_s)


def test_levels_known_answer(cuda_dev):
    # reference tests/test_units.py:168-176
    w = torch.tensor([[0.1345, 0.1063, 0.0921, 0.0855, 0.0829, 0.0705, 0.0682, 0.0214]], device=cuda_dev)
    lvl, skip = ops.levels(w, ops.PolicySpec("hobbit", t1=0.6, t2=0.9).to_c())
    assert (lvl[0] == 0).tolist() == [True] * 4 + [False] * 4
    assert skip[0].tolist() == [0] * 7 + [1]


# -- dispatch -----------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,k,E,P", [(1, 8, 64, 1), (37, 4, 16, 3), (64, 8, 64, 2), (1024, 1, 4, 1), (2048, 8, 128, 1),
                                     (4096, 10, 512, 3), (3000, 10, 512, 2)])
def test_dispatch_bit_exact(cuda_dev, T, k, E, P):
    g = torch.Generator(device=cuda_dev).manual_seed(T + E)
    # zipf-like skew so some experts are hot and some empty
    logits = torch.randn(T, E, generator=g, device=cuda_dev) + torch.linspace(3, -3, E, device=cuda_dev)
    idx = torch.topk(logits, k, dim=-1).indices
    level = torch.randint(0, 3, (T, k), generator=g, device=cuda_dev).to(torch.uint8)
    skip = (torch.rand(T, k, generator=g, device=cuda_dev) < 0.1).to(torch.uint8)
    d = ops.dispatch(idx, level, skip, E, P)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), P))(level.cpu().numpy())
    o = O.dispatch(idx.cpu().numpy(), slot, skip.cpu().numpy().astype(bool), E, P)
    n = int(d["n_kept"].item())
    assert n == len(o["pos_e"])
    assert np.array_equal(d["counts_e"].cpu().numpy(), o["counts_e"])
    assert np.array_equal(d["counts_k"].cpu().numpy(), o["counts_k"])
    assert np.array_equal(d["pos_e"].cpu().numpy()[:n], o["pos_e"])
    assert np.array_equal(d["pos_k"].cpu().numpy()[:n], o["pos_k"])


def test_dispatch_matches_reference_decide_general(cuda_dev, golden, golden_meta):
    for case in ("d1", "d2", "d3"):
        m = golden_meta["cases"][f"dsp/{case}"]
        idx = torch.from_numpy(golden[f"dsp/{case}/idx"]).to(cuda_dev)
        skip = torch.from_numpy(golden[f"dsp/{case}/skip"].astype(np.uint8)).to(cuda_dev)
        d = ops.dispatch(idx, None, skip, m["E"], 1)
        n = int(d["n_kept"].item())
        assert np.array_equal(d["pos_e"].cpu().numpy()[:n] // m["k"], golden[f"dsp/{case}/tok"])


@pytest.mark.parametrize("T,k,E", [(1, 8, 64), (37, 4, 16), (256, 10, 512), (2048, 8, 128)])
def test_levels_vote_matches_oracle(cuda_dev, T, k, E):
    g = np.random.default_rng(T * 7 + E)
    idx = np.stack([g.choice(E, k, replace=False) for _ in range(T)]).astype(np.int64)
    lvl = g.integers(0, 3, (T, k)).astype(np.uint8)
    skip = g.random((T, k)) < 0.1
    for hv in (0.5, 0.3, 1.0):
        _, ref = O.expert_vote(idx, lvl, skip, E, hv)
        level = torch.from_numpy(lvl.copy()).to(cuda_dev)
        ops.levels_vote(torch.from_numpy(idx).to(cuda_dev), level, torch.from_numpy(skip.astype(np.uint8)).to(cuda_dev),
                        E, hv)
        assert np.array_equal(level.cpu().numpy(), ref), hv


def test_levels_vote_matches_reference_goldens(cuda_dev, golden, golden_meta):
    for case in ("d1", "d2", "d3"):
        m = golden_meta["cases"][f"dsp/{case}"]
        idx, skip, lvl = golden[f"dsp/{case}/idx"], golden[f"dsp/{case}/skip"], golden[f"dsp/{case}/lvl"]
        level = torch.from_numpy(lvl.astype(np.uint8)).to(cuda_dev)
        ops.levels_vote(torch.from_numpy(idx).to(cuda_dev), level, torch.from_numpy(skip.astype(np.uint8)).to(cuda_dev),
                        m["E"], 0.5)
        got = level.cpu().numpy()
        experts = golden[f"dsp/{case}/experts"]
        keep = ~skip.astype(bool)
        for e, prec in zip(experts, golden[f"dsp/{case}/vote_prec"]):
            sel = keep & (idx == e)
            assert set(O.level_to_slot(int(v), 3) for v in got[sel]) == {int(prec)}, (case, e)


def test_layer_with_per_expert_vote_matches_oracle(cuda_dev):
    H, I, E, k, T = 2048, 512, 32, 8, 48
    precs = ["fp16", "int8", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=41, device=cuda_dev, std=0.02)
    pol = ops.PolicySpec("hobbit", t1=0.5, t_mid=0.8, hi_vote=0.5)
    rt = B200Runtime(precs, lays, E, cuda_dev, pol, layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    g = torch.Generator(device=cuda_dev).manual_seed(8)
    x = torch.randn(T, H, generator=g, device=cuda_dev).half()
    wv, idx = torch.topk(torch.randn(T, E, generator=g, device=cuda_dev).softmax(-1), k, dim=-1)
    out = rt.run_layer(0, x, idx, wv, torch.nn.SiLU())
    lv0, sk0 = O.hobbit_levels(wv.cpu().numpy(), t1=0.5, t_mid=0.8)
    _, lv = O.expert_vote(idx.cpu().numpy(), lv0, sk0, E, 0.5)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), 3))(lv.astype(np.int64))
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, sk0, recs_np, [lays[p] for p in precs], E)
    assert O.max_rel_err(act_np(out), ref) < TOL
    # the vote changed some pairs' precision (otherwise this test proves nothing)
    assert not np.array_equal(lv, lv0)


# -- the experts module: whole MoE layer ------------------------------------------------------------------------
LAYER_CASES = [
    # (name, H, I, E, k, T, precs, policy, act)
    ("olmoe_c0_T1", 2048, 1024, 64, 8, 1, ["int4"], dict(mode="lo"), "fp16"),
    ("olmoe_c1_T8_thr", 2048, 1024, 64, 8, 8, ["fp16", "int4"], dict(mode="threshold", thr=0.1), "fp16"),
    ("olmoe_c1_T64_hobbit", 2048, 1024, 64, 8, 64, ["fp16", "int4"], dict(mode="hobbit", t1=0.6), "fp16"),
    ("qwen3next_T1_int8_int4", 2048, 512, 512, 10, 1, ["int8", "int4"], dict(mode="hobbit", t1=0.6), "bf16"),
    ("qwen3next_T256_mix", 2048, 512, 512, 10, 256, ["fp16", "int4"], dict(mode="threshold", thr=0.05), "fp16"),
    ("qwen3_30b_T512", 2048, 768, 128, 8, 512, ["int4"], dict(mode="lo"), "bf16"),
    ("tiny_3prec", 64, 32, 8, 3, 5, ["fp16", "int8", "int4"], dict(mode="hobbit", t1=0.5, t_mid=0.8), "fp16"),
]


def _run_on_path(path, fn):
    """fn() with the expert-product path forced; a shape the fused decode kernel does not take is
    skipped (the automatic path would use the grouped GEMV there)."""
    ops.set_path(path)
    try:
        return fn()
    except _lib.MoeB200Error as exc:
        if path in ("decode", "ws") and exc.code == _lib.ERR_UNSUPPORTED:
            pytest.skip(f"layout not taken by the {path} path")
        raise
    finally:
        ops.set_path("auto")


@pytest.mark.parametrize("path", ["gemv", "decode", "ws"])
@pytest.mark.parametrize("case", LAYER_CASES, ids=[c[0] for c in LAYER_CASES])
def test_experts_forward_matches_oracle(cuda_dev, case, path):
    name, H, I, E, k, T, precs, pol, act = case
    dt = ACTS[act]
    lays, recs = layer_records(precs, H, I, E, seed=zlib.crc32(name.encode()) % 1000, device=cuda_dev, std=0.02 if H > 64 else 0.05)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec(**pol), layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    x = torch.randn(T, H, generator=g, device=cuda_dev).to(dt)
    logits = torch.randn(T, E, generator=g, device=cuda_dev)
    wv, idx = torch.topk(logits.softmax(-1), k, dim=-1)
    out = _run_on_path(path, lambda: rt.run_layer(0, x, idx, wv, torch.nn.SiLU()))
    lvl, skip = rt.levels(0, wv)
    P = len(precs)
    lv = np.zeros((T, k), np.int64) if lvl is None else lvl.cpu().numpy().astype(np.int64)
    sk = None if skip is None else skip.cpu().numpy().astype(bool)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), P))(lv)
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, sk, recs_np, [lays[p] for p in precs], E)
    err = O.max_rel_err(act_np(out), ref)
    assert err < TOL, (name, err)
    assert int(rt.miss.item()) == 0


@pytest.mark.parametrize("path", ["gemv", "decode", "ws"])
def test_calls_in_a_row_reuse_the_workspace(cuda_dev, path):
    # The GEMV job counters and the split-K arrival counters (decode kernel: unit claims, per-item
    # and per-row-block counters) live in the workspace and are zeroed by the kernel that writes each
    # call's items: T = 1 (K split), T = 64 (jobs drawn from the counter), then T = 3 and T = 1 again
    # on the same workspace must each match the oracle.
    H, I, E, k = 2048, 1024, 64, 8
    precs = ["fp16", "int4"]
    lays, recs = layer_records(precs, H, I, E, seed=77, device=cuda_dev, std=0.02)
    rt = B200Runtime(precs, lays, E, cuda_dev, ops.PolicySpec("threshold", thr=0.1), layers=[0])
    for p in precs:
        for e in range(E):
            rt.add_record(0, e, p, recs[p][e])
    recs_np = [[b.cpu().numpy() for b in recs[p]] for p in precs]
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    ops.set_path(path)
    try:
        for T in (1, 64, 3, 1):
            x = torch.randn(T, H, generator=g, device=cuda_dev).half()
            logits = torch.randn(T, E, generator=g, device=cuda_dev)
            wv, idx = torch.topk(logits.softmax(-1), k, dim=-1)
            out = rt.run_layer(0, x, idx, wv, torch.nn.SiLU())
            lvl, skip = rt.levels(0, wv)
            lv = np.zeros((T, k), np.int64) if lvl is None else lvl.cpu().numpy().astype(np.int64)
            sk = None if skip is None else skip.cpu().numpy().astype(bool)
            slot = np.vectorize(lambda v: O.level_to_slot(int(v), 2))(lv)
            ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), slot, sk, recs_np,
                              [lays[p] for p in precs], E)
            err = O.max_rel_err(act_np(out), ref)
            assert err < TOL, (T, err)
    finally:
        ops.set_path("auto")


def test_missing_expert_counted_and_skipped(cuda_dev):
    H, I, E, k, T = 256, 128, 16, 4, 6
    lays, recs = layer_records(["int4"], H, I, E, seed=9, device=cuda_dev, std=0.05)
    rt = B200Runtime(["int4"], lays, E, cuda_dev, ops.PolicySpec("lo"), layers=[0])
    for e in range(E):
        if e != 3:
            rt.add_record(0, e, "int4", recs["int4"][e])
    x = torch.randn(T, H, device=cuda_dev).half()
    idx = torch.tensor([[3, 1, 2, 4]] * T, device=cuda_dev)
    wv = torch.full((T, k), 0.25, device=cuda_dev)
    out = rt.run_layer(0, x, idx, wv)
    assert int(rt.miss.item()) == T
    skip = (idx == 3).cpu().numpy()
    ref = O.moe_layer(act_np(x), idx.cpu().numpy(), wv.cpu().numpy(), None, skip,
                      [[b.cpu().numpy() for b in recs["int4"]]], [lays["int4"]], E)
    assert O.max_rel_err(act_np(out), ref) < TOL


@pytest.mark.parametrize("path", ["gemv", "decode", "ws"])
def test_every_pair_skipped_gives_zero_output(cuda_dev, path):
    # no work item at all: the output must still be written (zeros), on every path
    H, I, E, k, T = 2048, 512, 16, 4, 3
    lays, recs = layer_records(["int4"], H, I, E, seed=4, device=cuda_dev, std=0.02)
    rt = B200Runtime(["int4"], lays, E, cuda_dev, ops.PolicySpec("lo"), layers=[0])
    for e in range(E):
        rt.add_record(0, e, "int4", recs["int4"][e])
    x = torch.randn(T, H, device=cuda_dev).half()
    idx = torch.arange(k, device=cuda_dev).repeat(T, 1)
    wv = torch.full((T, k), 0.25, device=cuda_dev)
    skip = torch.ones(T, k, dtype=torch.uint8, device=cuda_dev)
    out = torch.full((T, H), 7.0, dtype=torch.float16, device=cuda_dev)
    _run_on_path(path, lambda: rt.run_layer(0, x, idx, wv, out=out, level=torch.zeros_like(skip), skip=skip))
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
