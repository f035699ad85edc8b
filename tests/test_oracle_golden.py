"""The oracle against the reference's golden vectors and its tests' known answers (CPU only)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import moe_oracle as O


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


# -- format --------------------------------------------------------------------------------------
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("method", ["absmax", "mse"])
def test_quantize_matches_reference(golden, bits, method):
    q, s = O.quantize(golden["quant/w"], bits, 64, method)
    assert np.array_equal(q, golden[f"quant/q{bits}_{method}"])
    assert np.array_equal(s.view(np.uint16), golden[f"quant/s{bits}_{method}"].view(np.uint16))


def test_quantize_mse_negative_scales_match_reference(golden):
    q, s = O.quantize(golden["quant/wt"], 4, 64, "mse")
    ref_s = golden["quant/s4_mse_tail"]
    assert (ref_s.astype(np.float32) < 0).any(), "fixture should contain signed '/-8' scales"
    assert np.array_equal(q, golden["quant/q4_mse_tail"])
    assert np.array_equal(s.view(np.uint16), ref_s.view(np.uint16))


def test_int4_packing_order_known_answer():
    # reference tests/test_units.py:33-38
    w = np.zeros((1, 64), np.float32)
    w[0, 0], w[0, 1] = 7.0, -7.0
    q, s = O.quantize(w, 4, 64)
    assert q[0, 0] == (7 + 8) | ((-7 + 8) << 4)
    assert np.array_equal(O.dequantize(q, s, 4)[0, :2], np.array([7.0, -7.0], np.float32))


def test_zero_group_and_group_size_known_answer():
    # reference tests/test_units.py:41-45
    q, s = O.quantize(np.zeros((4, 64), np.float32), 4, 64)
    assert np.array_equal(O.dequantize(q, s, 4), np.zeros((4, 64), np.float32))
    assert O.pick_group_size(1024) == 64 and O.pick_group_size(32) == 32 and O.pick_group_size(768) == 64


@pytest.mark.parametrize("bits,tol", [(8, 0.008), (4, 0.12)])
def test_quant_roundtrip_bound(golden, bits, tol):
    # reference tests/test_units.py:19-30
    w = golden["quant/w"]
    q, s = O.quantize(w, bits, 64)
    back = O.dequantize(q, s, bits)
    assert np.linalg.norm(back - w) / np.linalg.norm(w) < tol


def test_layouts_match_reference(golden_meta):
    for key, lay in golden_meta["layouts"].items():
        prec, h, i = key.split("_")
        mine = O.record_layout(prec, int(h), int(i))
        assert mine == lay, key
    # record sizes quoted for the configs
    assert O.record_layout("int4", 2048, 1024)["record_bytes"] == 3342336
    assert O.record_layout("int8", 2048, 1024)["record_bytes"] == 6488064
    assert O.record_layout("fp16", 2048, 1024)["record_bytes"] == 12582912
    assert O.record_layout("int4", 2048, 768)["record_bytes"] == 2506752
    assert O.record_layout("int4", 2048, 512)["record_bytes"] == 1671168
    assert O.record_layout("int8", 2048, 512)["record_bytes"] == 3244032


@pytest.mark.parametrize("prec", ["fp32", "fp16", "bf16", "int8", "int4"])
def test_records_match_reference(golden, golden_meta, prec):
    lay = golden_meta["layouts"][f"{prec}_128_64"]
    blob = O.encode_record(lay, golden["rec/gu"], golden["rec/dn"])
    assert np.array_equal(blob, golden[f"rec/{prec}"])
    g2, d2 = O.materialize_f32(lay, golden[f"rec/{prec}"])
    assert np.array_equal(g2, golden[f"rec/{prec}_gu_f32"])
    assert np.array_equal(d2, golden[f"rec/{prec}_dn_f32"])


# -- grouped expert sums ---------------------------------------------------------------------------
def _regen_group_case(meta):
    """Inputs of tests/test_kernels.py:34-38, regenerated from their torch seed and pinned by hash."""
    import torch

    H, I, prec = meta["H"], meta["I"], meta["prec"]
    torch.manual_seed(meta["seed"])
    lay = O.record_layout(prec, H, I)
    recs = []
    for _ in range(3):
        gu = (torch.randn(2 * I, H) * 0.1).numpy()
        dn = (torch.randn(H, I) * 0.1).numpy()
        recs.append(O.encode_record(lay, gu, dn))
    x = torch.randn(1, H).numpy()
    return lay, recs, x


def test_grouped_ffn_matches_reference(golden, golden_meta):
    for key, meta in golden_meta["cases"].items():
        if not key.startswith("grp/"):
            continue
        lay, recs, x = _regen_group_case(meta)
        assert [_sha(b) for b in recs] == meta["recs_sha"], f"{key}: regenerated records differ"
        assert _sha(x) == meta["x_sha"]
        got = O.grouped_ffn(x, recs, lay, meta["ws"])
        err = O.max_rel_err(got, golden[key + "/ref"])
        assert err < 1e-5, (key, err)


# -- HOBBIT mask -------------------------------------------------------------------------------------
def test_hobbit_known_answer():
    # reference tests/test_units.py:168-176
    w = np.array([[0.1345, 0.1063, 0.0921, 0.0855, 0.0829, 0.0705, 0.0682, 0.0214]], np.float32)
    s = O.unimportance(w)[0]
    assert np.allclose(s, [0.0, 0.2034, 0.3641, 0.5034, 0.6327, 0.7580, 0.8646, 0.9677], atol=2e-4)
    lvl, skip = O.hobbit_levels(w, O.MODE_HOBBIT, t1=0.6, t2=0.9)
    assert (lvl[0] == 0).tolist() == [True] * 4 + [False] * 4
    assert skip[0].tolist() == [False] * 7 + [True]
    lvl, _ = O.hobbit_levels(np.array([[0.05, 0.6, 0.35]], np.float32), O.MODE_HOBBIT, t1=0.6)
    assert (lvl[0] == 0).tolist() == [False, True, True]


def test_hobbit_levels_match_reference(golden, golden_meta):
    w = golden["hob/w"]
    assert np.allclose(O.unimportance(w), golden["hob/s"], atol=1e-6)
    for name, (t1, tm, t2) in golden_meta["hobbit"].items():
        lvl, skip = O.hobbit_levels(w, O.MODE_HOBBIT, t1, tm, t2)
        assert np.array_equal(lvl, golden[f"hob/{name}/lvl"].astype(np.uint8)), name
        assert np.array_equal(skip, golden[f"hob/{name}/skip"]), name
    lvl, _ = O.hobbit_levels(w, O.MODE_HI)
    assert np.array_equal(lvl, golden["hob/hi/lvl"].astype(np.uint8))
    lvl, _ = O.hobbit_levels(w, O.MODE_LO)
    assert np.array_equal(lvl, golden["hob/lo/lvl"].astype(np.uint8))


# -- dispatch ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["d1", "d2", "d3"])
def test_dispatch_matches_reference_decide_general(golden, golden_meta, case):
    m = golden_meta["cases"][f"dsp/{case}"]
    T, k, E = m["T"], m["k"], m["E"]
    idx, skip = golden[f"dsp/{case}/idx"], golden[f"dsp/{case}/skip"]
    d = O.dispatch(idx, None, skip, E, 1)
    # the reference's token list (flat positions // k, stable by expert)
    assert np.array_equal(d["pos_e"] // k, golden[f"dsp/{case}/tok"])
    experts = golden[f"dsp/{case}/experts"]
    starts, stops = golden[f"dsp/{case}/starts"], golden[f"dsp/{case}/stops"]
    nz = np.nonzero(d["counts_e"])[0]
    assert np.array_equal(nz, experts)
    off = np.concatenate([[0], np.cumsum(d["counts_e"])])
    assert np.array_equal(off[experts], starts) and np.array_equal(off[experts + 1], stops)
    w = golden[f"dsp/{case}/w"].reshape(-1)
    assert np.array_equal(w[d["pos_e"]], golden[f"dsp/{case}/w_sorted"])


@pytest.mark.parametrize("case", ["d1", "d2", "d3"])
def test_expert_vote_matches_reference_decide_general(golden, golden_meta, case):
    # the reference votes one precision per expert (hi_vote 0.5) over its 3-precision store
    m = golden_meta["cases"][f"dsp/{case}"]
    idx, skip, lvl = golden[f"dsp/{case}/idx"], golden[f"dsp/{case}/skip"], golden[f"dsp/{case}/lvl"]
    vote, per_pair = O.expert_vote(idx, lvl, skip, m["E"], 0.5)
    experts = golden[f"dsp/{case}/experts"]
    assert np.array_equal(np.nonzero(vote >= 0)[0], experts)
    got = [O.level_to_slot(int(v), 3) for v in vote[experts]]
    assert got == golden[f"dsp/{case}/vote_prec"].tolist()
    keep = ~skip.astype(bool)
    assert np.array_equal(per_pair[keep], vote[idx[keep]].astype(np.uint8))
    assert np.array_equal(per_pair[~keep], lvl.astype(np.uint8)[~keep])


def test_expert_vote_known_answers():
    # expert 0: levels 0, 0, 2 -> 2 of 3 at <= 0 >= 1.5 -> 0; expert 1: 1, 2 -> 1 of 2 at <= 1 -> 1;
    # expert 2: 2, 2, 0 (last skipped) -> 2; expert 3: no pair -> -1
    idx = np.array([[0, 1, 2], [0, 1, 2], [0, 2, 2]])
    lvl = np.array([[0, 1, 2], [0, 2, 2], [2, 2, 0]])
    skip = np.array([[0, 0, 0], [0, 0, 0], [0, 0, 1]], bool)
    vote, per_pair = O.expert_vote(idx, lvl, skip, 4, 0.5)
    assert vote.tolist() == [0, 1, 2, -1]
    assert per_pair.tolist() == [[0, 1, 2], [0, 1, 2], [0, 2, 0]]
    # hi_vote 1.0: every pair of the expert must ask for the level
    vote, _ = O.expert_vote(idx, lvl, skip, 4, 1.0)
    assert vote.tolist() == [2, 2, 2, -1]


# -- router -----------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["olmoe_f32", "qwen3_f32", "olmoe_bf16"])
def test_router_matches_transformers(golden, golden_meta, case):
    m = golden_meta["cases"][f"rt/{case}"]
    h, wr = golden[f"rt/{case}/h"], golden[f"rt/{case}/wr"]
    probs, w, idx, logits = O.router(h, wr, m["k"], m["renorm"], m["dtype"])
    ref_idx = golden[f"rt/{case}/idx"]
    for t in range(idx.shape[0]):
        if np.array_equal(idx[t], ref_idx[t]):
            continue
        # torch.topk's order among exactly equal logits is unspecified; the build fixes it as
        # lower index first. A difference is only allowed inside a run of equal logits.
        assert sorted(idx[t]) == sorted(ref_idx[t]), (t, idx[t], ref_idx[t])
        assert np.array_equal(logits[t][idx[t]], logits[t][ref_idx[t]]), (t, idx[t], ref_idx[t])
        for a in range(len(idx[t]) - 1):
            if logits[t][idx[t][a]] == logits[t][idx[t][a + 1]]:
                assert idx[t][a] < idx[t][a + 1]
        w_ref = golden[f"rt/{case}/w"][t]
        assert np.allclose(np.sort(w[t]), np.sort(w_ref), rtol=1e-5, atol=1e-7)
    same = (idx == ref_idx).all(axis=1)
    assert np.allclose(w[same], golden[f"rt/{case}/w"][same], rtol=1e-5, atol=1e-7)
    assert np.allclose(probs, golden[f"rt/{case}/probs"], rtol=1e-5, atol=1e-7)


# -- whole layer ------------------------------------------------------------------------------------------
def test_layer_matches_reference_cpu_path(golden, golden_meta):
    m = golden_meta["cases"]["layer"]
    precs = m["precs"]
    lays = [O.record_layout(p, m["H"], m["I"]) for p in precs]
    recs = [list(golden[f"layer/{p}"]) for p in precs]
    lvl = golden["layer/lvl"].astype(np.int64)
    slot = np.vectorize(lambda v: O.level_to_slot(int(v), len(precs)))(lvl)
    got = O.moe_layer(golden["layer/x"], golden["layer/idx"], golden["layer/w"], slot, None, recs, lays, m["E"])
    assert O.max_rel_err(got, golden["layer/ref"]) < 1e-5


# -- dense int8 layers --------------------------------------------------------------------------------
@pytest.mark.parametrize("name,dt", [("fp16", "float16"), ("bf16", "bfloat16")])
def test_dense_dequant_matches_reference(golden, name, dt):
    got = O.dense_int8_dequant(golden["dense/q"], golden["dense/s"], dt)
    ref = golden[f"dense/w_{name}"]  # moelab dequantize(q, s, 8, dtype) bit patterns
    bits = got.astype(np.float16).view(np.int16) if dt == "float16" else (O.f32_to_bf16_bits(got)).view(np.int16)
    assert np.array_equal(bits, ref)


def test_dense_linear_matches_reference_qlinear(golden):
    q = golden["dense/q"]
    # the oracle in float32 activations: the reference QLinear on the CPU (dequantise + F.linear)
    got = O.dense_int8_linear(golden["dense/x"], q, golden["dense/s"], golden["dense/bias"], "float32")
    ref = golden["dense/y_f32"]
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


def test_dense_quantize_matches_reference(golden):
    # QLinear.from_linear (denseq.py:81-87) quantises with absmax scales: quant.quantize(w, 8, gs)
    q, s = O.quantize(golden["dense/w"], 8, 64, "absmax")
    assert np.array_equal(q, golden["dense/q"])
    assert np.array_equal(s.view(np.uint16), golden["dense/s"].view(np.uint16))
