"""Host-side checks that need no GPU: the C ABI library loads and exports every declared symbol,
the record format matches the reference byte for byte, and bad arguments are refused before any
CUDA call."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import moeb200
from moeb200 import _lib
from moeb200 import format as F
from oracle import moe_oracle as O

ROOT = Path(__file__).resolve().parents[1]


def header_symbols() -> list[str]:
    text = (ROOT / "include" / "moeb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moeb200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(_lib.exported_symbols()), set(syms) ^ set(_lib.exported_symbols())
    assert L.moeb200_version().startswith(b"moeb200")


def test_no_cpu_fallback_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(_lib.MoeB200Error):
        _lib.lib()


@pytest.mark.parametrize("prec", ["fp32", "fp16", "bf16", "int8", "int4"])
@pytest.mark.parametrize("H,I", [(128, 64), (2048, 1024), (2048, 768), (2048, 512), (96, 48), (64, 32)])
def test_layout_matches_oracle(prec, H, I):
    assert F.record_layout(prec, H, I) == O.record_layout(prec, H, I)


def test_layout_to_c():
    lay = F.record_layout("int4", 2048, 1024)
    c = F.to_c(lay)
    assert (c.wtype, c.hidden, c.inter, c.gs_up, c.gs_dn) == (_lib.I4, 2048, 1024, 64, 64)
    assert (c.off_gu_q, c.off_gu_s, c.off_dn_q, c.off_dn_s, c.record_bytes) == (0, 2097152, 2228224, 3276800, 3342336)
    assert F.field_offsets(lay) == [0, 2097152, 2228224, 3276800]


@pytest.mark.parametrize("prec", ["fp32", "fp16", "bf16"])
def test_package_float_records_match_reference(golden, golden_meta, prec):
    lay = golden_meta["layouts"][f"{prec}_128_64"]
    blob = F.encode_record(lay, torch.from_numpy(golden["rec/gu"]), torch.from_numpy(golden["rec/dn"]))
    assert np.array_equal(blob.numpy(), golden[f"rec/{prec}"])


@pytest.mark.parametrize("prec", ["int8", "int4"])
def test_package_int_records_need_the_gpu_quantiser(golden_meta, prec):
    # integer records are quantised by the library's device kernel; there is no host quantiser in
    # the package (the oracle's numpy restatement is test-side only)
    lay = golden_meta["layouts"][f"{prec}_128_64"]
    with pytest.raises(ValueError, match="GPU"):
        F.encode_record(lay, torch.zeros(128, 128), torch.zeros(128, 64))


def test_invalid_arguments_refused_without_cuda():
    L = _lib.lib()
    t = _lib.ExpertTable()
    t.n_prec, t.num_experts = 1, 64
    t.layout[0] = F.to_c(F.record_layout("int4", 2048, 1024))
    rc = L.moeb200_experts_forward(C.byref(t), None, _lib.F16, 1, None, None, 8, None, None, None, None, None, 0, None)
    assert rc == _lib.ERR_INVALID
    assert "null" in _lib.last_error()[1]
    # group size 48 cannot be served by the int4 kernels: refused, never run
    lay = F.to_c(F.record_layout("int4", 96, 48))
    fake = C.c_void_p(256)
    rc = L.moeb200_grouped_ffn(C.byref(lay), fake, fake, 2, fake, _lib.F16, fake, fake, 1 << 20, None)
    assert rc == _lib.ERR_UNSUPPORTED, _lib.last_error()
    # fp32 activations are not tensor-core operands
    lay = F.to_c(F.record_layout("int4", 2048, 1024))
    rc = L.moeb200_grouped_ffn(C.byref(lay), fake, fake, 2, fake, _lib.F32, fake, fake, 1 << 20, None)
    assert rc == _lib.ERR_UNSUPPORTED
    # workspace too small
    rc = L.moeb200_grouped_ffn(C.byref(lay), fake, fake, 2, fake, _lib.F16, fake, fake, 16, None)
    assert rc == _lib.ERR_WORKSPACE
    # router: k > E
    rc = L.moeb200_router(fake, fake, None, _lib.F16, 1, 2048, 4, 8, 0, None, fake, fake, None, None, None, None,
                          fake, 1 << 20, None)
    assert rc == _lib.ERR_INVALID


def test_workspace_queries():
    L = _lib.lib()
    t = _lib.ExpertTable()
    t.n_prec, t.num_experts = 2, 64
    t.layout[0] = F.to_c(F.record_layout("fp16", 2048, 1024))
    t.layout[1] = F.to_c(F.record_layout("int4", 2048, 1024))
    a = L.moeb200_experts_workspace(C.byref(t), 1, 8)
    b = L.moeb200_experts_workspace(C.byref(t), 64, 8)
    assert 0 < a < b
    assert b >= 64 * 8 * 1024 * 2 + 64 * 2048 * 4  # h and acc scratch
    assert L.moeb200_dispatch_workspace(4096, 10, 512, 3) > 0
    assert L.moeb200_router_workspace(64, 512) >= 64 * 512 * 4


def test_modules_refuse_non_silu():
    lay = {"int4": F.record_layout("int4", 64, 32)}
    with pytest.raises(moeb200.MoeB200Error):
        rt = moeb200.B200Runtime.__new__(moeb200.B200Runtime)
        moeb200.B200Experts(rt, 0, torch.nn.GELU(), 8)
    assert lay


def test_policy_to_c():
    p = moeb200.PolicySpec("hobbit", t1=0.5, t2=0.9, protect_layers=frozenset({3}))
    c = p.to_c(0)
    assert (c.mode, round(c.t1, 6), c.t_mid, round(c.t2, 6)) == (2, 0.5, -1.0, 0.9)
    assert p.to_c(3).mode == 0
