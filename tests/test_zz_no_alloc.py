"""The workspace-free grouped-expert entry point (moeb200_grouped_ffn_noalloc) against the entry
point that takes a caller workspace (moeb200_grouped_ffn), through the C ABI (needs a B200).

The workspace-free call exists for callers that cannot allocate device scratch (a host binding the
C ABI with no device allocator, or code that must not call cudaMalloc); it keeps its scratch in one
static 1 MiB device array per GPU. This file is collected last so a failure here never hides the
other tests' results; it passes alone in a fresh process and after the rest of the suite.
Also checked: the largest call the array admits (and the next size refused), that a call allocates
no device memory, and the companion status call.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from moeb200 import _lib, ops
from moeb200 import format as F
from oracle import moe_oracle as O

from gpu_util import TOL, act_np, make_records

pytestmark = pytest.mark.gpu


def _table(lay, blobs, weights, dev):
    offs = F.field_offsets(lay)
    tab = torch.tensor([[b.data_ptr() + o for o in offs] for b in blobs], dtype=torch.int64, device=dev)
    w = torch.tensor(weights, dtype=torch.float32, device=dev)
    return tab, w


def _noalloc(lay_c, tab, w, x, out):
    _lib.check(_lib.lib().moeb200_grouped_ffn_noalloc(
        C.byref(lay_c), C.c_void_p(tab.data_ptr()), C.c_void_p(w.data_ptr()), tab.shape[0],
        C.c_void_p(x.data_ptr()), _lib.F16 if x.dtype == torch.float16 else _lib.BF16,
        C.c_void_p(out.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream)))


def test_noalloc_matches_workspace_entry_two_calls(cuda_dev):
    # two calls in a row on different records and tokens: the second must not see the first's scratch
    cases = [("int4", 2048, 1024, [0.3, 0.2, 0.15, 0.1, 0.1, 0.08, 0.05, 0.02], torch.float16, 11),
             ("int8", 2048, 512, [0.4, 0.0, 0.35, 0.25], torch.bfloat16, 12)]
    for prec, H, I, weights, dt, seed in cases:
        lay, blobs, nps = make_records(prec, H, I, len(weights), seed, cuda_dev)
        lay_c = F.to_c(lay)
        lay_c.off_gu_q = lay_c.off_gu_s = lay_c.off_dn_q = lay_c.off_dn_s = 0  # table holds field addresses
        tab, w = _table(lay, blobs, weights, cuda_dev)
        x = torch.randn(1, H, generator=torch.Generator(device=cuda_dev).manual_seed(seed), device=cuda_dev).to(dt)
        ref_out = torch.zeros(H, dtype=dt, device=cuda_dev)
        ops.grouped_ffn_table(lay_c, tab, w, x.reshape(-1), ref_out)
        out = torch.zeros(H, dtype=dt, device=cuda_dev)
        _noalloc(lay_c, tab, w, x.reshape(-1), out)
        torch.cuda.synchronize()
        err = O.max_rel_err(act_np(out), act_np(ref_out))
        assert err < TOL, (prec, err)
        # and both agree with the oracle
        assert O.max_rel_err(act_np(out), O.grouped_ffn(act_np(x), nps, lay, weights)[0]) < TOL


def test_noalloc_refuses_sizes_beyond_the_array(cuda_dev):
    lay_c = F.to_c(F.record_layout("int4", 2048, 1024))
    n = 1024  # 1024 experts x 1024 x 2 bytes of h alone (2 MiB) exceed the 1 MiB array
    dummy = torch.zeros(4, dtype=torch.int64, device=cuda_dev)
    rc = _lib.lib().moeb200_grouped_ffn_noalloc(C.byref(lay_c), C.c_void_p(dummy.data_ptr()),
                                                C.c_void_p(dummy.data_ptr()), n, C.c_void_p(dummy.data_ptr()),
                                                _lib.F16, C.c_void_p(dummy.data_ptr()), None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()[1]


def _largest_n(lay_c) -> int:
    L = _lib.lib()
    cap = _lib.NOALLOC_SCRATCH_BYTES
    n = 1
    while n < 4096 and L.moeb200_grouped_ffn_workspace(C.byref(lay_c), n + 1) <= cap:
        n += 1
    return n


def _status() -> int:
    st = C.c_int32(-1)
    _lib.check(_lib.lib().moeb200_noalloc_check_status(C.byref(st), C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return st.value


def test_noalloc_largest_call_and_next_refused(cuda_dev):
    # one-token items at the OLMoE shape: the largest n whose scratch fits the array runs and matches
    # the workspace entry point; n + 1 is refused before anything launches
    H, I = 2048, 1024
    lay = F.record_layout("int4", H, I)
    lay_c = F.to_c(lay)
    n = _largest_n(lay_c)
    assert n >= 8
    m = 6  # distinct records, repeated through the table (the kernels read records in place)
    lay, blobs, nps = make_records("int4", H, I, m, 21, cuda_dev)
    lay_c = F.to_c(lay)
    lay_c.off_gu_q = lay_c.off_gu_s = lay_c.off_dn_q = lay_c.off_dn_s = 0
    g = torch.Generator(device=cuda_dev).manual_seed(22)
    weights = (torch.rand(n, generator=g, device=cuda_dev) / n).tolist()
    tab, w = _table(lay, [blobs[i % m] for i in range(n)], weights, cuda_dev)
    x = torch.randn(H, generator=g, device=cuda_dev).half()
    ref_out = torch.zeros(H, dtype=torch.float16, device=cuda_dev)
    ops.grouped_ffn_table(lay_c, tab, w, x, ref_out)
    out = torch.zeros(H, dtype=torch.float16, device=cuda_dev)
    _noalloc(lay_c, tab, w, x, out)
    torch.cuda.synchronize()
    assert O.max_rel_err(act_np(out), act_np(ref_out)) < TOL, n
    assert _status() == 0
    big = torch.zeros(4 * (n + 1), dtype=torch.int64, device=cuda_dev)
    wb = torch.zeros(n + 1, dtype=torch.float32, device=cuda_dev)
    rc = _lib.lib().moeb200_grouped_ffn_noalloc(C.byref(lay_c), C.c_void_p(big.data_ptr()), C.c_void_p(wb.data_ptr()),
                                                n + 1, C.c_void_p(x.data_ptr()), _lib.F16,
                                                C.c_void_p(out.data_ptr()), None)
    assert rc == _lib.ERR_UNSUPPORTED, n + 1
    assert "scratch" in _lib.last_error()[1]


def test_noalloc_call_allocates_nothing(cuda_dev):
    H, I = 2048, 512
    lay, blobs, nps = make_records("int8", H, I, 4, 31, cuda_dev)
    lay_c = F.to_c(lay)
    lay_c.off_gu_q = lay_c.off_gu_s = lay_c.off_dn_q = lay_c.off_dn_s = 0
    tab, w = _table(lay, blobs, [0.4, 0.3, 0.2, 0.1], cuda_dev)
    x = torch.randn(H, generator=torch.Generator(device=cuda_dev).manual_seed(32), device=cuda_dev).half()
    out = torch.zeros(H, dtype=torch.float16, device=cuda_dev)
    _noalloc(lay_c, tab, w, x, out)  # warm: module load, address lookup, kernel attributes
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated(cuda_dev)
    free_before, _ = torch.cuda.mem_get_info(cuda_dev)
    for _ in range(3):
        _noalloc(lay_c, tab, w, x, out)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda_dev)
    assert torch.cuda.memory_allocated(cuda_dev) == torch_before
    assert free_after == free_before
    assert _status() == 0
