"""The workspace-free grouped-expert entry point (moeb200_grouped_ffn_noalloc) against the entry
point that takes a caller workspace (moeb200_grouped_ffn), through the C ABI (needs a B200).

The workspace-free call exists for callers that cannot allocate device scratch (a host binding the
C ABI with no device allocator, or code that must not call cudaMalloc); it keeps its scratch in one
static 1 MiB device array per GPU. This file is collected last so a failure here never hides the
other tests' results; it passes alone in a fresh process and after the rest of the suite.
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
