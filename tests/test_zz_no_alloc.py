"""fa_mla_decode_static_workspace: MLA decode for callers that cannot allocate.

Serving engines that reserve nearly all device memory for their KV-cache pool,
and plugin / FFI hosts that receive device pointers but no allocator, cannot
provide the split workspace fa_mla_decode needs.  This entry point takes that
scratch from a fixed device array inside the library instead.  The test calls
it through the C ABI with no workspace pointers at all and checks it against
fa_mla_decode (which uses a caller-provided workspace), on two calls in a row
with different inputs: both run the same kernels on the same partition of
the work, so the results must be bit-identical.  The file
name sorts last so a run that stops at the first failure has already run
every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

import flagattention_b200 as fa
from flagattention_b200 import _lib
from flagattention_b200 import _torch as fat
from flagattention_b200.mla import MlaCall
from mla_cases import D_V, build_dense

pytestmark = pytest.mark.gpu


def _prepared(seed, lens, parts):
    d = build_dense(seed, lens, heads=128)
    meta, splits = fa.get_mla_metadata(d["lens"], 128, 1, num_sm_parts_override=parts)
    kc = d["kc"]

    def call(out, lse):
        return MlaCall(d["q"], kc, kc.stride(0), kc.stride(1), kc.shape[0], kc.shape[1],
                       d["bt"], d["lens"], 0, meta, splits, out, lse, 576 ** -0.5)
    return d, call


def _static_decode(call):
    a = _lib.MlaArgs.from_buffer_copy(call.args)
    a.part_o = None              # the entry point must not need a workspace
    a.part_lse = None
    st = _lib.lib().fa_mla_decode_static_workspace(ctypes.byref(a), fat.stream_of(call._keep[0]))
    _lib.check(st, "fa_mla_decode_static_workspace")


def test_static_workspace_matches_workspace_entry_point_twice():
    # lengths and part counts chosen so several sequences are split across
    # parts: the combine then reads partials from the static array
    cases = [(31, [1, 700, 3000, 64, 4100], 9), (32, [5000, 17, 2500, 129], 13)]
    for seed, lens, parts in cases:
        d, call = _prepared(seed, lens, parts)
        B = len(lens)
        ref_o = torch.empty((B, 1, 128, D_V), dtype=torch.bfloat16, device="cuda")
        ref_l = torch.empty((B, 128, 1), dtype=torch.float32, device="cuda")
        call(ref_o, ref_l).run()
        out = torch.full((B, 1, 128, D_V), float("nan"), dtype=torch.bfloat16, device="cuda")
        lse = torch.full((B, 128, 1), float("nan"), dtype=torch.float32, device="cuda")
        _static_decode(call(out, lse))
        torch.cuda.synchronize()
        assert fat.read_status(torch.device("cuda")) == 0
        assert torch.equal(out, ref_o), "static-workspace output differs from fa_mla_decode"
        assert torch.equal(lse, ref_l), "static-workspace LSE differs from fa_mla_decode"


def test_static_workspace_rejects_oversized_call():
    d, call = _prepared(33, [100], 2)
    a = _lib.MlaArgs.from_buffer_copy(call(torch.empty((1, 1, 128, D_V), dtype=torch.bfloat16,
                                                       device="cuda"),
                                           torch.empty((1, 128, 1), dtype=torch.float32,
                                                       device="cuda")).args)
    a.batch = 1 << 20            # far more split scratch than the fixed array holds
    st = _lib.lib().fa_mla_decode_static_workspace(ctypes.byref(a), None)
    assert st == _lib.FA_ERR_INVALID_ARGUMENT
    assert b"static workspace too small" in _lib.lib().fa_last_error()
