"""The bounded mbarrier wait inside every kernel of the library, run on a
barrier that nothing completes: it must give up after its limit (about 2 s),
report through the device status word, and leave the CUDA context usable --
a decode right afterwards still matches the oracle.  The failure is made the
way this library expects real ones (a lost arrival), not by faulting."""

import ctypes
import time

import pytest
import torch

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _lib
from mla_cases import D_QK, D_V, assert_close, build_dense

pytestmark = pytest.mark.gpu

FA_DEVICE_TIMEOUT_SELFTEST = 7   # include/flagattn_b200.h


def test_bounded_wait_reports_and_context_survives():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.time()
    st = _lib.lib().fa_selftest_wait_timeout(
        ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.FA_OK
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert int(status.item()) == FA_DEVICE_TIMEOUT_SELFTEST
    assert 0.5 < elapsed < 30, elapsed            # it waited, and it stopped waiting

    d = build_dense(24, [100, 700], heads=128)
    meta, splits = fa.get_mla_metadata(d["lens"], 128, 1)
    out, lse = fa.flash_mla_with_kvcache(d["q"], d["kc"], d["bt"], d["lens"], D_V, meta, splits,
                                         softmax_scale=D_QK ** -0.5)
    torch.cuda.synchronize()
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, D_QK ** -0.5)
    assert_close("out", out.float().cpu().numpy(), want_o)
    assert_close("lse", lse.cpu().numpy(), want_l)
