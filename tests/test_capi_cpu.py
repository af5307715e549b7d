"""The C-ABI library loads and exports what include/*.h declares (CPU only).

Only pure host functions are called here (the reference's split heuristics);
nothing touches a GPU.
"""

import ctypes
import glob
import json
import os
import re

import pytest

from flagattention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(fa_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _declared_functions()
    assert len(declared) >= 15
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(declared) == bound, set(declared) ^ bound


def test_version_and_status_strings():
    lib = _lib.lib()
    assert lib.fa_version() == 0x000300
    assert lib.fa_status_string(0) == b"ok"
    assert lib.fa_status_string(-1) == b"invalid argument"


@pytest.fixture(scope="module")
def heuristics():
    with open(os.path.join(ROOT, "tests", "golden", "heuristics.json")) as f:
        return json.load(f)


def test_paged_rule_matches_reference_through_abi(heuristics):
    lib = _lib.lib()
    ns, ps = ctypes.c_int32(), ctypes.c_int32()
    for seqs, hkv, ctx, blk, sms, req, want_ns, want_ps in heuristics["paged_rule"]:
        assert lib.fa_paged_num_splits(seqs, hkv, ctx, blk, sms, req, ctypes.byref(ns),
                                       ctypes.byref(ps)) == 0
        assert ns.value == want_ns, (seqs, hkv, ctx, blk, sms, req)
        if want_ns > 1:
            assert ps.value == want_ps, (seqs, hkv, ctx, blk, sms, req)


def test_split_kv_heuristic_matches_reference_through_abi(heuristics):
    lib = _lib.lib()
    out = ctypes.c_int32()
    for B, H, M, N, bm, bn, sms, mx, want in heuristics["split_kv"]:
        assert lib.fa_split_kv_num_splits(B, H, M, N, bm, bn, sms, mx, ctypes.byref(out)) == 0
        assert out.value == want, (B, H, M, N, sms)


def test_invalid_arguments_are_rejected_on_host():
    lib = _lib.lib()
    a = _lib.MlaArgs()
    assert lib.fa_mla_decode(ctypes.byref(a), None) == _lib.FA_ERR_INVALID_ARGUMENT
    d = _lib.DecodeArgs()
    assert lib.fa_paged_attention(ctypes.byref(d), None) == _lib.FA_ERR_INVALID_ARGUMENT
    assert lib.fa_lse_combine(None, None, 0, 0, 0, None, 0, None, None) == \
        _lib.FA_ERR_INVALID_ARGUMENT
    # value widths above 512 are refused before anything is launched
    fake = ctypes.c_void_p(1 << 20)
    assert lib.fa_lse_combine(fake, fake, 2, 4, 516, fake, 0, None, None) == \
        _lib.FA_ERR_UNSUPPORTED
    with pytest.raises(_lib.InvalidArgument):
        _lib.check(_lib.FA_ERR_INVALID_ARGUMENT, "x")


def test_append_rows_rejected_on_host():
    """fa_mla_append_rows checks its arguments before any CUDA call (the
    pointers below are never dereferenced)."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(1 << 20)
    page_stride, tok_stride = 64 * 576, 576
    args = lambda rows, rs, n, dtype: (rows, rs, fake, n, fake, page_stride, tok_stride, 4, 64,  # noqa: E731
                                       dtype, None)
    assert lib.fa_mla_append_rows(*args(fake, 576, -1, 0)) == _lib.FA_ERR_INVALID_ARGUMENT
    assert lib.fa_mla_append_rows(*args(fake, 576, 4, 2)) == _lib.FA_ERR_UNSUPPORTED  # f32
    assert lib.fa_mla_append_rows(*args(fake, 570, 4, 0)) == _lib.FA_ERR_INVALID_ARGUMENT
    assert lib.fa_mla_append_rows(*args(ctypes.c_void_p((1 << 20) + 8), 576, 4, 0)) == \
        _lib.FA_ERR_INVALID_ARGUMENT                                           # misaligned rows
    assert lib.fa_mla_append_rows(None, 576, None, 0, None, page_stride, tok_stride, 4, 64, 0,
                                  None) == _lib.FA_OK                           # nothing to write


def test_append_oracle_skips_negative_and_out_of_pool_slots():
    import numpy as np
    import oracle
    cache = np.zeros((2, 4, 1, 3), np.float32)
    rows = np.arange(12, dtype=np.float32).reshape(4, 3)
    out = oracle.mla_append_rows(cache, rows, [5, -1, 8, 0])
    assert np.array_equal(out[1, 1, 0], rows[0]) and np.array_equal(out[0, 0, 0], rows[3])
    assert np.count_nonzero(out) == 6 - 1 and not np.any(cache)   # row 0 holds a 0; input untouched
