"""Writing new latent rows into the paged pool (fa_mla_append_rows) on the
B200 vs the numpy restatement in oracle/: bit-exact (it is byte movement),
including skipped slots, f16, a padded pool and strided rows; then a decode
over a cache whose last tokens were appended equals the oracle decode of the
same cache."""

import numpy as np
import pytest
import torch

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _torch as fat
from mla_cases import D_QK, D_V, PAGE, assert_close, build_dense, to_dev

pytestmark = pytest.mark.gpu


def _pool(rs, pages, dtype, pad_rows=0):
    """A random pool [pages, 64, 1, 576]; with pad_rows the pages lie
    64 + pad_rows rows apart (a view of a larger allocation)."""
    full = torch.from_numpy(rs.standard_normal((pages, PAGE + pad_rows, 1, D_QK)).astype(np.float32))
    full = full.to(dtype).cuda()
    return full, full[:, :PAGE]


@pytest.mark.parametrize("dtype,pad_rows,row_stride",
                         [(torch.bfloat16, 0, D_QK), (torch.float16, 0, D_QK),
                          (torch.bfloat16, 1, D_QK + 64)])
def test_append_matches_oracle(dtype, pad_rows, row_stride):
    rs = np.random.RandomState(21)
    pages, n = 40, 700
    full, kc = _pool(rs, pages, dtype, pad_rows)
    before = kc.float().cpu().numpy()
    slots = rs.choice(pages * PAGE, size=n, replace=False).astype(np.int64)
    slots[[3, 100]] = -1                            # padding tokens: skipped
    slots[200] = pages * PAGE + 5                   # past the pool: skipped
    src = torch.from_numpy(rs.standard_normal((n, row_stride)).astype(np.float32)).to(dtype).cuda()
    rows = src[:, :D_QK]
    fa.append_kv_rows(rows, kc, to_dev(slots))
    torch.cuda.synchronize()
    want = oracle.mla_append_rows(before, rows.float().cpu().numpy(), slots)
    assert np.array_equal(kc.float().cpu().numpy(), want)
    if pad_rows:                                    # the spare rows are untouched
        assert torch.equal(full[:, PAGE:], _pool(np.random.RandomState(21), pages, dtype,
                                                 pad_rows)[0][:, PAGE:])


def test_decode_after_append():
    """The last 1-3 tokens of every sequence reach the cache through the
    append (their rows zeroed first), then the decode sees the same cache as
    the oracle."""
    lens = [65, 300, 1000, 2047]
    d = build_dense(22, lens, heads=128, poison_tail=False)
    kc = d["kc"]
    rows, slots = [], []
    for b, n in enumerate(lens):
        for t in range(n - 1 - b % 3, n):
            slot = int(d["bt_np"][b][t // PAGE]) * PAGE + t % PAGE
            slots.append(slot)
            rows.append(kc.view(-1, D_QK)[slot].clone())
            kc.view(-1, D_QK)[slot] = 0
    fa.append_kv_rows(torch.stack(rows), kc, to_dev(np.array(slots, np.int64)))
    meta, splits = fa.get_mla_metadata(d["lens"], 128, 1)
    out, lse = fa.flash_mla_with_kvcache(d["q"], kc, d["bt"], d["lens"], D_V, meta, splits,
                                         softmax_scale=D_QK ** -0.5)
    torch.cuda.synchronize()
    assert fat.read_status(torch.device("cuda")) == 0
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, D_QK ** -0.5)
    assert_close("out", out.float().cpu().numpy(), want_o)
    assert_close("lse", lse.cpu().numpy(), want_l)


def test_append_nothing_and_bad_arguments():
    rs = np.random.RandomState(23)
    _, kc = _pool(rs, 2, torch.bfloat16)
    fa.append_kv_rows(torch.empty((0, D_QK), dtype=torch.bfloat16, device="cuda"), kc,
                      torch.empty(0, dtype=torch.int64, device="cuda"))
    with pytest.raises(fa.InvalidArgument):
        fa.append_kv_rows(torch.zeros((2, D_QK), dtype=torch.float16, device="cuda"), kc,
                          torch.zeros(2, dtype=torch.int64, device="cuda"))
    with pytest.raises(fa.InvalidArgument):
        fa.append_kv_rows(torch.zeros((2, D_QK), dtype=torch.bfloat16, device="cuda"), kc,
                          torch.zeros(2, dtype=torch.int32, device="cuda"))
