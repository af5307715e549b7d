"""MLA decode on the B200 vs the CPU oracle and the reference's golden outputs.

Every call goes through the C ABI (flagattention_b200 -> libflagattn_b200.so).
"""

import os

import numpy as np
import pytest
import torch

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _torch as fat
from mla_cases import D_QK, D_V, PAGE, assert_close, build_dense, build_sparse, to_dev
from inputs import digest, mla_inputs

pytestmark = pytest.mark.gpu

SCALE = D_QK ** -0.5


def _status_ok():
    assert fat.read_status(torch.device("cuda")) == 0, "a bounded wait inside a kernel gave up"


def _decode(d, causal=False, parts=None, indices=None, topk=None):
    if indices is None:
        meta, splits = fa.get_mla_metadata(d["lens"], d["q"].shape[1] * d["q"].shape[2], 1,
                                           num_sm_parts_override=parts)
    else:
        meta, splits = fa.get_mla_metadata(d["lens"], d["q"].shape[1] * d["q"].shape[2], 1,
                                           num_heads_q=d["q"].shape[2], topk=topk,
                                           num_sm_parts_override=parts)
    out, lse = fa.flash_mla_with_kvcache(d["q"], d["kc"], d["bt"], d["lens"], D_V, meta, splits,
                                         softmax_scale=SCALE, causal=causal, indices=indices)
    torch.cuda.synchronize()
    _status_ok()
    return out.float().cpu().numpy(), lse.cpu().numpy(), meta, splits


@pytest.mark.parametrize("topk", [0, 2048])
def test_metadata_bit_exact(topk):
    rs = np.random.RandomState(5)
    for trial in range(40):
        B = int(rs.randint(1, 200))
        lens = rs.randint(0 if trial % 3 == 0 else 1, 20000, size=B).astype(np.int32)
        parts = int(rs.randint(1, 150))
        meta, splits = fa.get_mla_metadata(to_dev(lens), 128, 1, num_heads_q=128 if topk else None,
                                           topk=topk or None, num_sm_parts_override=parts)
        want_meta, want_splits = oracle.mla_schedule([topk] * B if topk else lens, parts)
        assert np.array_equal(meta.cpu().numpy(), np.asarray(want_meta, np.int32))
        assert np.array_equal(splits.cpu().numpy(), np.asarray(want_splits, np.int32))


def test_config1_matches_reference_golden(golden_dir):
    """BASELINE config 1 (fp32 N(0,1) inputs) computed in bf16 on the GPU."""
    z = np.load(os.path.join(golden_dir, "mla_config1.npz"))
    q, kc, bt = mla_inputs(int(z["seed"]), 4, 1, 16, z["lens"], bf16=False)
    assert digest(q, kc) == str(z["digest"])
    d = dict(q=to_dev(q, torch.bfloat16), kc=to_dev(kc, torch.bfloat16), bt=to_dev(bt),
             lens=to_dev(z["lens"]))
    out, lse, _, _ = _decode(d)
    assert_close("out", out, z["out"])
    assert_close("lse", lse, z["lse"])


@pytest.mark.parametrize("heads", [16, 128])
@pytest.mark.parametrize("parts", [None, 1, 3, 37])
def test_dense_ragged_lengths(heads, parts):
    lens = [1, 63, 64, 65, 127, 200, 1000, 4097]
    d = build_dense(11, lens, heads=heads)
    out, lse, _, _ = _decode(d, parts=parts)
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, SCALE)
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


def test_dense_fp16():
    d = build_dense(12, [300, 77, 1500], heads=128, dtype=torch.float16)
    out, lse, _, _ = _decode(d)
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, SCALE)
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


def test_output_rows_not_32_byte_aligned():
    """A caller's output view with a padded row stride whose rows start 16
    bytes past a 32-byte boundary gets the same result as a fresh output, bit
    for bit (split and unsplit sequences), and nothing outside the view."""
    d = build_dense(14, [3000, 64, 1201, 5000], heads=128)
    meta, splits = fa.get_mla_metadata(d["lens"], 128, 1, num_sm_parts_override=9)
    ref_o, ref_l = fa.flash_mla_with_kvcache(d["q"], d["kc"], d["bt"], d["lens"], D_V, meta,
                                             splits, softmax_scale=SCALE)
    big = torch.full((4, 1, 128, D_V + 8), float("nan"), dtype=ref_o.dtype, device="cuda")
    out = big[..., 8:]  # row stride 520 elements: 16- but not 32-byte aligned rows
    assert out.data_ptr() % 32 == 16
    o2, l2 = fa.flash_mla_with_kvcache(d["q"], d["kc"], d["bt"], d["lens"], D_V, meta, splits,
                                       softmax_scale=SCALE, out=out)
    torch.cuda.synchronize()
    _status_ok()
    assert o2.data_ptr() == out.data_ptr()
    assert torch.equal(out, ref_o) and torch.equal(l2, ref_l)
    assert torch.isnan(big[..., :8]).all()  # nothing written outside the view


def test_zero_length_sequence():
    d = build_dense(13, [0, 100, 0], heads=128)
    out, lse, _, _ = _decode(d)
    assert np.all(out[0] == 0) and np.all(out[2] == 0)
    assert np.all(np.isneginf(lse[0])) and np.all(np.isneginf(lse[2]))
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, SCALE)
    assert_close("out", out, want_o)


@pytest.mark.parametrize("causal", [True, False])
def test_mtp_matches_reference_golden(golden_dir, causal):
    z = np.load(os.path.join(golden_dir, "mla_mtp_causal.npz"))
    q, kc, bt = mla_inputs(int(z["seed"]), 3, 2, 16, z["lens"], bf16=True)
    d = dict(q=to_dev(q, torch.bfloat16), kc=to_dev(kc, torch.bfloat16), bt=to_dev(bt),
             lens=to_dev(z["lens"]))
    out, lse, _, _ = _decode(d, causal=causal)
    sfx = "" if causal else "_noncausal"
    assert_close("out", out, z["out" + sfx])
    assert_close("lse", lse, z["lse" + sfx])


@pytest.mark.parametrize("parts", [None, 2])
def test_mtp_128_heads_causal(parts):
    d = build_dense(14, [1, 2, 64, 65, 513, 3000], s_q=2, heads=128)
    out, lse, _, _ = _decode(d, causal=True, parts=parts)
    want_o, want_l = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"],
                                             D_V, SCALE, causal=True)
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


def test_sparse_matches_reference_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "mla_sparse.npz"))
    q, kc, bt = mla_inputs(int(z["seed"]), 2, 2, 16, z["lens"], bf16=True)
    d = dict(q=to_dev(q, torch.bfloat16), kc=to_dev(kc, torch.bfloat16), bt=to_dev(bt),
             lens=to_dev(z["lens"]))
    idx = to_dev(z["indices"])
    out, lse, _, _ = _decode(d, indices=idx, topk=int(z["topk"]))
    assert_close("out", out, z["out"])
    assert_close("lse", lse, z["lse"])


@pytest.mark.parametrize("parts", [None, 5])
def test_sparse_padding_and_out_of_range(parts):
    d = build_sparse(15, [100, 3000, 1], topk=256, s_q=1, heads=128)
    d["idx_np"][1, 0, 7] = -1                        # a hole in the middle
    d["idx_np"][1, 0, 9] = 10 ** 9                   # out of range: masked too
    d["idx"] = to_dev(d["idx_np"])
    out, lse, _, _ = _decode(d, indices=d["idx"], topk=256, parts=parts)
    want_o, want_l = oracle.mla_decode_sparse(d["q_np"], d["kc_np"], d["idx_np"], D_V, SCALE)
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


def test_sparse_padded_pool_row_copy_route():
    """Top-k over a pool whose pages are not back to back (64-row pages
    allocated 65 rows apart, the spare rows NaN): no single row map covers it,
    so rows come in one-row boxes of the page map, against the same oracle."""
    d = build_sparse(17, [300, 5000], topk=512, s_q=1, heads=128)
    kc = d["kc"]
    padded = torch.full((kc.shape[0], PAGE + 1, 1, D_QK), float("nan"), dtype=kc.dtype,
                        device="cuda")
    padded[:, :PAGE] = kc
    d["kc"] = padded[:, :PAGE]
    assert d["kc"].stride(0) != PAGE * d["kc"].stride(1)
    d["idx_np"][1, 0, 3] = -1                        # a masked entry on this route too
    d["idx"] = to_dev(d["idx_np"])
    out, lse, _, _ = _decode(d, indices=d["idx"], topk=512)
    want_o, want_l = oracle.mla_decode_sparse(d["q_np"], d["kc_np"], d["idx_np"], D_V, SCALE)
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


@pytest.mark.parametrize("padded_pool", [False, True])
def test_sparse_unreferenced_rows_nan(padded_pool):
    """Every pool row no index list refers to is NaN, pool row 0 included (a
    NaN page is put in front of the pool and the indices moved past it);
    lists longer than their sequence end in -1 padding, one query's list is
    all -1 (out 0, lse -inf) and one holds a single valid row.  A masked
    column must contribute exactly nothing, whatever its row holds."""
    lens = [40, 3000, 500, 1]
    d = build_sparse(18, lens, topk=256, s_q=2, heads=128)
    idx = d["idx_np"].copy()
    idx[idx >= 0] += PAGE
    idx[2, 1, :] = -1                                 # no valid entry at all
    idx[3, 0, 1:] = -1                                # one valid entry
    kc_np = np.concatenate([np.full((1, PAGE, 1, D_QK), np.nan, np.float32), d["kc_np"]])
    n_pages = kc_np.shape[0]
    stride = PAGE + 1 if padded_pool else PAGE
    pool = torch.full((n_pages, stride, 1, D_QK), float("nan"), dtype=torch.bfloat16,
                      device="cuda")
    pool[:, :PAGE] = to_dev(kc_np, torch.bfloat16)
    used = torch.zeros(n_pages * PAGE, dtype=torch.bool, device="cuda")
    used[to_dev(np.unique(idx[idx >= 0]).astype(np.int64))] = True
    rows = pool[:, :PAGE]
    rows[~used.view(n_pages, PAGE)] = float("nan")
    assert not bool(used[0]) and torch.isnan(rows[0, 0]).all()
    d["kc"] = rows
    d["idx"] = to_dev(idx)
    out, lse, _, _ = _decode(d, indices=d["idx"], topk=256)
    want_o, want_l = oracle.mla_decode_sparse(d["q_np"], kc_np, idx, D_V, SCALE)
    assert np.isneginf(want_l[2, :, 1]).all() and (want_o[2, 1] == 0).all()
    assert_close("out", out, want_o)
    assert_close("lse", lse, want_l)


def test_contiguous_split_kv_mla_route():
    """flash_attention_split_kv with the MLA shape takes the tensor-core path."""
    rs = np.random.RandomState(16)
    B, H, N = 2, 128, 700
    k = torch.from_numpy(rs.standard_normal((B, 1, N, D_QK)).astype(np.float32)).cuda().bfloat16()
    q = torch.from_numpy(rs.standard_normal((B, H, 1, D_QK)).astype(np.float32)).cuda().bfloat16()
    o, L, _ = fa.flash_attention(q, k, k[..., :D_V], False, None, return_log_normalizer=True)
    torch.cuda.synchronize()
    want_o, want_l = oracle.flash_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                            k[..., :D_V].float().cpu().numpy(), False, None, True)
    assert_close("out", o.float().cpu().numpy(), want_o)
    assert_close("lse", L.cpu().numpy(), want_l)


def test_paged_attention_mla_route():
    """flag_attn.paged_attention signature with the MLA cache (value = key[..., :512])."""
    d = build_dense(17, [90, 1000, 64], heads=128)
    kc = d["kc"].permute(0, 2, 1, 3)                  # [P, 1, page, 576] view
    out = fa.paged_attention(d["q"][:, 0], kc, kc[..., :D_V], d["lens"], d["bt"], SCALE,
                             int(d["lens_np"].max()))
    torch.cuda.synchronize()
    want_o, _ = oracle.mla_decode_dense(d["q_np"], d["kc_np"], d["bt_np"], d["lens_np"], D_V,
                                        SCALE)
    assert_close("out", out.float().cpu().numpy(), want_o[:, 0])


def test_full_size_config2_sampled():
    """BASELINE config 2 at full size: sampled sequences vs the oracle plus
    the split-invariance property (any scheduler partition gives the same)."""
    rs = np.random.RandomState(2)
    lens = rs.randint(1024, 8193, size=64).astype(np.int32)
    d = build_dense(20, lens, heads=128, poison_tail=True)
    out, lse, meta, splits = _decode(d)
    assert (np.diff(splits.cpu().numpy()) >= 1).all()
    pick = [0, 17, 40, 63]
    want_o, want_l = oracle.mla_decode_dense(d["q_np"][pick], d["kc_np"], d["bt_np"][pick],
                                             d["lens_np"][pick], D_V, SCALE)
    assert_close("out", out[pick], want_o)
    assert_close("lse", lse[pick], want_l)
    out2, lse2, _, _ = _decode(d, parts=7)
    assert_close("split invariance out", out2, out, atol=1e-2, rtol=1e-2)
    assert_close("split invariance lse", lse2, lse, atol=1e-3, rtol=1e-3)
