"""Pin the CPU oracle to outputs of the reference itself (CPU only).

The fixtures under tests/golden were produced by FlagAttention's own
``flag_attn.testing`` functions and heuristics (tests/golden/make_golden.py).
"""

import json
import os

import numpy as np
import pytest

import oracle
from inputs import digest, mla_inputs

D_QK, D_V = 576, 512


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _regen(z, batch, s_q, heads, bf16):
    q, kc, bt = mla_inputs(int(z["seed"]), batch, s_q, heads, z["lens"], bf16=bf16)
    assert digest(q, kc) == str(z["digest"]), "RandomState stream changed: regenerate fixtures"
    assert np.array_equal(bt, z["block_table"])
    return q, kc, bt


def test_config1_dense_matches_reference(golden_dir):
    z = _load(golden_dir, "mla_config1.npz")
    q, kc, bt = _regen(z, 4, 1, 16, bf16=False)
    out, lse = oracle.mla_decode_dense(q, kc, bt, z["lens"], D_V, D_QK ** -0.5)
    np.testing.assert_allclose(out, z["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(out, z["out_paged"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(lse, z["lse"], rtol=1e-5, atol=1e-5)
    assert out.shape == (4, 1, 16, 512) and lse.shape == (4, 16, 1)


def test_config1_paged_oracle_matches_reference(golden_dir):
    z = _load(golden_dir, "mla_config1.npz")
    q, kc, bt = _regen(z, 4, 1, 16, bf16=False)
    kcache = np.transpose(kc, (0, 2, 1, 3))          # [P, Hkv=1, page, D]
    out = oracle.paged_attention(q[:, 0], kcache, kcache[..., :D_V], bt, z["lens"], D_QK ** -0.5)
    np.testing.assert_allclose(out, z["out_paged"][:, 0], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("causal", [True, False])
def test_mtp_matches_reference(golden_dir, causal):
    z = _load(golden_dir, "mla_mtp_causal.npz")
    q, kc, bt = _regen(z, 3, 2, 16, bf16=True)
    out, lse = oracle.mla_decode_dense(q, kc, bt, z["lens"], D_V, D_QK ** -0.5, causal=causal)
    sfx = "" if causal else "_noncausal"
    np.testing.assert_allclose(out, z["out" + sfx], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(lse, z["lse" + sfx], rtol=1e-5, atol=1e-5)


def test_sparse_matches_reference(golden_dir):
    z = _load(golden_dir, "mla_sparse.npz")
    q, kc, bt = _regen(z, 2, 2, 16, bf16=True)
    idx = z["indices"]
    assert (idx[0] == -1).any(), "fixture must exercise -1 padding (len < topk)"
    out, lse = oracle.mla_decode_sparse(q, kc, idx, D_V, D_QK ** -0.5)
    np.testing.assert_allclose(out, z["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(lse, z["lse"], rtol=1e-5, atol=1e-5)


def test_paged_gqa_matches_reference(golden_dir):
    z = _load(golden_dir, "paged_gqa.npz")
    for c in range(int(z["num_cases"])):
        g = lambda n: z[f"c{c}_{n}"]  # noqa: E731
        out = oracle.paged_attention(g("q").astype(np.float32), g("k").astype(np.float32),
                                     g("v").astype(np.float32), g("bt"), g("lens"), float(g("scale")))
        np.testing.assert_allclose(out, g("out_f32"), rtol=1e-4, atol=1e-5)
        # the reference casts to f16; the cast oracle must agree bit-for-bit up to rounding ties
        np.testing.assert_allclose(out.astype(np.float16).astype(np.float32),
                                   g("out").astype(np.float32), rtol=0, atol=1e-3)


def test_split_kv_matches_reference(golden_dir):
    z = _load(golden_dir, "split_kv.npz")
    for c in range(int(z["num_cases"])):
        g = lambda n: z[f"c{c}_{n}"]  # noqa: E731
        o, lse = oracle.flash_attention(g("q").astype(np.float32), g("k").astype(np.float32),
                                        g("v").astype(np.float32), bool(g("causal")),
                                        return_log_normalizer=True)
        np.testing.assert_allclose(o, g("out_f32"), rtol=1e-4, atol=2e-5)
        np.testing.assert_allclose(lse, g("lse"), rtol=1e-5, atol=1e-5)


def test_combine_reconstructs_reference(golden_dir):
    z = _load(golden_dir, "combine.npz")
    o, lse = oracle.lse_combine(z["part_o"], z["part_lse"])
    np.testing.assert_allclose(o, z["out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse, z["lse"], rtol=1e-6, atol=1e-5)


def test_paged_v2_reduce_equals_lse_combine():
    rs = np.random.RandomState(7)
    S, G, D = 5, 8, 16
    o = rs.randn(S, G, D).astype(np.float32)
    m = rs.randn(S, G).astype(np.float32)
    l = rs.rand(S, G).astype(np.float32) + 0.5
    lse = m + np.log(l)
    a = oracle.paged_v2_reduce(o, m, l)
    b, _ = oracle.lse_combine(o, lse)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)


def test_heuristics_match_reference(golden_dir):
    with open(os.path.join(golden_dir, "heuristics.json")) as f:
        d = json.load(f)
    for seqs, hkv, ctx, blk, sms, req, ns, ps in d["paged_rule"]:
        got_ns, got_ps = oracle.paged_num_splits(seqs, hkv, ctx, blk, sms, req)
        assert got_ns == ns, (seqs, hkv, ctx, blk, sms, req)
        if ns > 1:
            assert got_ps == ps, (seqs, hkv, ctx, blk, sms, req)
    for B, H, M, N, bm, bn, sms, mx, s in d["split_kv"]:
        assert oracle.num_splits_heuristic(B, H, M, N, bm, bn, sms, mx) == s


def test_mla_schedule_invariants():
    rs = np.random.RandomState(11)
    for trial in range(200):
        B = int(rs.randint(1, 40))
        parts = int(rs.randint(1, 80))
        lens = rs.randint(0, 5000, size=B)
        meta, prefix = oracle.mla_schedule(lens, parts)
        nb = [(int(x) + 63) // 64 for x in lens]
        covered = [[] for _ in range(B)]
        for p in range(parts):
            b0, k0, b1, k1, idx0, n, _, _ = meta[p]
            for i in range(n):
                b = b0 + i
                lo = k0 if i == 0 else 0
                hi = k1 if b == b1 else nb[b]
                covered[b].append((lo, hi, (idx0 if i == 0 else 0)))
        for b in range(B):
            pieces = covered[b]
            assert len(pieces) == prefix[b + 1] - prefix[b] >= 1
            pos = 0
            for j, (lo, hi, idx) in enumerate(pieces):
                assert lo == pos and hi >= lo and idx == j
                pos = hi
            assert pos == nb[b]
