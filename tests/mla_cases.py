"""Shared builders for the GPU MLA tests (test infrastructure)."""

import numpy as np
import torch

from inputs import mla_inputs, round_bf16, sparse_indices

D_QK, D_V, PAGE = 576, 512, 64
# Tolerance of the spec: bf16 outputs and LSE within atol/rtol 2e-2 of the
# fp32-upcast reference.
ATOL = RTOL = 2e-2


def to_dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def build_dense(seed, lens, s_q=1, heads=128, dtype=torch.bfloat16, poison_tail=True,
                extra_pages=0):
    """Inputs on the GPU + the same (rounded) values as float32 numpy.

    poison_tail fills every cache slot past a sequence's length with NaN, so a
    kernel that multiplies masked probabilities by those rows fails loudly.
    """
    lens = np.asarray(lens, np.int32)
    q, kc, bt = mla_inputs(seed, len(lens), s_q, heads, lens, bf16=(dtype == torch.bfloat16))
    if dtype == torch.float16:
        q, kc = q.astype(np.float16).astype(np.float32), kc.astype(np.float16).astype(np.float32)
    if extra_pages:
        kc = np.concatenate([kc, np.zeros((extra_pages,) + kc.shape[1:], np.float32)])
    kc_dev = to_dev(kc, dtype)
    if poison_tail:
        flat = kc_dev.view(-1, D_QK)
        valid = torch.zeros(flat.shape[0], dtype=torch.bool, device="cuda")
        for b, n in enumerate(lens):
            tok = np.arange(int(n))
            rows = bt[b][tok // PAGE] * PAGE + tok % PAGE
            valid[to_dev(rows.astype(np.int64))] = True
        flat[~valid] = float("nan")
    return dict(q=to_dev(q, dtype), kc=kc_dev, bt=to_dev(bt), lens=to_dev(lens),
                q_np=q, kc_np=kc, bt_np=bt, lens_np=lens)


def build_sparse(seed, lens, topk, s_q=1, heads=128, dtype=torch.bfloat16):
    d = build_dense(seed, lens, s_q=s_q, heads=heads, dtype=dtype, poison_tail=False)
    idx = sparse_indices(seed + 5, d["lens_np"], s_q, topk, d["bt_np"])
    d["idx_np"] = idx
    d["idx"] = to_dev(idx)
    return d


def assert_close(name, got, want, atol=ATOL, rtol=RTOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (name, got.shape, want.shape)
    finite_want = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), finite_want), f"{name}: non-finite mismatch"
    g, w = got[finite_want], want[finite_want]
    err = np.abs(g - w) - (atol + rtol * np.abs(w))
    worst = float(np.max(np.abs(g - w))) if g.size else 0.0
    assert (err <= 0).all(), f"{name}: max |diff| {worst:.3e} exceeds atol={atol} rtol={rtol}"
    return worst
