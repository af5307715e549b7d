"""Generic paged / split-KV decode on the GPU (the reference's own API shapes).

Mirrors tests/flag_attn/test_paged_attention.py (atol 2e-3 in f16 against the
reference oracle) and the split-KV test of test_flash_attention.py (error at
most twice that of torch's low-precision attention, plus 1e-5).
"""

import ctypes
import os

import numpy as np
import pytest
import torch

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _lib

pytestmark = pytest.mark.gpu


def test_paged_gqa_matches_reference_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "paged_gqa.npz"))
    for c in range(int(z["num_cases"])):
        g = lambda n: torch.from_numpy(z[f"c{c}_{n}"]).cuda()  # noqa: E731
        lens = g("lens")
        out = fa.paged_attention(g("q"), g("k"), g("v"), lens, g("bt"), float(z[f"c{c}_scale"]),
                                 int(lens.max()))
        torch.cuda.synchronize()
        ref = g("out")
        assert torch.allclose(out, ref, atol=2e-3, rtol=1e-5), (c, (out - ref).abs().max())


def _paged_case(num_seqs, num_query_heads, group, head_size, block_size, max_seq_len,
                num_splits=0, dtype=torch.float16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nkv = num_query_heads // group
    nblocks = 300
    lens = torch.randint(1, max_seq_len, (num_seqs,), generator=g, device="cuda",
                         dtype=torch.int32) if max_seq_len > 1 else \
        torch.ones(num_seqs, dtype=torch.int32, device="cuda")
    lens[0] = max_seq_len
    scale = head_size ** -0.5
    q = (torch.rand(num_seqs, num_query_heads, head_size, generator=g, device="cuda") * 2 - 1) * scale
    k = (torch.rand(nblocks, nkv, block_size, head_size, generator=g, device="cuda") * 2 - 1) * scale
    v = (torch.rand(nblocks, nkv, block_size, head_size, generator=g, device="cuda") * 2 - 1) * scale
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    width = (max_seq_len + block_size - 1) // block_size
    bt = torch.randint(0, nblocks, (num_seqs, width), generator=g, device="cuda", dtype=torch.int32)
    out = fa.paged_attention(q, k, v, lens, bt, scale, int(lens.max()), num_splits)
    torch.cuda.synchronize()
    ref = oracle.paged_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                 v.float().cpu().numpy(), bt.cpu().numpy(), lens.cpu().numpy(),
                                 scale)
    ref = torch.from_numpy(ref).to(dtype).float()
    diff = (out.float().cpu() - ref).abs().max().item()
    assert torch.allclose(out.float().cpu(), ref, atol=2e-3, rtol=1e-5), diff


@pytest.mark.parametrize("num_seqs", [1, 32])
@pytest.mark.parametrize("group", [1, 8])
@pytest.mark.parametrize("head_size", [64, 128])
@pytest.mark.parametrize("block_size", [16, 128, 256])
@pytest.mark.parametrize("max_seq_len", [512, 4096])
def test_paged_attention_default(num_seqs, group, head_size, block_size, max_seq_len):
    _paged_case(num_seqs, 64, group, head_size, block_size, max_seq_len)


@pytest.mark.parametrize("num_splits", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("group", [1, 8])
def test_paged_attention_by_num_splits(num_splits, group):
    _paged_case(16, 64, group, 64, 16, 2048, num_splits=num_splits)


@pytest.mark.parametrize("case", [(1, 12, 1, 64, 16, 2, 0), (16, 64, 8, 32, 16, 2048, 2),
                                  (16, 64, 1, 64, 16, 2048, 6)])
def test_paged_attention_by_case(case):
    _paged_case(*case)


def test_split_kv_matches_reference_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "split_kv.npz"))
    for c in range(int(z["num_cases"])):
        g = lambda n: torch.from_numpy(z[f"c{c}_{n}"]).cuda()  # noqa: E731
        o, L, _ = fa.flash_attention(g("q"), g("k"), g("v"), bool(z[f"c{c}_causal"]),
                                     return_log_normalizer=True)
        torch.cuda.synchronize()
        ref32 = g("out_f32")
        torch_err = (g("out").float() - ref32).abs().max().item()
        err = (o.float() - ref32).abs().max().item()
        assert err <= 2 * torch_err + 1e-5 or err < 2e-3, (c, err, torch_err)
        assert torch.allclose(L, g("lse"), atol=1e-3, rtol=1e-4), c


@pytest.mark.parametrize("B, Hq, Hk, M, N, D", [
    (2, 4, 4, 1, 612, 128), (2, 4, 4, 1, 1034, 64), (2, 4, 4, 2, 4000, 128),
    (1, 2, 2, 4, 8202, 16), (2, 4, 1, 1, 4096, 64), (1, 2, 1, 4, 8202, 16)])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_split_kv_vs_oracle(B, Hq, Hk, M, N, D, causal, dtype):
    g = torch.Generator(device="cuda").manual_seed(10086)
    q = torch.empty((B, Hq, M, D), dtype=dtype, device="cuda").normal_(std=10.0, generator=g)
    k = torch.empty((B, Hk, N, D), dtype=dtype, device="cuda").normal_(std=10.0, generator=g)
    v = torch.empty((B, Hk, N, D), dtype=dtype, device="cuda").normal_(std=10.0, generator=g)
    o = fa.flash_attention_split_kv(q, k, v, causal)
    torch.cuda.synchronize()
    ref = torch.from_numpy(oracle.flash_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                  v.float().cpu().numpy(), causal))
    low = _torch_lowprec(q, k, v, causal).float().cpu()
    torch_err = (low - ref).abs().max().item()
    err = (o.float().cpu() - ref).abs().max().item()
    assert err <= 2 * torch_err + 1e-5, (err, torch_err)


def _torch_lowprec(q, k, v, causal):
    """testing/flash.py:19-84 with upcast=False: the 'torch' arm of the
    reference's three-implementations criterion (README.md:111-117)."""
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    M, N = q.shape[2], k.shape[2]
    s = torch.matmul(q, k.transpose(2, 3)) * (q.shape[-1] ** -0.5)
    if causal:
        ms = torch.arange(M, device=q.device)[:, None]
        ns = torch.arange(N, device=q.device)
        s = torch.where(ms + (N - M) >= ns, s, float("-inf"))
    p = torch.softmax(s.float(), dim=-1)
    return torch.matmul(p.to(v.dtype), v).to(q.dtype)


def test_lse_combine_matches_reference_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "combine.npz"))
    po = torch.from_numpy(z["part_o"]).cuda().contiguous()          # [S, B, H, M, D]
    pl = torch.from_numpy(z["part_lse"]).cuda().contiguous()        # [S, B, H, M]
    S = po.shape[0]
    rows = pl[0].numel()
    d_v = po.shape[-1]
    out = torch.empty((rows, d_v), dtype=torch.float32, device="cuda")
    lse = torch.empty((rows,), dtype=torch.float32, device="cuda")
    st = _lib.lib().fa_lse_combine(ctypes.c_void_p(po.data_ptr()), ctypes.c_void_p(pl.data_ptr()),
                                   S, rows, d_v, ctypes.c_void_p(out.data_ptr()),
                                   _lib.FA_DTYPE_F32, ctypes.c_void_p(lse.data_ptr()),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), z["out"].reshape(rows, d_v), rtol=1e-5,
                               atol=1e-5)
    np.testing.assert_allclose(lse.cpu().numpy(), z["lse"].reshape(rows), rtol=1e-5, atol=1e-5)
