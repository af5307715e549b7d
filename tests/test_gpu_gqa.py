"""Grouped-query decode on the tcgen05 kernel (csrc/gqa_tc.cu).

The reference's paged test grid runs through the same kernel in
test_gpu_generic.py; these cases pin what is specific to the tensor-core
path: that it is the path taken, the balanced schedule of (sequence, kv head)
entries bit-for-bit against its host specification, the copy layouts for
1..128 query rows per kv head, head sizes 16, 32 (32- / 64-byte swizzled
tiles), 64, 128 and 256 (64-token tiles), value rows past a sequence end
holding NaN,
explicit and automatic split counts, causal multi-token rows on contiguous
caches, and a clean status word.
"""

import ctypes

import numpy as np
import pytest
import torch

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _lib
from flagattention_b200._torch import dtype_code, read_status

pytestmark = pytest.mark.gpu


def _paged_inputs(num_seqs, hq, group, d, block, max_len, dtype, seed, nblocks=300,
                  lens=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hkv = hq // group
    if lens is None:
        lens = torch.randint(1, max_len, (num_seqs,), generator=g, device="cuda",
                             dtype=torch.int32)
        lens[0] = max_len
    else:
        lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = d ** -0.5
    q = ((torch.rand(num_seqs, hq, d, generator=g, device="cuda") * 2 - 1) * scale).to(dtype)
    k = ((torch.rand(nblocks, hkv, block, d, generator=g, device="cuda") * 2 - 1) * scale).to(dtype)
    v = ((torch.rand(nblocks, hkv, block, d, generator=g, device="cuda") * 2 - 1) * scale).to(dtype)
    width = (int(lens.max()) + block - 1) // block
    bt = torch.randint(0, nblocks, (num_seqs, width), generator=g, device="cuda",
                       dtype=torch.int32)
    return q, k, v, lens, bt, scale


def _oracle(q, k, v, bt, lens, scale):
    """oracle.paged_attention on the pages the block table names (gathered
    into a compact cache first, so large pools stay on the device)."""
    pages, remap = torch.unique(bt.long(), return_inverse=True)
    ref = oracle.paged_attention(q.float().cpu().numpy(), k[pages].float().cpu().numpy(),
                                 v[pages].float().cpu().numpy(), remap.cpu().numpy(),
                                 lens.cpu().numpy(), scale)
    return torch.from_numpy(ref)


def _args_for(q, k, lens, bt, out):
    a = _lib.DecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
    a.k = a.v = k.data_ptr()
    a.k_stride_seq, a.k_stride_head, a.k_stride_tok = k.stride(0), k.stride(1), k.stride(2)
    a.block_table, a.bt_stride, a.page_size = bt.data_ptr(), bt.stride(0), k.shape[2]
    a.num_pages = k.shape[0]
    a.seq_lens = lens.data_ptr()
    a.batch, a.num_q_heads, a.num_kv_heads, a.m_q = q.shape[0], q.shape[1], k.shape[1], 1
    a.d_qk = a.d_v = q.shape[2]
    a.dtype = dtype_code(q)
    a.scale = q.shape[2] ** -0.5
    a.o = out.data_ptr()
    a.o_stride_b, a.o_stride_h = out.stride(0), out.stride(1)
    return a


@pytest.mark.parametrize("d, group, block, dtype, want", [
    (128, 8, 16, torch.float16, 1), (64, 1, 256, torch.bfloat16, 1), (128, 128, 128,
                                                                       torch.float16, 1),
    (32, 8, 16, torch.float16, 1), (16, 1, 128, torch.bfloat16, 1), (48, 8, 16, torch.float16, 0),
    (128, 8, 16, torch.float32, 0), (128, 8, 48, torch.float16, 0),
    (128, 256, 16, torch.float16, 0), (256, 8, 16, torch.bfloat16, 1),
    (256, 4, 128, torch.float16, 1), (256, 8, 32, torch.float16, 1), (256, 8, 96, torch.float16, 0)])
def test_tensor_core_path_selection(d, group, block, dtype, want):
    q, k, _, lens, bt, _ = _paged_inputs(2, max(group, 8), group, d, block, 64, dtype, 0,
                                         nblocks=8)
    out = torch.empty_like(q)
    a = _args_for(q, k, lens, bt, out)
    assert _lib.lib().fa_decode_uses_tensor_cores(ctypes.byref(a)) == want


@pytest.mark.parametrize("d", [32, 64, 128, 256])
def test_balanced_schedule_bit_exact(d):
    """The merge records the kernel writes for every entry equal the host
    specification (oracle.gqa_schedule with the kernel's tile as the block),
    and the outputs match the oracle."""
    rs = np.random.RandomState(7 + d)
    lib = _lib.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for trial in range(12):
        B = int(rs.randint(1, 60))
        group = int(rs.choice([1, 4, 8]))
        hkv = int(rs.choice([1, 2, 8]))
        lens = rs.randint(0 if trial % 4 == 0 else 1, 3000, size=B).astype(np.int32)
        lens[0] = max(int(lens[0]), 1)
        q, k, v, lens_t, bt, scale = _paged_inputs(B, hkv * group, group, d, 16, 3000,
                                                   torch.float16, trial, nblocks=400,
                                                   lens=lens.tolist())
        out = torch.empty_like(q)
        a = _args_for(q, k, lens_t, bt, out)
        a.v = v.data_ptr()
        a.num_splits = 0
        # heads 128 / 256 over 16-token pages with an even kv-head count:
        # entries cover two kv heads (half the entries; 64 / 32 tokens of each
        # per tile)
        paired = d in (128, 256) and hkv % 2 == 0
        ents = hkv // 2 if paired else hkv
        po, pl, sc = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        assert lib.fa_decode_workspace_size(ctypes.byref(a), ctypes.byref(po), ctypes.byref(pl),
                                            ctypes.byref(sc)) == 0
        assert sc.value == B * ents * 16
        ws = torch.empty(po.value + pl.value + sc.value, dtype=torch.uint8, device="cuda")
        a.part_o, a.part_lse = ws.data_ptr(), ws.data_ptr() + po.value
        a.sched = ws.data_ptr() + po.value + pl.value
        st = lib.fa_paged_attention(ctypes.byref(a),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == 0
        torch.cuda.synchronize()
        got = ws[po.value + pl.value:].view(torch.int32).view(-1, 4)[:, :3].cpu().numpy()
        # tile tokens: 64 for head 256, 192 for heads up to 64 with at most
        # 64 query rows per kv head, else 128
        block_n = ({128: 64, 256: 32}[d] if paired else
                   64 if d == 256 else (192 if d <= 64 else 128))
        _, merge = oracle.gqa_schedule(lens, ents, sms, block_n=block_n)
        assert np.array_equal(got, np.asarray(merge, np.int32)), trial
        ref = _oracle(q, k, v, bt, lens_t, scale).to(torch.float16).float()
        assert torch.allclose(out.float().cpu(), ref, atol=2e-3, rtol=1e-5), trial


@pytest.mark.parametrize("hq, group", [(64, 1), (64, 8), (16, 16), (64, 32), (64, 64), (96, 96),
                                       (128, 128)])
@pytest.mark.parametrize("d", [16, 32, 64, 128, 256])
def test_rows_per_kv_head(hq, group, d):
    """1..128 query rows per kv head: four, two or one copies of each row."""
    q, k, v, lens, bt, scale = _paged_inputs(5, hq, group, d, 16, 700, torch.bfloat16, group + d)
    out = fa.paged_attention(q, k, v, lens, bt, scale, int(lens.max()))
    torch.cuda.synchronize()
    ref = _oracle(q, k, v, bt, lens, scale).to(torch.bfloat16).float()
    assert torch.allclose(out.float().cpu(), ref, atol=2e-2, rtol=2e-2), \
        (out.float().cpu() - ref).abs().max()
    assert read_status(q.device) == 0


@pytest.mark.parametrize("d, block", [(128, 16), (128, 32), (128, 128), (128, 256), (256, 16),
                                      (256, 32), (256, 128), (32, 16), (16, 128)])
@pytest.mark.parametrize("num_splits", [0, 1, 3, 8])
def test_nan_past_sequence_end_and_splits(d, block, num_splits):
    """Value / key slots past each sequence's end in its last page hold NaN;
    the output stays finite and equal to the oracle's."""
    lens = [1, 17, 129, 300, 1000, 4096, 77]
    width = (max(lens) + block - 1) // block
    q, k, v, lens_t, bt, scale = _paged_inputs(len(lens), 64, 8, d, block, 4096,
                                               torch.float16, block + num_splits,
                                               nblocks=len(lens) * width, lens=lens)
    # distinct pages per sequence so that poisoning one tail cannot touch
    # another sequence's live rows
    bt = torch.arange(len(lens) * width, dtype=torch.int32, device="cuda").view(len(lens), width)
    for s, n in enumerate(lens):
        last, off = (n - 1) // block, n % block
        if off:
            page = bt[s, last].item()
            k[page, :, off:] = float("nan")
            v[page, :, off:] = float("nan")
    out = fa.paged_attention(q, k, v, lens_t, bt, scale, max(lens), num_splits)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    ref = _oracle(q, torch.nan_to_num(k), torch.nan_to_num(v), bt, lens_t, scale)
    ref = ref.to(torch.float16).float()
    assert torch.allclose(out.float().cpu(), ref, atol=2e-3, rtol=1e-5), \
        (out.float().cpu() - ref).abs().max()
    assert read_status(q.device) == 0


def test_bench_shape_matches_oracle():
    """The bench's grouped-query case (32 sequences x 4096 tokens, 64 query /
    8 kv heads, head 128, page 16) on the balanced schedule."""
    q, k, v, lens, bt, scale = _paged_inputs(32, 64, 8, 128, 16, 4096, torch.bfloat16, 11,
                                             nblocks=8192, lens=[4096] * 32)
    out = fa.paged_attention(q, k, v, lens, bt, scale, 4096)
    torch.cuda.synchronize()
    idx = [0, 13, 31]
    ref = _oracle(q[idx], k, v, bt[idx], lens[idx], scale).to(torch.bfloat16).float()
    assert torch.allclose(out[idx].float().cpu(), ref, atol=2e-2, rtol=2e-2)
    assert read_status(q.device) == 0


@pytest.mark.parametrize("M", [1, 3, 4])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [16, 32, 128, 256])
def test_contiguous_causal_rows(M, causal, D):
    """Contiguous caches (split-KV decoding) with several query tokens per
    sequence and bottom-right causal masking, GQA group 4."""
    g = torch.Generator(device="cuda").manual_seed(M * 2 + causal + D)
    B, Hq, Hk, N = 3, 16, 4, 3001
    q = torch.randn(B, Hq, M, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hk, N, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hk, N, D, generator=g, device="cuda").to(torch.bfloat16)
    o, lse, _ = fa.flash_attention(q, k, v, causal, return_log_normalizer=True)
    torch.cuda.synchronize()
    ref_o, ref_l = oracle.flash_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                          v.float().cpu().numpy(), causal,
                                          return_log_normalizer=True)
    assert torch.allclose(o.float().cpu(), torch.from_numpy(ref_o), atol=2e-2, rtol=2e-2)
    assert torch.allclose(lse.cpu(), torch.from_numpy(ref_l), atol=1e-3, rtol=1e-4)
    assert read_status(q.device) == 0
