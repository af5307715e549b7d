"""Reference-compatible ``paged_attention`` (FlagAttention ``paged.py:20-177``).

Same signature, argument meaning and result as ``flag_attn.paged_attention``:
query [num_seqs, num_q_heads, head_size], caches [num_blocks, num_kv_heads,
block_size, head_size] with identical strides, int32 context_lens and
block_tables, returns ``out`` shaped like the query (with the value width).

Two paths, chosen by shape:

* the MLA latent shape (one kv head, 576-dim keys, values = the first 512
  dims of the same cache rows, block size a multiple of 64, bf16/f16) runs on
  the tcgen05 tensor-core kernel with the balanced tile scheduler;
* bf16/f16 with head size 16, 32, 64, 128 or 256, up to 128 query heads per
  kv head and a block size that the kernel's TMA boxes tile runs the tcgen05
  grouped-query kernel (``csrc/gqa_tc.cu``); with the default
  ``num_splits=0`` the device scheduler balances the key blocks over the
  SMs, an explicit ``num_splits`` keeps the reference's partitions;
* every other shape (head size 512, f32, more heads per kv head) runs the
  CUDA-core kernel with
  the reference's split rule (``paged.py:54-67``, bit-exact through
  ``fa_paged_num_splits``).
"""

import ctypes

import torch

from flagattention_b200 import _decode, _lib
from flagattention_b200._torch import dtype_code, require_cuda, sm_count, status_word, stream_of


def paged_num_splits(num_seqs, num_kv_heads, max_context_len, kv_block_size, num_sms,
                     num_splits=0):
    """(num_splits, partition_size) per the reference rule (paged.py:54-67)."""
    ns, ps = ctypes.c_int32(0), ctypes.c_int32(0)
    _lib.check(_lib.lib().fa_paged_num_splits(num_seqs, num_kv_heads, max_context_len,
                                              kv_block_size, num_sms, num_splits,
                                              ctypes.byref(ns), ctypes.byref(ps)),
               "fa_paged_num_splits")
    return ns.value, ps.value


def _is_mla(query, key_cache, value_cache):
    return (key_cache.shape[1] == 1 and key_cache.shape[3] == 576 and value_cache.shape[3] == 512
            and value_cache.data_ptr() == key_cache.data_ptr()
            and value_cache.stride() == key_cache.stride()
            and key_cache.shape[2] % 64 == 0 and query.dtype in (torch.bfloat16, torch.float16))


def _mla_paged(query, key_cache, context_lens, block_tables, attn_scale):
    from flagattention_b200.mla import get_mla_metadata, mla_decode
    S, H, _ = query.shape
    meta, splits = get_mla_metadata(context_lens, H, 1)
    q = query.unsqueeze(1)                                # [S, 1, H, 576]
    out = torch.empty((S, H, 512), dtype=query.dtype, device=query.device)
    lse = torch.empty((S, H, 1), dtype=torch.float32, device=query.device)
    mla_decode(q, key_cache, key_cache.stride(0), key_cache.stride(2), key_cache.shape[0],
               key_cache.shape[2], block_tables, context_lens, 0, meta, splits,
               out.unsqueeze(1), lse, attn_scale)
    return out


def paged_attention(query, key_cache, value_cache, context_lens, block_tables, attn_scale,
                    max_context_len, num_splits=0):
    """Drop-in for ``flag_attn.paged_attention`` (paged.py:20)."""
    require_cuda(query, key_cache, value_cache, context_lens, block_tables)
    num_seqs, num_q_heads, head_size = query.shape
    num_kv_heads, block_size = key_cache.shape[1], key_cache.shape[2]
    if key_cache.shape[3] != head_size:
        raise _lib.InvalidArgument("query and key_cache head sizes differ")
    if value_cache.shape[:3] != key_cache.shape[:3] or value_cache.stride() != key_cache.stride():
        raise _lib.InvalidArgument("value_cache must have the same shape/strides as key_cache")
    if num_q_heads % num_kv_heads != 0:
        raise _lib.InvalidArgument("num_q_heads must be a multiple of num_kv_heads")
    if context_lens.dtype != torch.int32 or block_tables.dtype != torch.int32:
        raise _lib.InvalidArgument("context_lens and block_tables must be int32")
    if _is_mla(query, key_cache, value_cache):
        return _mla_paged(query, key_cache, context_lens, block_tables, attn_scale)
    if query.stride(-1) != 1 or key_cache.stride(-1) != 1:
        raise _lib.InvalidArgument("last dims must be contiguous")
    d_v = value_cache.shape[3]

    def reference_splits():
        ns, ps = paged_num_splits(num_seqs, num_kv_heads, int(max_context_len), block_size,
                                  sm_count(query.device), int(num_splits))
        if ns > 1 and not (ps >= block_size and ps % block_size == 0):
            # the reference asserts this (paged.py:124)
            raise _lib.InvalidArgument(f"partition_size={ps}, kv_block_size={block_size}")
        return ns, ps

    out = torch.empty((num_seqs, num_q_heads, d_v), dtype=query.dtype, device=query.device)
    a = _lib.DecodeArgs()
    a.q = query.data_ptr()
    a.q_stride_b, a.q_stride_h, a.q_stride_m = query.stride(0), query.stride(1), 0
    a.k, a.v = key_cache.data_ptr(), value_cache.data_ptr()
    a.k_stride_seq, a.k_stride_head, a.k_stride_tok = (key_cache.stride(0), key_cache.stride(1),
                                                       key_cache.stride(2))
    a.block_table = block_tables.data_ptr()
    a.bt_stride = block_tables.stride(0)
    a.page_size = block_size
    a.num_pages = key_cache.shape[0]
    a.seq_lens = context_lens.data_ptr()
    a.batch, a.num_q_heads, a.num_kv_heads, a.m_q = num_seqs, num_q_heads, num_kv_heads, 1
    a.d_qk, a.d_v = head_size, d_v
    a.causal = 0
    a.dtype = dtype_code(query)
    a.scale = float(attn_scale)
    a.o = out.data_ptr()
    a.o_stride_b, a.o_stride_h, a.o_stride_m = out.stride(0), out.stride(1), 0
    a.status = status_word(query.device).data_ptr()
    _decode.run(a, "fa_paged_attention", query.device, stream_of(query), int(num_splits),
                reference_splits)
    return out
