"""MLA decode operators: the metadata call and the with-kvcache call.

Signatures follow the FlashMLA-style convention the reference path is
specified against (``get_mla_metadata`` / ``flash_mla_with_kvcache``); the
math is the reference's paged decode (``paged.py:208-363``) at the MLA shape:
576-dim latent+rope keys, values = the first 512 dims of the same rows, all
query heads sharing one latent head.
"""

import ctypes

import torch

from flagattention_b200 import _lib
from flagattention_b200._torch import (dtype_code, ptr, require_cuda, sm_count, status_word,
                                       stream_of)

D_QK, D_V = 576, 512


def num_sm_parts(device, s_q, h_q, sparse):
    out = ctypes.c_int32(0)
    dev = device.index if device.index is not None else torch.cuda.current_device()
    _lib.check(_lib.lib().fa_mla_num_sm_parts(dev, s_q, h_q, int(bool(sparse)), ctypes.byref(out)),
               "fa_mla_num_sm_parts")
    return out.value


def get_mla_metadata(cache_seqlens, num_q_tokens_per_head_k, num_heads_k, num_heads_q=None,
                     is_fp8_kvcache=False, topk=None, num_sm_parts_override=None):
    """Tile-scheduler metadata for ``flash_mla_with_kvcache``.

    cache_seqlens: int32 [batch] on the GPU.  num_q_tokens_per_head_k =
    s_q * h_q // h_k.  For sparse decode pass ``topk`` and ``num_heads_q``.
    Returns (tile_scheduler_metadata int32 [num_sm_parts, 8],
    num_splits int32 [batch + 1]), computed by the device scheduler kernel.
    """
    require_cuda(cache_seqlens)
    if is_fp8_kvcache:
        raise _lib.Unsupported("fp8 latent cache is not implemented")
    if num_heads_k != 1:
        raise _lib.Unsupported("MLA decode needs one latent kv head")
    if cache_seqlens.dtype != torch.int32:
        raise _lib.InvalidArgument("cache_seqlens must be int32")
    dev = cache_seqlens.device
    rows = int(num_q_tokens_per_head_k) * int(num_heads_k)
    sparse = topk is not None
    if sparse:
        if num_heads_q is None:
            raise _lib.InvalidArgument("sparse metadata needs num_heads_q")
        s_q, h_q = rows // num_heads_q, num_heads_q
    else:
        s_q, h_q = 1, rows
    parts = num_sm_parts_override or num_sm_parts(dev, s_q, h_q, sparse)
    batch = cache_seqlens.shape[0]
    seq = cache_seqlens.contiguous()
    meta = torch.empty((parts, _lib.FA_MLA_META_INTS), dtype=torch.int32, device=dev)
    splits = torch.empty((batch + 1,), dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().fa_mla_get_metadata(ptr(seq), batch, int(topk) if sparse else 0, parts,
                                              ptr(meta), ptr(splits), stream_of(seq)),
               "fa_mla_get_metadata")
    return meta, splits


_workspaces = {}


def _workspace(device, batch, s_q, h_q, parts):
    """Split scratch (f32 partial O and LSE), cached per device and grown;
    returns (buffer, part_o address, part_lse address)."""
    po, pl = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _lib.check(_lib.lib().fa_mla_workspace_size(batch, s_q, h_q, D_V, parts, ctypes.byref(po),
                                                ctypes.byref(pl)), "fa_mla_workspace_size")
    off = (po.value + 255) // 256 * 256
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < off + pl.value:
        buf = torch.empty(off + pl.value, dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf, buf.data_ptr(), buf.data_ptr() + off


class MlaCall:
    """Decode arguments bound once (C struct + the tensors it points to).

    q: [B, s_q, h_q, 576] view (last dim dense); out: [B, s_q, h_q, 512]
    view of q's dtype or float32; lse: f32 [B, h_q, s_q] contiguous.
    Strides are read off the views.  ``run`` = decode + combine;
    ``partial`` / ``combine`` launch the two kernels separately.
    """

    def __init__(self, q, kcache, kv_stride_page, kv_stride_tok, num_pages, page_size,
                 block_table, seq_lens, n_ctx, tile_meta, num_splits, out, lse, scale,
                 causal=False, indices=None):
        B, s_q, h_q, d_qk = q.shape
        parts = tile_meta.shape[0]
        ws, po, pl = _workspace(q.device, B, s_q, h_q, parts)
        # the workspace is kept alive with the call: a later, larger call
        # replaces the cached buffer but must not free this one under it
        self._keep = (q, kcache, block_table, seq_lens, tile_meta, num_splits, out, lse, indices,
                      ws)
        a = _lib.MlaArgs()
        a.q = q.data_ptr()
        a.q_stride_b, a.q_stride_s, a.q_stride_h = q.stride(0), q.stride(1), q.stride(2)
        a.kcache = kcache.data_ptr()
        a.kv_stride_page, a.kv_stride_tok = kv_stride_page, kv_stride_tok
        a.num_pages, a.page_size = num_pages, page_size
        a.block_table = block_table.data_ptr() if block_table is not None else None
        a.bt_stride = block_table.stride(0) if block_table is not None else 0
        a.seq_lens = seq_lens.data_ptr() if seq_lens is not None else None
        a.n_ctx = n_ctx
        if indices is not None:
            a.indices = indices.data_ptr()
            a.idx_stride_b, a.idx_stride_s = indices.stride(0), indices.stride(1)
            a.topk = indices.shape[-1]
        a.tile_meta = tile_meta.data_ptr()
        a.num_splits = num_splits.data_ptr()
        a.num_sm_parts = parts
        a.out = out.data_ptr()
        a.o_stride_b, a.o_stride_s, a.o_stride_h = out.stride(0), out.stride(1), out.stride(2)
        a.lse = lse.data_ptr()
        a.part_o, a.part_lse = po, pl
        a.batch, a.s_q, a.h_q, a.d_qk, a.d_v = B, s_q, h_q, d_qk, out.shape[-1]
        a.causal = int(bool(causal))
        a.dtype = dtype_code(q)
        a.out_dtype = dtype_code(out)
        a.scale = float(scale)
        a.status = status_word(q.device).data_ptr()
        self.args = a
        self._ref = ctypes.byref(a)
        self._stream = stream_of(q)

    def run(self):
        _lib.check(_lib.lib().fa_mla_decode(self._ref, self._stream), "fa_mla_decode")

    def partial(self):
        _lib.check(_lib.lib().fa_mla_decode_partial(self._ref, self._stream),
                   "fa_mla_decode_partial")

    def combine(self):
        _lib.check(_lib.lib().fa_mla_combine(self._ref, self._stream), "fa_mla_combine")


def mla_decode(*args, **kwargs):
    """One decode (+ combine) launch; arguments as for ``MlaCall``."""
    MlaCall(*args, **kwargs).run()


def flash_mla_with_kvcache(q, k_cache, block_table, cache_seqlens, head_dim_v,
                           tile_scheduler_metadata, num_splits, softmax_scale=None, causal=False,
                           is_fp8_kvcache=False, indices=None, out=None):
    """MLA decode over a paged latent cache.

    q: [B, s_q, h_q, 576] bf16/f16; k_cache: [num_blocks, page_size, 1, 576];
    block_table: int32 [B, max_blocks] (may be None for sparse);
    cache_seqlens: int32 [B] (may be None for sparse); head_dim_v must be 512.
    indices (sparse): int32 [B, s_q, topk] of physical rows
    ``page * page_size + offset``; -1 entries are masked.
    Returns (out [B, s_q, h_q, 512], softmax_lse f32 [B, h_q, s_q]).
    """
    require_cuda(q, k_cache, block_table, cache_seqlens, indices, tile_scheduler_metadata,
                 num_splits)
    if is_fp8_kvcache:
        raise _lib.Unsupported("fp8 latent cache is not implemented")
    if head_dim_v != D_V or q.shape[-1] != D_QK or k_cache.shape[-1] != D_QK:
        raise _lib.InvalidArgument(f"MLA shapes are d_qk={D_QK}, d_v={D_V}")
    if k_cache.dim() != 4 or k_cache.shape[2] != 1:
        raise _lib.InvalidArgument("k_cache must be [num_blocks, page_size, 1, 576]")
    if k_cache.dtype != q.dtype:
        raise _lib.InvalidArgument("q and k_cache dtypes differ")
    if indices is not None and causal:
        raise _lib.InvalidArgument("causal must be False for sparse decode")
    if indices is None and (block_table is None or cache_seqlens is None):
        raise _lib.InvalidArgument("dense decode needs block_table and cache_seqlens")
    B, s_q, h_q, _ = q.shape
    if softmax_scale is None:
        softmax_scale = D_QK ** -0.5
    if out is None:
        out = torch.empty((B, s_q, h_q, D_V), dtype=q.dtype, device=q.device)
    elif out.shape != (B, s_q, h_q, D_V) or out.dtype not in (q.dtype, torch.float32):
        raise _lib.InvalidArgument("out must be [B, s_q, h_q, 512] of q's dtype or float32")
    lse = torch.empty((B, h_q, s_q), dtype=torch.float32, device=q.device)
    if q.stride(-1) != 1:
        q = q.contiguous()
    if indices is not None and indices.dtype != torch.int32:
        raise _lib.InvalidArgument("indices must be int32")
    mla_decode(q, k_cache, k_cache.stride(0), k_cache.stride(1), k_cache.shape[0],
               k_cache.shape[1], block_table, cache_seqlens, 0, tile_scheduler_metadata,
               num_splits, out, lse, softmax_scale, causal, indices)
    return out, lse


def append_kv_rows(kv_rows, k_cache, slot_mapping):
    """Write new tokens' latent rows into the paged cache, in place.

    kv_rows: [n, 576] (or [n, 1, 576]) in k_cache's dtype, unit inner stride;
    k_cache: [num_blocks, page_size, 1, 576]; slot_mapping: int64 [n] of pool
    rows (block * page_size + offset in block).  A negative slot skips its
    row (padding).  Slots must be distinct.  The step before a decode whose
    cache_seqlens count the appended tokens.  No function in the reference
    (its caches are written by the caller, in the layout of paged.py:22-23).
    """
    require_cuda(kv_rows, k_cache, slot_mapping)
    if kv_rows.dim() == 3:
        kv_rows = kv_rows.reshape(kv_rows.shape[0], kv_rows.shape[-1])
    if kv_rows.dim() != 2 or kv_rows.shape[-1] != D_QK:
        raise _lib.InvalidArgument("kv_rows must be [n, 576]")
    if k_cache.dim() != 4 or k_cache.shape[2] != 1 or k_cache.shape[-1] != D_QK:
        raise _lib.InvalidArgument("k_cache must be [num_blocks, page_size, 1, 576]")
    if kv_rows.dtype != k_cache.dtype:
        raise _lib.InvalidArgument("kv_rows and k_cache dtypes differ")
    if k_cache.stride(-1) != 1:
        raise _lib.InvalidArgument("k_cache must have a unit inner stride (576 contiguous dims)")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or \
            slot_mapping.shape[0] != kv_rows.shape[0]:
        raise _lib.InvalidArgument("slot_mapping must be int64 [n]")
    if kv_rows.stride(-1) != 1:
        kv_rows = kv_rows.contiguous()
    slot_mapping = slot_mapping.contiguous()
    _lib.check(_lib.lib().fa_mla_append_rows(ptr(kv_rows), kv_rows.stride(0), ptr(slot_mapping),
                                             kv_rows.shape[0], ptr(k_cache), k_cache.stride(0),
                                             k_cache.stride(1), k_cache.shape[0],
                                             k_cache.shape[1], dtype_code(k_cache),
                                             stream_of(k_cache)),
               "fa_mla_append_rows")
    return k_cache
