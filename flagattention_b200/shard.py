"""Multi-GPU sharding of MLA decode (one process per GPU, torch.distributed).

The reference is single-GPU; its split-KV merge algebra (split_kv.py:198-228)
is what makes both modes exact:

* **Batched decode** -- ``partition_sequences`` assigns whole sequences to
  ranks, longest first onto the least-loaded rank (by KV bytes).  Ranks share
  nothing on the data path: no collective.
* **Long-context decode** -- ``page_range`` gives each rank an even,
  contiguous range of one sequence's KV pages.  Every rank decodes its range to
  an f32 partial (O, LSE); ``exchange_partials`` all-gathers them (NCCL over
  NVLink on GPUs, any backend in tests) and ``merge_partials`` runs the
  log-sum-exp combine kernel on every rank.
"""

import ctypes
import datetime

import torch
import torch.distributed as dist

from flagattention_b200 import _lib
from flagattention_b200._torch import dtype_code, stream_of

KV_ROW_BYTES = 576 * 2


def partition_sequences(seq_lens, world, row_bytes=KV_ROW_BYTES):
    """Greedy longest-processing-time assignment of sequences to ranks.

    Returns ``world`` sorted lists of sequence indices.  Ties go to the lower
    rank / lower index, so every rank computes the same answer.
    """
    lens = [int(x) for x in seq_lens]
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    loads = [0] * world
    bins = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        bins[r].append(i)
        loads[r] += lens[i] * row_bytes
    return [sorted(b) for b in bins]


def page_range(num_pages, world, rank):
    """Contiguous, even split of a sequence's pages: [lo, hi) for ``rank``."""
    return num_pages * rank // world, num_pages * (rank + 1) // world


def shard_pages(block_table, seq_lens, page_size, world, rank):
    """This rank's share of every sequence's KV pages, for KV-page sharding.

    block_table [B, W] and seq_lens [B] (any int array-likes; numpy or CPU
    torch).  Sequence b has ceil(len / page_size) pages; the rank keeps pages
    ``page_range(n_pages, world, rank)`` of it, so the ranks' token ranges tile
    [0, len) in order and only the last rank holding pages can hold a partial
    page.  Returns (local_block_table int32 [B, W'] with the kept page ids
    left-aligned, local_lens int32 [B]) -- page ids are unchanged, i.e. they
    still index the pool the rank's pages live in.
    """
    import numpy as np
    bt = np.asarray(block_table, np.int64)
    lens = np.asarray(seq_lens, np.int64)
    B = lens.shape[0]
    spans = []
    for b in range(B):
        n_pages = -(-int(lens[b]) // page_size)
        lo, hi = page_range(n_pages, world, rank)
        n_tok = max(0, min(int(lens[b]), hi * page_size) - lo * page_size)
        spans.append((lo, hi, n_tok))
    width = max([1] + [hi - lo for lo, hi, _ in spans])
    local_bt = np.zeros((B, width), np.int32)
    local_lens = np.zeros((B,), np.int32)
    for b, (lo, hi, n_tok) in enumerate(spans):
        local_bt[b, :hi - lo] = bt[b, lo:hi]
        local_lens[b] = n_tok
    return local_bt, local_lens


def new_group_with_timeout(backend, seconds, **kw):
    """init_process_group with a short timeout so a dead rank ends the
    collective with an error instead of hanging its peers."""
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=seconds), **kw)


def exchange_partials(part_o, part_lse, group=None):
    """All-gather each rank's partial (O, LSE) -> ([world, ...], [world, ...])."""
    world = dist.get_world_size(group)
    os_ = [torch.empty_like(part_o) for _ in range(world)]
    ls_ = [torch.empty_like(part_lse) for _ in range(world)]
    dist.all_gather(os_, part_o.contiguous(), group=group)
    dist.all_gather(ls_, part_lse.contiguous(), group=group)
    return torch.stack(os_), torch.stack(ls_)


def merge_partials(all_o, all_lse, out_dtype=torch.bfloat16):
    """Log-sum-exp merge of gathered partials on the GPU (fa_lse_combine).

    all_o: f32 [P, rows..., d_v]; all_lse: f32 [P, rows...].  Returns
    (out [rows..., d_v] of out_dtype, lse f32 [rows...]).
    """
    P = all_o.shape[0]
    d_v = all_o.shape[-1]
    rows = all_lse[0].numel()
    all_o = all_o.contiguous()
    all_lse = all_lse.contiguous()
    out = torch.empty(all_o.shape[1:], dtype=out_dtype, device=all_o.device)
    lse = torch.empty(all_lse.shape[1:], dtype=torch.float32, device=all_o.device)
    _lib.check(_lib.lib().fa_lse_combine(ctypes.c_void_p(all_o.data_ptr()),
                                         ctypes.c_void_p(all_lse.data_ptr()), P, rows, d_v,
                                         ctypes.c_void_p(out.data_ptr()), dtype_code(out),
                                         ctypes.c_void_p(lse.data_ptr()), stream_of(out)),
               "fa_lse_combine")
    return out, lse


def decode_partial(q, kcache, block_table, seq_lens, softmax_scale=None):
    """One rank's share of a KV-page-sharded decode: f32 partial (O, LSE).

    q [B, 1, h_q, 576] (replicated); kcache / block_table / seq_lens describe
    the tokens this rank holds (``shard_pages``).  Returns (part_o f32
    [B, 1, h_q, 512], part_lse f32 [B, 1, h_q]); a rank holding no token of a
    sequence gives O = 0 and LSE = -inf there, which the merge ignores.
    """
    from flagattention_b200.mla import flash_mla_with_kvcache, get_mla_metadata
    B, s_q, h_q, _ = q.shape
    if s_q != 1:
        raise _lib.Unsupported("KV-page sharding is implemented for s_q == 1 (non-causal)")
    meta, splits = get_mla_metadata(seq_lens, s_q * h_q, 1)
    part_o = torch.empty((B, s_q, h_q, 512), dtype=torch.float32, device=q.device)
    _, lse = flash_mla_with_kvcache(q, kcache, block_table, seq_lens, 512, meta, splits,
                                    softmax_scale=softmax_scale, out=part_o)
    return part_o, lse.transpose(1, 2).contiguous()     # lse rows ordered like part_o


def long_context_decode(q, kcache, block_table, seq_lens, softmax_scale=None, group=None):
    """Decode sequences whose KV pages are split across the ranks of ``group``.

    Each rank passes its own shard: ``kcache`` / ``block_table`` / ``seq_lens``
    describe the tokens it holds (``shard_pages``).  q [B, 1, h_q, 576] is
    replicated.  Returns (out [B, 1, h_q, 512] of q's dtype, lse f32
    [B, h_q, 1]) identical on every rank.
    """
    part_o, part_lse = decode_partial(q, kcache, block_table, seq_lens, softmax_scale)
    all_o, all_l = exchange_partials(part_o, part_lse, group)
    out, lse_m = merge_partials(all_o, all_l, q.dtype)
    return out, lse_m.transpose(1, 2).contiguous()
