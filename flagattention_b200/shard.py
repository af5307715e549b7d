"""Multi-GPU sharding of MLA decode (one process per GPU, torch.distributed).

The reference is single-GPU; its split-KV merge algebra (split_kv.py:198-228)
is what makes both modes exact:

* **Batched decode** -- ``partition_sequences`` assigns whole sequences to
  ranks, longest first onto the least-loaded rank (by KV bytes).  Ranks share
  nothing on the data path: no collective.
* **Long-context decode** -- ``page_range`` gives each rank an even,
  contiguous range of one sequence's KV pages.  Every rank decodes its range to
  an f32 partial (O, LSE).  ``PeerLongContextDecode`` exchanges the partials
  without a collective: the kernel that merges a rank's own split pieces
  writes each row into every rank's gather buffer (peer stores over NVLink,
  CUDA IPC mappings, ``PeerExchange``) and the merge kernel waits for all
  rows, bounded in time.  ``long_context_decode`` is the collective form: one
  all-gather of packed partials (NCCL, or any backend in tests) and
  ``merge_partials``.
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


def packed_partial(batch, h_q, d_v=512, device=None):
    """One rank's partial result of a KV-page-sharded decode, in the layout
    that travels between GPUs: f32 [batch*h_q*d_v + batch*h_q], the O rows
    (b, h) first, then their LSEs in the same row order."""
    return torch.empty(batch * h_q * (d_v + 1), dtype=torch.float32, device=device)


def unpack_partial(packed, batch, h_q, d_v=512):
    """Views (O [batch, 1, h_q, d_v], LSE [batch, h_q, 1]) of a packed partial."""
    rows = batch * h_q
    return (packed[:rows * d_v].view(batch, 1, h_q, d_v),
            packed[rows * d_v:rows * (d_v + 1)].view(batch, h_q, 1))


def exchange_partials(packed, group=None):
    """All-gather every rank's packed partial with ONE collective (NCCL over
    NVLink on GPUs, any backend in tests): returns f32 [world, packed.numel()],
    rank r's partial in row r."""
    world = dist.get_world_size(group)
    gathered = torch.empty(world * packed.numel(), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed.contiguous(), group=group)
    return gathered.view(world, packed.numel())


def merge_partials(gathered, rows, d_v=512, out_dtype=torch.bfloat16):
    """Log-sum-exp merge of gathered packed partials on the GPU
    (fa_lse_combine_strided, the algebra of split_kv.py:198-228).

    gathered: f32 [P, rows*(d_v+1)] (``exchange_partials``).  Returns
    (out [rows, d_v] of out_dtype, lse f32 [rows]).
    """
    P, n = gathered.shape
    if n != rows * (d_v + 1):
        raise _lib.InvalidArgument(f"packed partials of {n} floats, expected rows*(d_v+1)")
    gathered = gathered.contiguous()
    out = torch.empty((rows, d_v), dtype=out_dtype, device=gathered.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=gathered.device)
    base = gathered.data_ptr()
    _lib.check(_lib.lib().fa_lse_combine_strided(ctypes.c_void_p(base), n,
                                                 ctypes.c_void_p(base + rows * d_v * 4), n, P,
                                                 rows, d_v, ctypes.c_void_p(out.data_ptr()),
                                                 dtype_code(out), ctypes.c_void_p(lse.data_ptr()),
                                                 stream_of(out)),
               "fa_lse_combine_strided")
    return out, lse


class PartialDecode:
    """One rank's share of a KV-page-sharded decode, bound once: the decode
    writes its f32 partial (O, LSE) straight into the packed buffer that the
    all-gather sends, so no copy sits between the kernel and the collective.

    q [B, 1, h_q, 576] (replicated on every rank); kcache / block_table /
    seq_lens describe the tokens this rank holds (``shard_pages``).  A rank
    holding no token of a sequence gives O = 0 and LSE = -inf there, which
    the merge ignores.
    """

    def __init__(self, q, kcache, block_table, seq_lens, softmax_scale=None, num_sm_parts=None):
        from flagattention_b200.mla import MlaCall, get_mla_metadata
        B, s_q, h_q, _ = q.shape
        if s_q != 1:
            raise _lib.Unsupported("KV-page sharding is implemented for s_q == 1 (non-causal)")
        self.batch, self.h_q = B, h_q
        meta, splits = get_mla_metadata(seq_lens, s_q * h_q, 1,
                                        num_sm_parts_override=num_sm_parts)
        self.packed = packed_partial(B, h_q, 512, q.device)
        o, lse = unpack_partial(self.packed, B, h_q)
        scale = 576 ** -0.5 if softmax_scale is None else softmax_scale
        self.call = MlaCall(q, kcache, kcache.stride(0), kcache.stride(1), kcache.shape[0],
                            kcache.shape[1], block_table, seq_lens, 0, meta, splits, o, lse, scale)

    def run(self):
        """Decode into ``self.packed`` (asynchronous on the current stream)."""
        self.call.run()
        return self.packed


class PeerExchange:
    """Gather buffer of packed partials shared by the ranks of ``group``
    through CUDA IPC, for exchanging partials with peer stores instead of a
    collective (``fa_mla_combine_push`` / ``fa_lse_merge_wait``).

    Each rank allocates two gather buffers f32 [world][rows * (d_v + 1)]
    plus uint64 counters [world] (zeroed), exports them, and maps every
    peer's.  Exchange k uses buffer k % 2: a rank can push exchange k + 1
    while a slower peer still merges exchange k, but not exchange k + 2 (its
    own merge of k + 1 waited for that peer's push of k + 1, which the peer
    issues after its merge of k).  ``parts(k)`` / ``counters`` are this rank's
    device addresses of every rank's buffer for exchange k (ctypes arrays,
    index = rank).  The process-group call is only the one-time exchange of
    the IPC handles (``all_gather_object``).  Every rank must run the same
    sequence of exchanges; ``epoch`` counts them.  ``close`` unmaps the peers
    (call it on every rank, after a barrier, before the buffers are dropped).
    """

    def __init__(self, rows, d_v=512, device=None, group=None):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if world > _lib.FA_EXCHANGE_MAX_RANKS:
            raise _lib.Unsupported(f"peer exchange supports up to {_lib.FA_EXCHANGE_MAX_RANKS} ranks")
        self.world, self.rank, self.rows, self.d_v = world, rank, rows, d_v
        self._half = (world * rows * (d_v + 1) * 4 + 255) // 256 * 256
        self._cnt_off = 2 * self._half
        self.buf = torch.zeros(self._cnt_off + 8 * world, dtype=torch.uint8, device=device)
        handle = ctypes.create_string_buffer(_lib.FA_IPC_HANDLE_BYTES)
        off = ctypes.c_uint64(0)
        _lib.check(_lib.lib().fa_ipc_export(ctypes.c_void_p(self.buf.data_ptr()), handle,
                                            ctypes.byref(off)), "fa_ipc_export")
        mine = (bytes(handle.raw), int(off.value))
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = []
        addr = []
        for r, (h, o) in enumerate(everyone):
            if r == rank:
                addr.append(self.buf.data_ptr())
                continue
            base = ctypes.c_void_p(0)
            _lib.check(_lib.lib().fa_ipc_open(ctypes.create_string_buffer(h, len(h)),
                                              ctypes.byref(base)), "fa_ipc_open")
            self._opened.append(base)
            addr.append(base.value + o)
        self._parts = [(ctypes.c_void_p * world)(*[a + h * self._half for a in addr])
                       for h in (0, 1)]
        self.counters = (ctypes.c_void_p * world)(*[a + self._cnt_off for a in addr])
        self.epoch = 0

    def parts(self, epoch):
        return self._parts[epoch % 2]

    def local_parts(self, epoch):
        return self.buf.data_ptr() + (epoch % 2) * self._half

    @property
    def local_counters(self):
        return self.buf.data_ptr() + self._cnt_off

    def close(self):
        for base in self._opened:
            _lib.check(_lib.lib().fa_ipc_close(base), "fa_ipc_close")
        self._opened = []


class PeerLongContextDecode:
    """Long-context decode with the KV pages split over the ranks, partials
    exchanged by peer stores: per call one decode kernel and one cooperative
    exchange kernel that merges this rank's split pieces, stores each row
    straight into every rank's gather buffer (over NVLink), waits for every
    rank's rows (at most ``timeout_s``) and merges them (``push`` / ``merge``
    are the same two steps as separate launches).  No collective library call on the
    data path.  q [B, 1, h_q, 576] replicated; kcache / block_table /
    seq_lens are this rank's pages (``shard_pages``).  ``run`` returns
    (out [B, 1, h_q, 512] of q's dtype, lse f32 [B, h_q, 1]); a timed-out wait
    leaves them unwritten and sets the device status word (``read_status``).
    """

    def __init__(self, q, kcache, block_table, seq_lens, softmax_scale=None, group=None,
                 timeout_s=2.0):
        from flagattention_b200._torch import status_word
        B, _, h_q, _ = q.shape
        self.part = PartialDecode(q, kcache, block_table, seq_lens, softmax_scale)
        self.rows = B * h_q
        self.x = PeerExchange(self.rows, 512, q.device, group)
        self.out = torch.empty((B, 1, h_q, 512), dtype=q.dtype, device=q.device)
        self.lse = torch.empty((B, h_q, 1), dtype=torch.float32, device=q.device)
        self.status = status_word(q.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self._stream = stream_of(q)

    def decode(self):
        """This rank's decode kernel (its pages) into the split workspace /
        its f32 rows."""
        _lib.check(_lib.lib().fa_mla_decode_partial(self.part.call._ref, self._stream),
                   "fa_mla_decode_partial")

    def push(self):
        """Merge this rank's split pieces and store every row into every
        rank's gather buffer for the next exchange."""
        x = self.x
        x.epoch += 1
        _lib.check(_lib.lib().fa_mla_combine_push(self.part.call._ref, x.parts(x.epoch),
                                                  x.counters, x.world, x.rank, self._stream),
                   "fa_mla_combine_push")

    def merge(self):
        """Wait for every rank's rows of the current exchange, merge them."""
        x = self.x
        _lib.check(_lib.lib().fa_lse_merge_wait(
            ctypes.c_void_p(x.local_parts(x.epoch)), x.world, self.rows, 512,
            ctypes.c_void_p(x.local_counters), x.epoch * self.rows,
            ctypes.c_void_p(self.out.data_ptr()), dtype_code(self.out),
            ctypes.c_void_p(self.lse.data_ptr()), ctypes.c_void_p(self.status.data_ptr()),
            self.timeout_ns, self._stream), "fa_lse_merge_wait")

    def exchange(self):
        """Push and merge in one cooperative launch (fa_mla_combine_exchange)."""
        x = self.x
        x.epoch += 1
        _lib.check(_lib.lib().fa_mla_combine_exchange(
            self.part.call._ref, x.parts(x.epoch), x.counters, x.world, x.rank,
            x.epoch * self.rows, ctypes.c_void_p(self.out.data_ptr()), dtype_code(self.out),
            ctypes.c_void_p(self.lse.data_ptr()), ctypes.c_void_p(self.status.data_ptr()),
            self.timeout_ns, self._stream), "fa_mla_combine_exchange")

    def run(self):
        """Decode, then push + merge in one launch."""
        self.decode()
        self.exchange()
        return self.out, self.lse

    def close(self):
        self.x.close()


def decode_partial(q, kcache, block_table, seq_lens, softmax_scale=None):
    """One rank's packed f32 partial (see ``PartialDecode``)."""
    return PartialDecode(q, kcache, block_table, seq_lens, softmax_scale).run()


def long_context_decode(q, kcache, block_table, seq_lens, softmax_scale=None, group=None):
    """Decode sequences whose KV pages are split across the ranks of ``group``.

    Each rank passes its own shard: ``kcache`` / ``block_table`` / ``seq_lens``
    describe the tokens it holds (``shard_pages``).  q [B, 1, h_q, 576] is
    replicated.  Each rank decodes its pages into a packed partial, one
    all-gather exchanges the partials, and every rank merges them on its GPU.
    Returns (out [B, 1, h_q, 512] of q's dtype, lse f32 [B, h_q, 1]),
    identical on every rank.
    """
    B, _, h_q, _ = q.shape
    packed = decode_partial(q, kcache, block_table, seq_lens, softmax_scale)
    gathered = exchange_partials(packed, group)
    out, lse = merge_partials(gathered, B * h_q, 512, q.dtype)
    return out.view(B, 1, h_q, 512), lse.view(B, h_q, 1)
