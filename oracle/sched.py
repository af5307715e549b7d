"""Split heuristics and the MLA tile-scheduler spec (test oracle).

``paged_num_splits`` and ``num_splits_heuristic`` restate the reference's host
heuristics; ``mla_schedule`` is the specification of the metadata format
declared in ``include/flagattn_b200.h`` (the reference has no MLA scheduler,
so this spec is the pin the device kernel is compared with bit-for-bit).
"""

import math


def _cdiv(a, b):
    return (a + b - 1) // b


def _next_pow2(x):
    return 1 if x <= 1 else 1 << (int(x) - 1).bit_length()


def paged_num_splits(num_seqs, num_kv_heads, max_context_len, kv_block_size,
                     num_sms, num_splits=0):
    """Restates ``paged.py:54-67``: returns (num_splits, partition_size).

    partition_size is 0 when a single split is used (the reference leaves it
    unset).  With an explicit ``num_splits > 1`` the partition is
    ``next_pow2(cdiv(max_context_len, num_splits))`` (:65-67) and the count
    stays as requested.
    """
    partition_size = 0
    if num_splits == 0:
        if num_seqs * num_kv_heads > 2 * num_sms:
            num_splits = 1
            if max_context_len >= 4096:
                partition_size = max(256, kv_block_size)
                num_splits = _cdiv(max_context_len, partition_size)
        else:
            partition_size = max(256, kv_block_size)
            num_splits = _cdiv(max_context_len, partition_size)
            if max_context_len <= 1024 or kv_block_size >= 256:
                num_splits = 1
    elif num_splits > 1:
        partition_size = _next_pow2(_cdiv(max_context_len, num_splits))
    if num_splits == 1:
        partition_size = 0
    return num_splits, partition_size


def num_splits_heuristic(B, H, M, N, BLOCK_M, BLOCK_N, num_sms, max_splits):
    """Restates ``split_kv.py:247-276`` (FA2-style wave-efficiency rule)."""
    nb = B * H * _cdiv(M, BLOCK_M)
    if nb >= 0.8 * num_sms:
        return 1
    num_n_blocks = _cdiv(N, BLOCK_N)

    def available(s):
        per = _cdiv(num_n_blocks, s)
        return s == 1 or (per * s - num_n_blocks < per)

    def efficiency(s):
        n_waves = (nb * s) / num_sms
        return n_waves / math.ceil(n_waves)

    best = 0.0
    plans = []
    for s in range(1, min(num_sms, num_n_blocks, max_splits) + 1):
        if available(s):
            e = efficiency(s)
            plans.append((s, e))
            best = max(best, e)
    for s, e in plans:
        if e >= 0.85 * best:
            return s
    return 1


def mla_schedule(lens, num_parts, block_n=64, fixed=5):
    """Metadata spec: returns (tile_meta [num_parts][8], num_splits [B+1]).

    Work is counted in 64-token blocks plus ``fixed`` blocks per piece (one
    piece = the blocks of one sequence handled by one part).  Every part gets
    ``cdiv(total, parts) + fixed`` units and takes whole remaining sequences
    while they fit, then the largest prefix of the next one that still leaves
    at least one block for the following part.  Integer-only, so the device
    kernel reproduces it exactly.
    """
    B = len(lens)
    nb = [_cdiv(int(x), block_n) if int(x) > 0 else 0 for x in lens]
    total = sum(nb) + fixed * B
    payload = _cdiv(total, num_parts) + fixed
    meta = [[0] * 8 for _ in range(num_parts)]
    cnt = [0] * B
    b, blk = 0, 0
    for p in range(num_parts):
        begin_b, begin_blk = b, blk
        begin_idx = cnt[b] if b < B else 0
        pieces, end_b, end_blk = 0, b, blk
        remain = payload
        while b < B:
            left = nb[b] - blk
            if fixed + left <= remain:
                remain -= fixed + left
                cnt[b] += 1
                pieces += 1
                end_b, end_blk = b, nb[b]
                b += 1
                blk = 0
            else:
                take = remain - fixed
                if take > 0:
                    cnt[b] += 1
                    pieces += 1
                    blk += take
                    end_b, end_blk = b, blk
                break
        meta[p] = [begin_b, begin_blk, end_b, end_blk, begin_idx, pieces, 0, 0]
    prefix = [0] * (B + 1)
    for i in range(B):
        prefix[i + 1] = prefix[i] + cnt[i]
    return meta, prefix


def gqa_schedule(lens, hkv, parts, block_n=128):
    """Spec of the grouped-query decode's balanced schedule (the tensor-core
    kernel's per-CTA share; the reference has no counterpart, its split is
    the fixed partition rule of ``paged.py:54-67``).

    Entries e = b * hkv + h (sequence b, kv head h) lie on one cost line in
    order; entry e costs 1 + blocks(len_b) units (block_n tokens per block,
    the leading unit standing for the per-piece overhead), so its blocks sit
    at units X(e) + 1 + j.  With T units in all and P = min(parts, T), CTA p
    takes units [p T // P, (p + 1) T // P): the blocks there, and an empty
    entry whose leading unit is there.  A split entry's first piece (in CTA
    p_lo) goes to slot P + p_lo, its later pieces (CTA p) to slot p.

    Returns (pieces, merge): pieces[p] lists (entry, tok0, tok_end, final,
    slot) of CTA p; merge[e] = (first slot or -1 when unsplit, first later
    slot, number of later pieces), as the kernel writes it.  Integer-only.
    """
    lens = [int(x) for x in lens]
    B = len(lens)
    nb = [_cdiv(x, block_n) if x > 0 else 0 for x in lens]
    scan = [0]
    for b in range(B):
        scan.append(scan[-1] + 1 + nb[b])
    T = hkv * scan[B]
    P = min(parts, T)
    E = B * hkv

    def X(e):
        b, h = divmod(e, hkv)
        return hkv * scan[b] + h * (1 + nb[b])

    def part_of(u):
        return min(P - 1, ((u + 1) * P + T - 1) // T - 1)

    pieces = [[] for _ in range(parts)]
    merge = [None] * E
    for p in range(P):
        a0, a1 = p * T // P, (p + 1) * T // P
        for e in range(E):
            x, b = X(e), e // hkv
            n = nb[b]
            j0 = min(max(a0 - x - 1, 0), n)
            j1 = min(max(a1 - x - 1, 0), n)
            if not (j1 > j0 if n > 0 else a0 <= x < a1):
                continue
            p_lo = part_of(x + 1) if n else p
            p_hi = part_of(x + n) if n else p
            final = p_lo == p_hi
            slot = -1 if final else (P + p if j0 == 0 else p)
            pieces[p].append((e, j0 * block_n, min(j1 * block_n, max(lens[b], 0)), final, slot))
            if j0 == 0:
                merge[e] = (-1 if final else P + p_lo, p_lo + 1, p_hi - p_lo)
    return pieces, merge
