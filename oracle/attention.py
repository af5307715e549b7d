"""numpy restatement of FlagAttention's attention references (test oracle).

All math is float32 like the reference's upcast path; inputs are numpy arrays
(bf16/f16 data must be converted to float32 by the caller, which is exact).
"""

import math

import numpy as np


def _softmax_rows(s):
    """torch.softmax(S, dim=-1, dtype=float32) semantics, rows of -inf -> 0."""
    m = np.max(s, axis=-1, keepdims=True)
    m = np.where(np.isneginf(m), 0.0, m).astype(np.float32)
    e = np.exp(s - m)
    z = np.sum(e, axis=-1, keepdims=True)
    return np.where(z > 0, e / np.where(z > 0, z, 1), 0.0).astype(np.float32)


def _logsumexp_rows(s):
    """torch.logsumexp(S, dim=-1): max + log(sum(exp(S - max))), -inf if empty."""
    m = np.max(s, axis=-1, keepdims=True)
    safe = np.where(np.isneginf(m), 0.0, m).astype(np.float32)
    z = np.sum(np.exp(s - safe), axis=-1, keepdims=True)
    with np.errstate(divide="ignore"):
        out = safe + np.log(z)
    return out[..., 0].astype(np.float32)


def flash_attention(q, k, v, causal, sm_scale=None, return_log_normalizer=False):
    """Restates ``testing/flash.py:19-84`` with ``upcast=True``, no dropout.

    q [B, H, M, D], k [B, Hk, N, D], v [B, Hk, N, Dv] (Dv may differ from D,
    as the reference allows).  Grouped heads: query head h reads kv head
    h // (H // Hk) (``repeat_interleave``, :43-44).  Causal masking is
    bottom-right aligned, ``ms + p_seq >= ns`` (:47-55).  The log normaliser
    is ``logsumexp`` of the scaled scores (:59).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, H, M, D = q.shape
    Hk, N = k.shape[1], k.shape[2]
    assert H % Hk == 0
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    g = H // Hk
    # grouped heads: query head h reads kv head h // g.  Broadcasting over the
    # group axis gives the same products as the reference's repeat_interleave
    # without materialising g copies of K and V.
    qg = q.reshape(B, Hk, g, M, D)
    s = np.matmul(qg, np.swapaxes(k, 2, 3)[:, :, None]) * np.float32(sm_scale)  # [B,Hk,g,M,N]
    if causal:
        p_seq = N - M
        mask = (np.arange(M)[:, None] + p_seq) >= np.arange(N)[None, :]
        s = np.where(mask, s, -np.inf).astype(np.float32)
    lse = _logsumexp_rows(s).reshape(B, H, M) if return_log_normalizer else None
    p = _softmax_rows(s)
    o = np.matmul(p, v[:, :, None]).astype(np.float32).reshape(B, H, M, v.shape[-1])
    if return_log_normalizer:
        return o, lse
    return o


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, scale):
    """Restates ``testing/paged.py:18-65`` (returns float32, before the cast).

    query [S, Hq, D]; key_cache [P, Hkv, page, D]; value_cache
    [P, Hkv, page, Dv].  Token j of sequence i is row ``j % page`` of page
    ``block_tables[i][j // page]`` (:44-50); grouped heads repeat the kv head
    (:53-56); fp32 bmm -> softmax -> bmm (:58-60).  Unlike the reference the
    value width may differ from the key width (the MLA case, where values are
    the first 512 of 576 dims).
    """
    query = np.asarray(query, np.float32)
    key_cache = np.asarray(key_cache, np.float32)
    value_cache = np.asarray(value_cache, np.float32)
    S, Hq, _ = query.shape
    Hkv = key_cache.shape[1]
    page = key_cache.shape[2]
    dv = value_cache.shape[3]
    g = Hq // Hkv
    out = np.zeros((S, Hq, dv), np.float32)
    for i in range(S):
        n = int(context_lens[i])
        if n <= 0:
            continue
        tok = np.arange(n)
        pages = np.asarray(block_tables[i])[tok // page]
        keys = key_cache[pages, :, tok % page, :]      # [n, Hkv, D]
        vals = value_cache[pages, :, tok % page, :]    # [n, Hkv, Dv]
        # head h uses kv head h // g (the reference's repeat_interleave)
        qh = query[i].reshape(Hkv, g, -1)              # [Hkv, g, D]
        s = np.matmul(qh, np.transpose(keys, (1, 2, 0))) * np.float32(scale)  # [Hkv, g, n]
        p = _softmax_rows(s)
        out[i] = np.matmul(p, np.transpose(vals, (1, 0, 2))).reshape(Hq, dv)
    return out


def _gather_pages(kcache, block_table_row, n):
    """Rows 0..n-1 of one sequence from a [P, page, 1, D] (or [P, page, D]) pool."""
    kc = kcache.reshape(kcache.shape[0], kcache.shape[1], -1)
    page = kc.shape[1]
    tok = np.arange(n)
    return kc[np.asarray(block_table_row)[tok // page], tok % page, :]


def mla_decode_dense(q, kcache, block_table, seq_lens, d_v, scale, causal=False):
    """Dense paged MLA decode oracle.

    q [B, s_q, H, D]; kcache [P, page, 1, D]; values are the first d_v dims
    of each key row.  Per sequence the pages are gathered (``testing/paged.py
    :44-50``) and ``flash_attention`` above (``testing/flash.py``) runs with
    one kv head, so causal MTP is bottom-right aligned.  Returns
    (out [B, s_q, H, d_v] f32, lse [B, H, s_q] f32); a zero-length sequence
    gives out 0 and lse -inf.
    """
    q = np.asarray(q, np.float32)
    kcache = np.asarray(kcache, np.float32)
    B, s_q, H, D = q.shape
    out = np.zeros((B, s_q, H, d_v), np.float32)
    lse = np.full((B, H, s_q), -np.inf, np.float32)
    for b in range(B):
        n = int(seq_lens[b])
        if n <= 0:
            continue
        rows = _gather_pages(kcache, block_table[b], n)            # [n, D]
        k = rows[None, None]                                        # [1,1,n,D]
        v = rows[None, None, :, :d_v]
        qb = np.transpose(q[b], (1, 0, 2))[None]                    # [1,H,s_q,D]
        o, l = flash_attention(qb, k, v, causal, scale, True)
        out[b] = np.transpose(o[0], (1, 0, 2))
        lse[b] = l[0]
    return out, lse


def mla_decode_sparse(q, kcache, indices, d_v, scale):
    """Top-k sparse MLA decode oracle (no reference kernel exists).

    indices [B, s_q, topk] hold physical rows of the pool viewed as
    [P*page, D]; negative or out-of-range entries are dropped, then
    ``flash_attention`` (``testing/flash.py``) runs non-causally on the
    gathered rows.  A query with no valid index gives out 0, lse -inf.
    """
    q = np.asarray(q, np.float32)
    kc = np.asarray(kcache, np.float32).reshape(-1, q.shape[-1])
    B, s_q, H, D = q.shape
    out = np.zeros((B, s_q, H, d_v), np.float32)
    lse = np.full((B, H, s_q), -np.inf, np.float32)
    for b in range(B):
        for i in range(s_q):
            idx = np.asarray(indices[b, i])
            idx = idx[(idx >= 0) & (idx < kc.shape[0])]
            if idx.size == 0:
                continue
            rows = kc[idx]
            o, l = flash_attention(q[b, i][None, :, None, :], rows[None, None],
                                   rows[None, None, :, :d_v], False, scale, True)
            out[b, i] = o[0, :, 0, :]
            lse[b, :, i] = l[0, :, 0]
    return out, lse


def lse_combine(part_o, part_lse):
    """Restates ``split_kv.py:198-228`` (two-pass log-sum-exp merge).

    part_o [S, ..., Dv], part_lse [S, ...]; pass 1 is the online logsumexp
    (:198-211), pass 2 sums ``o_s * exp(l_s - l_acc)`` (:213-228).  Splits
    with lse -inf contribute nothing; all-empty rows give 0 / -inf.
    """
    part_o = np.asarray(part_o, np.float32)
    part_lse = np.asarray(part_lse, np.float32)
    m = np.full(part_lse.shape[1:], -np.inf, np.float32)
    acc = np.zeros(part_lse.shape[1:], np.float32)
    for s in range(part_lse.shape[0]):
        l_s = part_lse[s]
        m_new = np.maximum(m, l_s)
        safe = np.where(np.isneginf(m_new), 0.0, m_new)
        acc = acc * np.exp(m - safe) + np.exp(l_s - safe)
        m = m_new
    with np.errstate(divide="ignore"):
        l_acc = np.where(np.isneginf(m), -np.inf, m + np.log(np.where(acc > 0, acc, 1)))
    o = np.zeros(part_o.shape[1:], np.float32)
    for s in range(part_lse.shape[0]):
        w = np.where(np.isneginf(l_acc), 0.0, np.exp(part_lse[s] - np.where(np.isneginf(l_acc), 0, l_acc)))
        o += part_o[s] * w[..., None]
    return o.astype(np.float32), l_acc.astype(np.float32)


def paged_v2_reduce(tmp_out, m_i, l_i):
    """Restates ``paged.py:416-442`` (m/l form of the split merge).

    tmp_out [S, G, D] normalised partial outputs, m_i / l_i [S, G] running
    max and sum of each split (scores pre-scaled).  Global max over splits
    (:416-418), rescaled sums (:422-425), weights r = l_i / l (:427), output
    sum of tmp_out * r (:442).
    """
    tmp_out = np.asarray(tmp_out, np.float32)
    m_i = np.asarray(m_i, np.float32)
    l_i = np.asarray(l_i, np.float32)
    m = np.max(m_i, axis=0)
    l_scaled = l_i * np.exp(m_i - m[None])
    l_tot = np.sum(l_scaled, axis=0)
    r = l_scaled / l_tot[None]
    return np.sum(tmp_out * r[..., None], axis=0).astype(np.float32)


def mla_append_rows(cache, rows, slots):
    """Paged write of new latent rows (no reference function: the pool layout
    of ``paged.py:22-23``, ``[pages, page_size, heads, dim]``).

    Row r of ``rows`` goes to ``cache[slots[r] // page_size, slots[r] %
    page_size, 0]``; a negative slot or one past the pool skips the row.
    Returns a new array (the input is not modified).
    """
    out = np.array(cache, copy=True)
    page = out.shape[1]
    total = out.shape[0] * page
    for r, s in enumerate(np.asarray(slots, np.int64)):
        if 0 <= s < total:
            out[s // page, s % page, 0] = rows[r]
    return out
