"""Reference-compatible split-KV flash decoding on contiguous keys.

``flash_attention_split_kv(q, k, v, causal=False, sm_scale=None)`` follows
``split_kv.py:279-344`` and ``flash_attention(..., return_log_normalizer=True)``
the split branch of ``flash.py:72-171`` (forward only): q [B, H, M, D],
k [B, Hk, N, D], v [B, Hk, N, Dv], bottom-right causal masking, grouped
heads.  bf16/f16 with head size 16, 32, 64, 128 or 256 (up to 128 query
rows per kv head) runs the tcgen05 grouped-query kernel with the device scheduler's
balanced split; other shapes run the CUDA-core kernel with the reference
heuristic (``num_splits_herustic``, ``split_kv.py:247-276``, bit-exact through
``fa_split_kv_num_splits``) and its split size ``cdiv(cdiv(N, 128), S) * 128``
(``split_kv.py:313``).  The MLA shape (one kv head, 576-dim keys, v =
k[..., :512] sharing storage) runs on the MLA kernel.
"""

import ctypes
import math

import torch

from flagattention_b200 import _decode, _lib
from flagattention_b200._torch import dtype_code, require_cuda, sm_count, status_word, stream_of

BLOCK_M, BLOCK_N, MAX_SPLITS = 16, 128, 128


def _cdiv(a, b):
    return (a + b - 1) // b


def split_kv_num_splits(B, H, M, N, num_sms, block_m=BLOCK_M, block_n=BLOCK_N,
                        max_splits=MAX_SPLITS):
    out = ctypes.c_int32(0)
    _lib.check(_lib.lib().fa_split_kv_num_splits(B, H, M, N, block_m, block_n, num_sms,
                                                 max_splits, ctypes.byref(out)),
               "fa_split_kv_num_splits")
    return out.value


def _is_mla(k, v):
    return (k.shape[1] == 1 and k.shape[3] == 576 and v.shape[3] == 512
            and v.data_ptr() == k.data_ptr() and v.stride() == k.stride()
            and k.dtype in (torch.bfloat16, torch.float16))


def _mla_contiguous(q, k, causal, sm_scale):
    from flagattention_b200.mla import get_mla_metadata, mla_decode
    B, H, M, _ = q.shape
    N = k.shape[2]
    seq = torch.full((B,), N, dtype=torch.int32, device=q.device)
    meta, splits = get_mla_metadata(seq, M * H, 1)
    qm = q.transpose(1, 2)                                  # [B, M, H, 576]
    if M > 1 or qm.stride(-1) != 1:
        qm = qm.contiguous()
    out = torch.empty((B, H, M, 512), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, M), dtype=torch.float32, device=q.device)
    mla_decode(qm, k, k.stride(0), k.stride(2), B, 64, None, seq, N, meta, splits,
               out.transpose(1, 2), lse, sm_scale, causal)
    return out, lse


def _attention(q, k, v, causal, sm_scale):
    require_cuda(q, k, v)
    B, H, M, D = q.shape
    Hk, N = k.shape[1], k.shape[2]
    if k.shape[3] != D or v.shape[:3] != k.shape[:3]:
        raise _lib.InvalidArgument("q/k/v shapes disagree")
    if H % Hk != 0:
        raise _lib.InvalidArgument("number of heads in q must be a multiple of that in k & v")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if _is_mla(k, v) and N > 0:
        return _mla_contiguous(q, k, causal, sm_scale)
    q, k, v = (x if x.stride(-1) == 1 else x.contiguous() for x in (q, k, v))
    if k.stride() != v.stride():
        v = v.contiguous()
        k = k.contiguous()
    d_v = v.shape[3]

    def reference_splits():
        S = split_kv_num_splits(B, H, M, N, sm_count(q.device))
        # split_kv.py:313: N_SPLIT_SIZE = cdiv(cdiv(N, BLOCK_N), S) * BLOCK_N
        return S, (_cdiv(_cdiv(N, BLOCK_N), S) * BLOCK_N if S > 1 else 0)

    out = torch.empty((B, H, M, d_v), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, M), dtype=torch.float32, device=q.device)
    a = _lib.DecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_b, a.q_stride_h, a.q_stride_m = q.stride(0), q.stride(1), q.stride(2)
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.k_stride_seq, a.k_stride_head, a.k_stride_tok = k.stride(0), k.stride(1), k.stride(2)
    a.block_table = None
    a.seq_lens = None
    a.n_ctx = N
    a.batch, a.num_q_heads, a.num_kv_heads, a.m_q = B, H, Hk, M
    a.d_qk, a.d_v = D, d_v
    a.causal = int(bool(causal))
    a.dtype = dtype_code(q)
    a.scale = float(sm_scale)
    a.o = out.data_ptr()
    a.o_stride_b, a.o_stride_h, a.o_stride_m = out.stride(0), out.stride(1), out.stride(2)
    a.lse = lse.data_ptr()
    a.status = status_word(q.device).data_ptr()
    _decode.run(a, "fa_split_kv_attention", q.device, stream_of(q), 0, reference_splits)
    return out, lse


def flash_attention_split_kv(q, k, v, causal=False, sm_scale=None):
    """Drop-in for ``flag_attn.flash_attention_split_kv`` (split_kv.py:280)."""
    return _attention(q, k, v, causal, sm_scale)[0]


def flash_attention(q, k, v, causal=False, sm_scale=None, return_log_normalizer=False):
    """Forward of ``flag_attn.flash_attention`` (flash.py:269) for decode.

    With ``return_log_normalizer`` returns ``(o, L, None)`` like the
    reference's split-KV branch (flash.py:160-171); no autograd.
    """
    o, lse = _attention(q, k, v, causal, sm_scale)
    if return_log_normalizer:
        return o, lse, None
    return o
