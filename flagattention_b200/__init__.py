"""flagattention_b200 -- B200 (sm_100a) decode engine for FlagAttention's paged /
split-KV decode path and the MLA (latent attention) decode path.

Public operators (no CPU path: every call runs CUDA kernels of the in-tree
``libflagattn_b200.so`` and raises if that library is missing):

* ``paged_attention``            -- flag_attn.paged_attention drop-in
* ``flash_attention_split_kv``   -- flag_attn.flash_attention_split_kv drop-in
* ``flash_attention``            -- forward / LSE of flag_attn.flash_attention
* ``get_mla_metadata``, ``flash_mla_with_kvcache`` -- MLA metadata + decode
* ``shard``                      -- multi-GPU sharding (sequence / KV pages)
"""

from flagattention_b200._lib import CudaError, InvalidArgument, Unsupported  # noqa: F401
from flagattention_b200.mla import append_kv_rows, flash_mla_with_kvcache, get_mla_metadata  # noqa: F401
from flagattention_b200.paged import paged_attention  # noqa: F401
from flagattention_b200.split_kv import flash_attention, flash_attention_split_kv  # noqa: F401

__version__ = "0.1.0"
