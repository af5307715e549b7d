"""CPU oracle for the paged / MLA decode path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of FlagAttention's PyTorch
reference (``src/flag_attn/testing/paged.py``, ``testing/flash.py``), its split
merge math (``split_kv.py:198-228``, ``paged.py:416-442``), its host split
heuristics (``paged.py:54-67``, ``split_kv.py:247-276``) and the MLA and
grouped-query schedule specifications the device code must reproduce
bit-exactly.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import it, and only as the checker or as the timed CPU baseline.  The
product (``flagattention_b200``) never imports it and has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (imported
from its source tree in the build container) and commits its outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks every function here
against those fixtures.
"""

from oracle.attention import (  # noqa: F401
    flash_attention,
    lse_combine,
    mla_append_rows,
    mla_decode_dense,
    mla_decode_sparse,
    paged_attention,
    paged_v2_reduce,
)
from oracle.sched import (  # noqa: F401
    gqa_schedule,
    mla_schedule,
    num_splits_heuristic,
    paged_num_splits,
)
