"""Dispatch of a prepared ``fa_decode_args`` to the library (shared by
``paged_attention`` and ``flash_attention_split_kv``).

The library picks the kernel: the tensor-core kernel for the shapes it
serves (``fa_decode_uses_tensor_cores``), the CUDA-core kernel otherwise.
With the tensor-core kernel and an automatic split count the work is cut by
the device scheduler (every SM gets the same number of key blocks); an
explicit split count, and the CUDA-core kernel, use the reference's fixed
partitions (``reference_splits``).
"""

import ctypes

import torch

from flagattention_b200 import _lib


def uses_tensor_cores(a):
    return _lib.lib().fa_decode_uses_tensor_cores(ctypes.byref(a)) == 1


def workspace_bytes(a):
    """(part_o, part_lse, sched) bytes, or None when the library refuses the
    arguments (num_splits == 0 outside the tensor-core kernel)."""
    po, pl, sc = ctypes.c_size_t(0), ctypes.c_size_t(0), ctypes.c_size_t(0)
    st = _lib.lib().fa_decode_workspace_size(ctypes.byref(a), ctypes.byref(po), ctypes.byref(pl),
                                             ctypes.byref(sc))
    return (po.value, pl.value, sc.value) if st == _lib.FA_OK else None


def attach_workspace(a, sizes, device):
    """Allocate the split scratch and point the arguments at it; returns the
    owning tensor (None when nothing is split)."""
    po, pl, sc = sizes
    if po + pl + sc == 0:
        return None
    buf = torch.empty(po + pl + sc, dtype=torch.uint8, device=device)
    base = buf.data_ptr()
    a.part_o = base
    a.part_lse = base + po
    a.sched = base + po + pl if sc else None
    return buf


def run(a, entry, device, stream, requested_splits, reference_splits):
    """Launch entry point ``entry`` (fa_paged_attention / fa_split_kv_attention).

    requested_splits: the caller's split count (0 = automatic).
    reference_splits(): (num_splits, partition_size) of the reference's rule,
    used unless the tensor-core kernel balances the work itself.
    """
    sizes = None
    if requested_splits == 0:
        # the balanced schedule; refused (sizes None) unless the arguments
        # run on the tensor-core kernel
        a.num_splits, a.partition_size = 0, 0
        sizes = workspace_bytes(a)
    if sizes is None:
        a.num_splits, a.partition_size = reference_splits()
        sizes = workspace_bytes(a)
        if sizes is None:
            _lib.check(_lib.FA_ERR_INVALID_ARGUMENT, "fa_decode_workspace_size")
    buf = attach_workspace(a, sizes, device)
    _lib.check(getattr(_lib.lib(), entry)(ctypes.byref(a), stream), entry)
    return buf
