"""torch helpers shared by the operator modules (device memory, streams)."""

import ctypes

import torch

from flagattention_b200 import _lib

_DTYPES = {torch.bfloat16: _lib.FA_DTYPE_BF16, torch.float16: _lib.FA_DTYPE_F16,
           torch.float32: _lib.FA_DTYPE_F32}


def dtype_code(t):
    try:
        return _DTYPES[t.dtype]
    except KeyError as e:
        raise _lib.InvalidArgument(f"unsupported dtype {t.dtype}") from e


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise _lib.InvalidArgument("flagattention_b200 operators take CUDA tensors only "
                                       "(there is no CPU path)")


def sm_count(device):
    n = ctypes.c_int32(0)
    _lib.check(_lib.lib().fa_device_sm_count(device.index if device.index is not None
                                             else torch.cuda.current_device(), ctypes.byref(n)),
               "fa_device_sm_count")
    return n.value


_status = {}


def status_word(device):
    """Per-device int32 the kernels set when a bounded wait gives up."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status[key] = t
    return t


def read_status(device):
    """Synchronise and return (then clear) the device status word (0 = ok)."""
    t = status_word(device)
    v = int(t.item())
    if v:
        t.zero_()
    return v
