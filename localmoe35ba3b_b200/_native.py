"""ctypes binding of ``liblocalmoe_b200.so`` (the C ABI in include/localmoe_b200.h).

The library is loaded from this package's directory.  There is no fallback:
if it is missing or lacks a symbol, ``lib()`` raises, and every operator
raises with it.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, 'liblocalmoe_b200.so')

BF16, F16 = 0, 1
ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED = -1, -2, -3
DEVERR_TIMEOUT = 1
DEVERR_BAD_EXPERT = 2
DEVERR_BAD_INDEX = 4
WIRE_DTYPE, WIRE_INT8 = 0, 1

_P, _I64, _I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

# name -> (restype, argtypes); must match include/localmoe_b200.h
SIGNATURES = {
    'lmoe_abi_version': (_I, []),
    'lmoe_quantize_rows': (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    'lmoe_linear_w8a16': (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _P]),
    'lmoe_linear_w8a16_workspace_size': (_I64, [_I64, _I64, _I64]),
    'lmoe_linear_w8a16_ws': (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _I64, _P, _P]),
    'lmoe_linear_w8a8_workspace_size': (_I64, [_I64, _I64]),
    'lmoe_linear_w8a8': (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _P, _P]),
    'lmoe_grouped_linear_w8a16': (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P]),
    'lmoe_grouped_linear_w8a8': (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _P]),
    'lmoe_ordered_reduce': (_I, [_P, _P, _P, _P, _I64, _I64, _I, _P]),
    'lmoe_plan_workspace_size': (_I64, [_I64, _I64, _I64]),
    'lmoe_plan': (_I, [_P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P]),
    'lmoe_route_meta_size': (_I64, [_I64, _I64, _I64]),
    'lmoe_route_meta': (_I, [_P, _P, _I64, _I64, _I64, _I, _P, _P]),
    'lmoe_routed_linear_workspace_size': (_I64, [_I64, _I64, _I64]),
    'lmoe_routed_linear': (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _I, _P, _I, _P, _P, _P]),
    'lmoe_routed_reduce': (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    'lmoe_moe_workspace_size': (_I64, [_I64, _I64, _I64, _I64, _I64]),
    'lmoe_routed_moe': (_I, [_P, _P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I64,
                             _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    'lmoe_routed_moe_noalloc_limit': (_I64, []),
    'lmoe_routed_moe_noalloc': (_I, [_P, _P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I64,
                                     _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P]),
    'lmoe_decode_workspace_size': (_I64, [_I64, _I64, _I64]),
    'lmoe_decode_moe': (_I, [_P, _P, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64,
                             _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P]),
    'lmoe_router_topk': (_I, [_P, _I64, _I64, _I64, _P, _P, _P, _I, _P]),
    'lmoe_selftest_silu': (_I, [_I, _P, _P]),
    'lmoe_router_gemm_workspace_size': (_I64, [_I64, _I64]),
    'lmoe_router_gemm_topk': (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I, _P, _P]),
    'lmoe_moe_block_router': (_I, [_P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _P, _P, _I, _P, _P, _P]),
    'lmoe_ep_layer_row_bytes': (_I64, [_I64, _I64, _I]),
    'lmoe_ep_plan_workspace_size': (_I64, [_I64, _I64, _I64, _I64]),
    'lmoe_ep_owner_workspace_size': (_I64, [_I64, _I64, _I64, _I64, _I64, _I64, _I64]),
    'lmoe_ep_dispatch': (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I, _I, _P, _P, _P, _P, _P]),
    'lmoe_ep_owner': (_I, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P,
                           _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    'lmoe_ep_fold': (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _P, _I, _P, _P,
                          _P]),
    'lmoe_ipc_get_handle': (_I, [_P, _P, _P]),
    'lmoe_ipc_open_handle': (_I, [_P, _I64, _P, _P]),
    'lmoe_ipc_close': (_I, [_P]),
}

class EpPeers(ctypes.Structure):
    """lmoe_ep_peers (include/localmoe_b200.h): every rank's exchange buffers and flag
    words as mapped into this process, this rank's counters, rank and layer epoch."""
    _fields_ = [('recv', _P * 8), ('back', _P * 8), ('flags', _P * 8), ('counter', _P), ('rank', _I),
                ('epoch', ctypes.c_uint)]


_lib = None


class NativeError(RuntimeError):
    pass


def lib():
    """The loaded library; raises if it is absent (no CPU or eager fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeError(f'{LIB_PATH} is missing: build it with `python -m localmoe35ba3b_b200.build` '
                              '(there is no fallback path)')
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError names the missing symbol
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        what = {ERR_INVALID: 'invalid geometry', ERR_CUDA: 'CUDA launch error',
                ERR_UNSUPPORTED: 'unsupported geometry'}.get(rc, f'error {rc}')
        raise NativeError(f'{name}: {what}')
    return rc


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt):
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise ValueError(f'unsupported activation dtype {dt}')


_err_words = {}


def error_word(device):
    """Per-device int32 error word that kernels OR their LMOE_DEVERR_* bits into."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f'cuda:{idx}')
        _err_words[idx] = w
    return w


def check_device_errors(device=None, reset=True):
    """Read (synchronously) and optionally clear the device error word."""
    w = error_word(device if device is not None else torch.device('cuda'))
    v = int(w.item())
    if reset and v:
        w.zero_()
    if v:
        raise NativeError(f'device-side error bits 0x{v:x} (1 = a bounded wait timed out, '
                          '2 = an expert id out of range, 4 = a row index out of range)')
    return 0


_workspaces = {}


def workspace(device, nbytes, tag='ws', zeroed=False):
    """A cached uint8 device buffer of at least nbytes (grown, never shrunk); with
    ``zeroed`` a (re)allocated buffer starts as zeros."""
    key = (str(device), tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        alloc = torch.zeros if zeroed else torch.empty
        buf = alloc(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf
