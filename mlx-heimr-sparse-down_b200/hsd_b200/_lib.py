"""ctypes binding of libhsd.so (the C ABI declared in include/hsd.h).

The library is loaded from this package's directory; there is no fallback. Every wrapped
call raises RuntimeError with the library's own message when the status is not HSD_OK.
"""
import ctypes
import os

import torch

HSD_OK, HSD_ERR_SHAPE, HSD_ERR_ALIGN, HSD_ERR_DTYPE, HSD_ERR_CUDA = 0, 1, 2, 3, 4
HSD_ERR_TIMEOUT, HSD_ERR_NCCL, HSD_ERR_ARG, HSD_ERR_INDEX = 5, 6, 7, 8
STATUS_NAMES = {0: "HSD_OK", 1: "HSD_ERR_SHAPE", 2: "HSD_ERR_ALIGN", 3: "HSD_ERR_DTYPE",
                4: "HSD_ERR_CUDA", 5: "HSD_ERR_TIMEOUT", 6: "HSD_ERR_NCCL", 7: "HSD_ERR_ARG",
                8: "HSD_ERR_INDEX"}

HSD_F32, HSD_F16, HSD_BF16 = 0, 1, 2
DTYPE_CODE = {torch.float32: HSD_F32, torch.float16: HSD_F16, torch.bfloat16: HSD_BF16}

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhsd.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64

# name -> argtypes, in the order of include/hsd.h
SIGNATURES = {
    "hsd_last_error_string": [],
    "hsd_abi_version": [],
    "hsd_device_status": [_P, _P],
    "hsd_nibble_transpose": [_P, _P, _L, _L, _L, _P],
    "hsd_swap_last2_u16": [_P, _P, _L, _L, _L, _P],
    "hsd_sparse_down_decode": [_P, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I,
                               _I, _I, _I, _I, _I, _I, _I, _P],
    "hsd_dense_down_decode_nm": [_P, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I,
                                 _I, _I, _I, _I, _I, _I, _P],
    "hsd_decode_live_rows": [_P, _I, _P, _P, _I, _I, _I, _I, _P],
    "hsd_prefill_num_tiles": [_I, _I, _I, _I, _P, _P],
    "hsd_prefill_build_tiles": [_P, _I, _I, _I, _I, _P, _P, _P],
    "hsd_prefill_build_union": [_P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P],
    "hsd_prefill_workspace_bytes": [_I, _I, _I, _I, _I, _I, _P],
    "hsd_sparse_down_prefill": [_P, _I, _P, _P, _P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I,
                                _I, _I, _I, _I, _I, _I, _P, ctypes.c_size_t, _P],
    "hsd_mamba_conv_verify": [_P, _I, _L, _P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _P],
    "hsd_mamba_ssm_verify": [_P, _I, _L, _P, _I, _L, _P, _P, _P, ctypes.c_float, ctypes.c_float, _P, _P, _P,
                             _I, _I, _I, _I, _I, _I, _I, _P],
    "hsd_mamba_rollback": [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P],
    "hsd_mamba_conv_step": [_P, _I, _L, _P, _P, _I, _P, _I, _P, _P, _I, _I, _I, _I, _P],
    "hsd_mamba_ssm_step": [_P, _I, _L, _P, _I, _L, _P, _P, _P, ctypes.c_float, ctypes.c_float, _P, _P, _I, _P,
                           _I, _I, _I, _I, _I, _I, _P],
    "hsd_moe_up_decode": [_P, _I, _L, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
    "hsd_qlinear_decode": [_P, _I, _L, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P],
    "hsd_rms_norm": [_P, _I, _L, _P, _I, _P, _I, _I, _I, ctypes.c_float, _P],
    "hsd_gated_rms_norm": [_P, _I, _L, _P, _I, _L, _P, _I, _P, _I, _I, _I, _I, ctypes.c_float, _P],
    "hsd_router_topk": [_P, _I, _L, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P],
    "hsd_attn_decode_workspace_bytes": [_I, _I, _I, _P],
    "hsd_attn_decode": [_P, _L, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _P],
    "hsd_dense_down_decode": [_P, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I,
                              _I, _P],
    "hsd_prefill_noalloc_max_bytes": [_P],
    "hsd_sparse_down_prefill_noalloc": [_P, _I, _P, _P, _P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I,
                                        _I, _I, _I, _I, _I, _I, _P],
    "hsd_ep_buffer_bytes": [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P],
    "hsd_ep_alloc": [ctypes.c_size_t, _P],
    "hsd_ep_free": [_P],
    "hsd_ep_ipc_handle": [_P, _P],
    "hsd_ep_ipc_open": [_P, _P],
    "hsd_ep_ipc_close": [_P],
    "hsd_ep_set_peers": [_P, _P, _I, _P],
    "hsd_ep_dispatch": [_P, _I, _I, _I, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _P, ctypes.c_double, _P],
    "hsd_ep_expert": [_P, _P, _I, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                      ctypes.c_double, _P],
    "hsd_ep_combine": [_P, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, ctypes.c_double, _P],
}

_lib = None


class HsdError(RuntimeError):
    """A libhsd call returned a status other than HSD_OK."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def lib():
    """The loaded library (raises when libhsd.so has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libhsd.so is not built ({LIB_PATH}); run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = ctypes.c_char_p if name == "hsd_last_error_string" else ctypes.c_int
        _lib = L
    return _lib


def call(name, *args):
    """Call a libhsd entry point; raise HsdError on a failed status."""
    rc = getattr(lib(), name)(*args)
    if rc != HSD_OK:
        msg = lib().hsd_last_error_string().decode("utf-8", "replace")
        raise HsdError(rc, msg)
    return rc


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t=None):
    """The current torch stream of t's device, as the C ABI's void* stream."""
    dev = t.device if t is not None else torch.device("cuda", torch.cuda.current_device())
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def dtype_code(t, what):
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: unsupported dtype {t.dtype}") from None


def require_cuda(*ts, what):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what}: every tensor must be on a CUDA device (got {t.device})")
        if t is not None and not t.is_contiguous():
            raise ValueError(f"{what}: tensors must be contiguous")


def device_status(t=None):
    """Read and clear the device status word (HSD_OK when no device-side error was met)."""
    out = ctypes.c_int(0)
    call("hsd_device_status", ctypes.byref(out), stream_of(t))
    return out.value
