"""Loads libdrama3_b200.so (built in place by comfyui-drama3_b200/build.py) and declares its C ABI for ctypes.

There is no fallback: if the library is missing, or a call returns an error, the caller gets an exception.
"""
import ctypes
import functools
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdrama3_b200.so"

D3_OK, D3_ERR_ARG, D3_ERR_ALIGN, D3_ERR_CUDA, D3_ERR_DEVICE, D3_ERR_WORKSPACE, D3_ERR_TOO_LARGE = range(7)
FMT_FP8, FMT_INT8, FMT_W4, FMT_W6, FMT_FP8C, FMT_W4A8, FMT_W6A8 = range(7)
# the reference's layouts, then the BASELINE ones (per-channel fp8; W4A8 / W6A8 with int8 activations)
FORMATS = {"fp8": FMT_FP8, "int8": FMT_INT8, "w4": FMT_W4, "w6": FMT_W6, "fp8c": FMT_FP8C, "w4a8": FMT_W4A8,
           "w6a8": FMT_W6A8}
# field holding each format's weight rows
WEIGHT_KEY = {"fp8": "weight", "fp8c": "weight", "int8": "_qdata", "w4": "_qdata", "w6": "_qdata", "w4a8": "_qdata",
              "w6a8": "_qdata"}

_p = ctypes.c_void_p
_i = ctypes.c_int
_d = ctypes.c_double
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every name here is a symbol include/drama3_b200.h declares
SIGNATURES = {
    "d3_version": (_i, []),
    "d3_error_string": (ctypes.c_char_p, [_i]),
    "d3_last_cuda_error": (_i, []),
    "d3_device_check": (_i, []),
    "d3_take_fault": (_i, [ctypes.POINTER(ctypes.c_uint)]),
    "d3_route": (_i, [_p, _i, _i, _i, _p, _p, _p]),
    "d3_router": (_i, [_p, _i, _i, _p, _i, _i, _p, _p, _p, _p]),
    "d3_shared_expert": (_i, [_p, _i, _i, _p, _p, _p, _i, _p, _p, _p]),
    "d3_prefill_plan": (_i, [_p, _i, _i, _i, _p, _p, _p, _p]),
    "d3_weighted_sum": (_i, [_p, _p, _i, _i, _i, _p, _p]),
    "d3_rotate": (_i, [_p, _i, _i, _i, _p, _p, _p]),
    "d3_resolve": (_i, [_p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _d, _i, _d, _p]),
    "d3_gemv_fp8": (_i, [_p, _i, _p, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "d3_gemv_int8": (_i, [_p, _i, _p, _p, _p, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "d3_gemv_codes": (_i, [_p, _i, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _i, _i, _p]),
    "d3_grouped_fp8": (_i, [_p, _i, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "d3_grouped_int8": (_i, [_p, _i, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "d3_grouped_codes": (_i, [_p, _i, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _i, _i, _p]),
    "d3_grouped_mma_tile_rows": (_i, []),
    "d3_grouped_mma_workspace": (_sz, [_i, _i]),
    "d3_grouped_mma": (_i, [_i, _p, _i, _p, _i, _p, _i, _i, _p, _p, _p, _p, _i, _p, _i, _i, _p, _sz, _p]),
    "d3_prefill_combine": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _i, _p]),
    "d3_moe_decode_workspace": (_sz, [_i, _i, _i]),
    "d3_moe_decode": (_i, [_i, _p, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "d3_moe_decode_static": (_i, [_i, _p, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "d3_moe_decode_ep": (_i, [_i, _p, _i, _i, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                              _p, _sz, _p]),
    "d3_pack_fp8_blocks": (_i, [_p, ctypes.c_int64, _i, _p, _p, _i]),
    "d3_pack_int8_convrot": (_i, [_p, ctypes.c_int64, _i, _p, _p, _i]),
    "d3_pack_codes": (_i, [_p, ctypes.c_int64, _i, _i, _p, _p, _p, _p, _i]),
    "d3_pack_fp8c": (_i, [_p, ctypes.c_int64, _i, _p, _p, _i]),
    "d3_pack_wa8": (_i, [_p, ctypes.c_int64, _i, _i, _p, _p, _i]),
    "d3_ep_exchange_bytes": (_sz, [_i, _i, _i]),
    "d3_ep_reduce": (_i, [_p, _i, _i, _p, _p]),
    "d3_ipc_handle": (_i, [_p, _p, ctypes.POINTER(ctypes.c_size_t)]),
    "d3_ipc_open": (_i, [_p, _sz, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    "d3_ipc_close": (_i, [_p]),
}


class D3Error(RuntimeError):
    pass


@functools.cache
def lib():
    """The loaded library, with every signature declared. Raises if the library has not been built."""
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python comfyui-drama3_b200/build.py` "
                          "(there is no fallback implementation)")
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def check(status, what):
    """Raise D3Error for a non-zero status of call `what`."""
    if status != D3_OK:
        handle = lib()
        message = handle.d3_error_string(status).decode()
        if status == D3_ERR_CUDA:
            message += f" (cudaError {handle.d3_last_cuda_error()})"
        raise D3Error(f"{what}: {message}")


def take_fault():
    """Read and clear the current device's fault word (synchronizes)."""
    value = ctypes.c_uint(0)
    check(lib().d3_take_fault(ctypes.byref(value)), "d3_take_fault")
    return value.value
