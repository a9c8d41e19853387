"""ctypes binding of libqlin.so (the C ABI in include/qlin.h).

The library is built in-tree by mac-kernels-public_b200/build.py.  There is no fallback: if the
shared library is missing or fails to load, importing this module raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# QLIN_LIB selects another build of the same library (e.g. one compiled with different flags).
LIB_PATH = os.environ.get("QLIN_LIB") or os.path.join(_HERE, "libqlin.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python mac-kernels-public_b200/build.py`")

lib = ctypes.CDLL(LIB_PATH)

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t

# name -> (restype, argtypes); keep in the order of include/qlin.h
SIGNATURES = {
    "qlin_version": (ctypes.c_char_p, []),
    "qlin_last_error": (ctypes.c_char_p, []),
    "qlin_device_status": (_i, [_i, ctypes.POINTER(ctypes.c_uint32)]),
    "qlin_bounds_check": (_i, [_i, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                               ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint32)]),
    "qlin_int8_linear_workspace": (_sz, [_i64, _i64, _i64]),
    "qlin_int8_linear": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _i, _p, _i, _i, _p, _i, _i64, _p, _sz, _p]),
    "qlin_int8_linear_lora_workspace": (_sz, [_i64, _i64, _i64, _i64]),
    "qlin_int8_linear_lora": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _i, _p, _i, _i, _p, _i, _i64, _p, _i, _i64,
                                   _i64, ctypes.c_float, _p, _i, _i64, _p, _sz, _p]),
    "qlin_int8_linear_lora_down_workspace": (_sz, [_i64, _i64, _i64, _i64]),
    "qlin_int8_linear_lora_down": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _i, _p, _i, _i, _p, _i, _i64, _p, _i,
                                        _i64, _i64, ctypes.c_float, _p, _i, _i64, _p, _sz, _p]),
    "qlin_int8_grad_weight_bytes": (_sz, [_i64, _i64]),
    "qlin_int8_grad_weight": (_i, [_p, _i64, _i64, _p, _sz, _p]),
    "qlin_int8_linear_grad_input_workspace": (_sz, [_i64, _i64, _i64, _i]),
    "qlin_int8_linear_grad_input": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _i, _i, _p, _i, _i64, _p, _sz, _p]),
    "qlin_gguf_repacked_bytes": (_i, [_i, _i64, _i64, ctypes.POINTER(_sz), ctypes.POINTER(_i64)]),
    "qlin_gguf_repack": (_i, [_p, _i, _i64, _i64, _p, _sz, _p, _i64, _p]),
    "qlin_gguf_linear_workspace": (_sz, [_i64, _i64, _i64, _i, _i64]),
    "qlin_gguf_linear": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _i, _p, _i, _i64, _p, _sz, _p]),
    "qlin_gguf_linear_lora_workspace": (_sz, [_i64, _i64, _i64, _i, _i64, _i64]),
    "qlin_gguf_linear_lora": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _i, _p, _i, _i64, _p, _i, _i64,
                                   _i64, ctypes.c_float, _p, _i, _i64, _p, _sz, _p]),
    "qlin_gguf_linear_lora_down_workspace": (_sz, [_i64, _i64, _i64, _i, _i64, _i64]),
    "qlin_gguf_linear_lora_down": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _i, _p, _i, _i64, _p, _i, _i64,
                                        _i64, ctypes.c_float, _p, _i, _i64, _p, _sz, _p]),
    "qlin_gguf_linear_slabs": (_i, [_p, _i64, _i64, _i64, _i, _i64, _p, _p, _i, _i64, _p, _i, _p, _i, _i64, _p, _sz,
                                    _p]),
    "qlin_gguf_linear_allgather": (_i, [_p, _i64, _i64, _i64, _i, _i64, _p, _p, _i, _i64, _p, _i, _i, _i,
                                        ctypes.POINTER(_p), _i, _i64, ctypes.POINTER(_p), ctypes.c_uint32, _p, _sz,
                                        _p]),
    "qlin_peer_sync_bytes": (_sz, []),
    "qlin_peer_alloc": (_i, [_sz, ctypes.POINTER(_p)]),
    "qlin_peer_free": (_i, [_p]),
    "qlin_peer_export": (_i, [_p, _p]),
    "qlin_peer_import": (_i, [_p, ctypes.POINTER(_p)]),
    "qlin_peer_close": (_i, [_p]),
    "qlin_peer_wait": (_i, [_i, _i, ctypes.POINTER(_p), ctypes.c_uint32, _p]),
    "qlin_gguf_linear_noalloc": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _i, _p, _i, _i64, _p]),
    "qlin_gguf_dequantize": (_i, [_p, _i, _i64, _i64, _p, _i, _p]),
    "qlin_kitchen_w4a8_grid": (_i, [_p, _i, _p, _p, _i, _i64, _i64, _p, _p]),
    "qlin_prologue_f16": (_i, [_p, _i, _i64, _i64, _i64, _i, _p, _i64, _p, _p]),
    "qlin_quantize_rows_int8": (_i, [_p, _i, _i64, _i64, _i64, _i, _i, _p, _i64, _p, _p]),
    "qlin_w4a8_repacked_bytes": (_i, [_i, _i, _i64, _i64, ctypes.POINTER(_sz)]),
    "qlin_w4a8_repack": (_i, [_p, _i, _i, _i64, _i64, _p, _sz, _p]),
    "qlin_w4a8_linear_workspace": (_sz, [_i64, _i64, _i64, _i]),
    "qlin_w4a8_linear": (_i, [_p, _i, _i64, _i64, _i64, _p, _i, _i, _i64, _p, _i, _i, _p, _i, _p, _i, _i64, _p, _sz,
                              _p]),
}

for _name, (_res, _args) in SIGNATURES.items():
    if hasattr(lib, _name):
        _fn = getattr(lib, _name)
        _fn.restype = _res
        _fn.argtypes = _args

STATUS = {0: "QLIN_OK", 1: "QLIN_EDECLINE", 2: "QLIN_EINVAL", 3: "QLIN_ECUDA", 4: "QLIN_ETIMEOUT"}
DTYPE_CODE = {"float32": 0, "float16": 1, "bfloat16": 2, "int8": 3, "uint8": 4, "int32": 5, "float8_e4m3fn": 6}


class QlinError(RuntimeError):
    def __init__(self, code, where):
        msg = lib.qlin_last_error().decode(errors="replace")
        super().__init__(f"{where}: {STATUS.get(code, code)}: {msg}")
        self.code = code


class QlinDecline(QlinError, NotImplementedError):
    """Unsupported input for the fast path (QLIN_EDECLINE); the caller takes the stock path."""


def check(code, where):
    if code == 0:
        return
    if code == 1:
        raise QlinDecline(code, where)
    raise QlinError(code, where)


def exported_symbols():
    return [n for n in SIGNATURES if hasattr(lib, n)]
