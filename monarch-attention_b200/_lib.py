"""ctypes binding of the C ABI in include/ma_api.h (libmonarch_attn.so).

The library is built in-tree by ``build.py``; loading fails loudly when it is
missing -- there is no CPU or PyTorch fallback for the forward pass.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libmonarch_attn.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

# ma_dtype_t
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_E4M3 = 0, 1, 2, 3
# ma_mask_dtype_t
MASK_NONE, MASK_BOOL, MASK_I32, MASK_I64, MASK_F32, MASK_F16, MASK_BF16 = range(7)
# ma_impl_t
IMPL_AUTO, IMPL_GENERIC, IMPL_TC, IMPL_SMALL = 0, 1, 2, 3
IMPL_NAMES = {IMPL_GENERIC: "generic", IMPL_TC: "tc", IMPL_SMALL: "small"}

MA_OK = 0
MA_ERR_INJECTED = 8
MA_ERR_BAD_PARAMS = 9
MA_ERR_DEVICE = -2
MA_STATUS_WAIT_TIMEOUT = 0x1
MA_STATUS_TMEM_FAIL = 0x2
MA_STATUS_BAD_ITEM = 0x4

EXPORTED = (
    "ma_workspace_bytes",
    "ma_fwd",
    "ma_select_impl",
    "ma_error_string",
    "ma_last_error_detail",
    "ma_read_status",
    "ma_last_launch_count",
    "ma_api_version",
    "ma_bwd_workspace_bytes",
    "ma_bwd",
)

_i64x4 = ctypes.c_int64 * 4


class MaFwdParams(ctypes.Structure):
    """Mirror of ``ma_fwd_params`` (include/ma_api.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("q_stride", _i64x4),
        ("k_stride", _i64x4),
        ("v_stride", _i64x4),
        ("o_stride", _i64x4),
        ("mask", ctypes.c_void_p),
        ("mask_stride", ctypes.c_int64 * 2),
        ("mask_dtype", ctypes.c_int32),
        ("E", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("Dv", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_steps", ctypes.c_int32),
        ("pre_pad", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("q_scale", ctypes.c_void_p),
        ("k_scale", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
        ("impl", ctypes.c_int32),
        ("v_f32", ctypes.c_int32),
        ("status_host", ctypes.c_void_p),
        ("reserved", ctypes.c_int32 * 4),
    ]

    def __init__(self, **kw):
        super().__init__(**kw)
        self.struct_size = ctypes.sizeof(MaFwdParams)


class MaBwdParams(ctypes.Structure):
    """Mirror of ``ma_bwd_params`` (include/ma_api.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("fwd", MaFwdParams),
        ("dout", ctypes.c_void_p),
        ("dout_stride", _i64x4),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("dq_stride", _i64x4),
        ("dk_stride", _i64x4),
        ("dv_stride", _i64x4),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("reserved", ctypes.c_int32 * 8),
    ]

    def __init__(self, **kw):
        super().__init__(**kw)
        self.struct_size = ctypes.sizeof(MaBwdParams)
        self.fwd.struct_size = ctypes.sizeof(MaFwdParams)


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load libmonarch_attn.so (once); raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_NAME} is not built (expected at {LIB_PATH}); run "
                "`python -c 'import __graft_entry__ as g; g.build()'` from the repository root")
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER(MaFwdParams)
        lib.ma_workspace_bytes.argtypes = [P]
        lib.ma_workspace_bytes.restype = ctypes.c_size_t
        lib.ma_fwd.argtypes = [P, ctypes.c_void_p]
        lib.ma_fwd.restype = ctypes.c_int
        lib.ma_select_impl.argtypes = [P]
        lib.ma_select_impl.restype = ctypes.c_int
        lib.ma_error_string.argtypes = [ctypes.c_int]
        lib.ma_error_string.restype = ctypes.c_char_p
        lib.ma_last_error_detail.argtypes = []
        lib.ma_last_error_detail.restype = ctypes.c_char_p
        lib.ma_read_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.POINTER(ctypes.c_uint32)]
        lib.ma_read_status.restype = ctypes.c_int
        lib.ma_last_launch_count.argtypes = []
        lib.ma_last_launch_count.restype = ctypes.c_int
        lib.ma_api_version.argtypes = []
        lib.ma_api_version.restype = ctypes.c_int
        PB = ctypes.POINTER(MaBwdParams)
        lib.ma_bwd_workspace_bytes.argtypes = [PB]
        lib.ma_bwd_workspace_bytes.restype = ctypes.c_size_t
        lib.ma_bwd.argtypes = [PB, ctypes.c_void_p]
        lib.ma_bwd.restype = ctypes.c_int
        _lib = lib
        return lib


class MonarchAttentionError(RuntimeError):
    """Raised when the C ABI rejects a call or the device reports a failure."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(rc: int) -> None:
    if rc != MA_OK:
        lib = load()
        msg = lib.ma_error_string(rc).decode()
        detail = lib.ma_last_error_detail().decode()
        raise MonarchAttentionError(rc, f"monarch attention: {msg} (code {rc})"
                                        + (f": {detail}" if detail else ""))
