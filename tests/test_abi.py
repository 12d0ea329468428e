"""C ABI checks that need no GPU: the library loads, exports every function
declared in include/ma_api.h, and rejects bad arguments on the host before
anything is launched."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
import monarch_attention_b200 as mab
from monarch_attention_b200 import _lib

HEADER = os.path.join(ROOT, "include", "ma_api.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(ma_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_expected_symbols():
    assert set(_lib.EXPORTED) <= set(declared_functions())


def test_library_exports_every_declared_symbol():
    lib = mab.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.ma_api_version() == 2


def good_params(**over):
    p = _lib.MaFwdParams()
    p.E, p.H, p.N, p.D, p.Dv = 2, 3, 100, 64, 64
    p.block_size, p.num_steps, p.pre_pad = 16, 2, 0
    p.dtype = p.out_dtype = _lib.DTYPE_BF16
    for k, v in over.items():
        setattr(p, k, v)
    return p


def test_workspace_bytes_covers_intermediates():
    lib = mab.load_library()
    p = good_params()
    n = lib.ma_workspace_bytes(ctypes.byref(p))
    M = (100 + 15) // 16
    heads = 2 * 3
    # al, y, ar (bf16) + cl, cr, lmax, lsum (fp32)
    assert n >= heads * M * 16 * (64 + 64 + 64) * 2 + heads * M * 16 * 4 * 4


@pytest.mark.parametrize("field,value,code", [
    ("E", 0, 2), ("N", 0, 2), ("D", -1, 2), ("block_size", 0, 2), ("num_steps", 0, 2),
    ("dtype", 9, 3), ("out_dtype", _lib.DTYPE_F32, 3), ("mask_dtype", 11, 5),
    ("impl", 5, 9),
])
def test_invalid_arguments_rejected_before_launch(field, value, code):
    lib = mab.load_library()
    p = good_params(**{field: value})
    assert lib.ma_fwd(ctypes.byref(p), None) == code
    assert lib.ma_workspace_bytes(ctypes.byref(p)) == 0
    assert lib.ma_last_error_detail()


def test_struct_size_guard():
    lib = mab.load_library()
    p = good_params()
    p.struct_size = 8
    assert lib.ma_fwd(ctypes.byref(p), None) == 9


def test_null_pointers_and_workspace_checked():
    lib = mab.load_library()
    p = good_params()
    assert lib.ma_fwd(ctypes.byref(p), None) == 1  # q/k/v/out NULL
    p.q = p.k = p.v = p.out = 0x1000  # never dereferenced: rejected earlier
    p.status = 0x2000
    assert lib.ma_fwd(ctypes.byref(p), None) == 6  # no workspace
    p.mask_dtype = _lib.MASK_BOOL
    assert lib.ma_fwd(ctypes.byref(p), None) == 5  # mask dtype but NULL mask


def test_fault_injection(monkeypatch):
    lib = mab.load_library()
    monkeypatch.setenv("MA_FAULT_INJECT", "1")
    assert lib.ma_fwd(ctypes.byref(good_params()), None) == _lib.MA_ERR_INJECTED
    with pytest.raises(_lib.MonarchAttentionError) as ei:
        _lib.check(_lib.MA_ERR_INJECTED)
    assert "injected" in str(ei.value)


def test_error_strings():
    lib = mab.load_library()
    for code in (0, 1, 2, 3, 4, 5, 6, 7, 8, 9, -1, -2):
        assert lib.ma_error_string(code)


def test_impl_selection_is_host_only():
    lib = mab.load_library()
    p = good_params()
    assert lib.ma_select_impl(ctypes.byref(p)) == _lib.IMPL_GENERIC
    p.impl = _lib.IMPL_GENERIC
    assert lib.ma_select_impl(ctypes.byref(p)) == _lib.IMPL_GENERIC


def test_noalloc_entry_rejects_on_the_host():
    """ma_fwd_noalloc refuses shapes outside the tcgen05 kernel before any
    CUDA call (no GPU needed)."""
    lib = mab.load_library()
    fn = lib.ma_fwd_noalloc
    fn.argtypes = [ctypes.POINTER(_lib.MaFwdParams), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    p = good_params()  # block size 16: generic shapes only
    assert fn(ctypes.byref(p), None) == 7
    assert b"tcgen05" in lib.ma_last_error_detail()
    p = good_params(E=0)
    assert fn(ctypes.byref(p), None) == 2


def tc_params(E=4, H=16, N=16384, b=128, T=2, D=128):
    p = good_params(E=E, H=H, N=N, D=D, Dv=D, block_size=b, num_steps=T)
    strides = (H * N * D, N * D, D, 1)
    for name in ("q_stride", "k_stride", "v_stride", "o_stride"):
        arr = getattr(p, name)
        for i, s in enumerate(strides):
            arr[i] = s
    return p


@pytest.mark.parametrize("E,H,N,b,T", [(4, 16, 16384, 128, 2), (4, 16, 4096, 64, 2),
                                       (1, 3, 16384, 128, 3), (1, 8, 16384, 128, 2)])
def test_tc_workspace_holds_only_the_cycled_slots(E, H, N, b, T):
    """The persistent tcgen05 kernel cycles through at most 2 x (2T+1) head
    slots of al / y / ar / cl / cr (hgroup heads per wavefront phase: 2 at
    b = 128, 8 at b = 64 -> capped by the head count), not all E*H heads."""
    lib = mab.load_library()
    p = tc_params(E, H, N, b, T)
    assert lib.ma_select_impl(ctypes.byref(p)) == _lib.IMPL_TC
    n = lib.ma_workspace_bytes(ctypes.byref(p))
    M = N // b
    per_head = b * M * (128 * 3 * 2 + 4 + 4 + 16)
    hgroup = 2 if b == 128 else 8
    slots = min(E * H, hgroup * (2 * T + 1))
    ctrl = 4 * (64 + E * H * 2 * T) + 4096
    assert n <= slots * per_head + ctrl
    assert n >= slots * b * M * 128 * 3 * 2
    if b == 128 and E * H > slots:
        assert n < E * H * per_head / 3  # ~0.85 GB before, ~125 MB now
