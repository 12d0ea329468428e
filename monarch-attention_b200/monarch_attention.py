"""MonarchAttention operator surface backed by the sm_100a CUDA library.

Drop-in for the reference module ``ma/monarch_attention.py`` of
djmmoss/monarch-attention:

  * ``PadType``                       <- ma/monarch_attention.py:12-14
  * ``MonarchAttention(block_size, num_steps, pad_type, impl=None)``
                                      <- ma/monarch_attention.py:17-37
  * ``MonarchAttention.forward(query, key, value, attention_mask=None)``
                                      <- ma/monarch_attention.py:39-58
  * ``MonarchAttention.get_matrix(query, key, attention_mask=None)``
                                      <- ma/monarch_attention.py:60-70
  * ``monarch_attention(q, k, v, attn_mask, T, B, pre_pad)``
                                      <- ma/ma_torch.py:65-73

The ViT / RoBERTa / BART / DiT hooks call ``attn_module(q, k, v[, mask])`` with
(E, H, N, D) views of arbitrary strides (vit/model.py:97,
roberta/model.py:104-106, bart/model.py:150-152,
dit/attention_processor.py:143); those calls work unchanged.  The work runs
on the current CUDA stream through ``ma_fwd`` (include/ma_api.h).  Tensors on
any other device raise: there is no CPU path.  With inputs that require
gradients (training, e.g. the BART fine-tuning of the reference) the forward
runs on the forward kernels and the backward on the backward kernels
(``ma_bwd``, ``training.py``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from enum import StrEnum

import torch
import torch.nn as nn

from . import _lib, training

Tensor = torch.Tensor

_TORCH_TO_MA = {
    torch.float32: _lib.DTYPE_F32,
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float8_e4m3fn: _lib.DTYPE_E4M3,
}
_MASK_DTYPES = {
    torch.bool: _lib.MASK_BOOL,
    torch.uint8: _lib.MASK_BOOL,
    torch.int8: _lib.MASK_BOOL,
    torch.int32: _lib.MASK_I32,
    torch.int64: _lib.MASK_I64,
    torch.float32: _lib.MASK_F32,
    torch.float16: _lib.MASK_F16,
    torch.bfloat16: _lib.MASK_BF16,
}
_IMPL_ARG = {
    None: _lib.IMPL_AUTO,
    "auto": _lib.IMPL_AUTO,
    # the reference's own names: both are replaced by the B200 kernels
    "torch": _lib.IMPL_AUTO,
    "triton": _lib.IMPL_AUTO,
    "generic": _lib.IMPL_GENERIC,
    "tc": _lib.IMPL_TC,
    "small": _lib.IMPL_SMALL,
}


class PadType(StrEnum):
    pre = "pre"
    post = "post"


_status_lock = threading.Lock()
_status_words: dict[int, Tensor] = {}
_status_mirrors: dict[int, Tensor] = {}

# bits of the device status word (include/ma_api.h)
_STATUS_NAMES = {_lib.MA_STATUS_WAIT_TIMEOUT: "a bounded device wait ran out",
                 _lib.MA_STATUS_TMEM_FAIL: "tensor-memory allocation failed",
                 _lib.MA_STATUS_BAD_ITEM: "the scheduler produced an out-of-range item"}


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def status_word(device: torch.device) -> Tensor:
    """Per-device int32 word into which kernels OR failure bits (MA_STATUS_*)."""
    idx = _dev_index(device)
    with _status_lock:
        w = _status_words.get(idx)
        if w is None:
            w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _status_words[idx] = w
        return w


_mirror_refused: set[int] = set()


def _status_mirror(device: torch.device) -> Tensor:
    """Per-device page-locked host word a failing kernel also writes (the
    ``status_host`` field of ma_fwd_params): the host learns of a failure
    without reading device memory."""
    idx = _dev_index(device)
    with _status_lock:
        h = _status_mirrors.get(idx)
        if h is None:
            h = torch.zeros(1, dtype=torch.int32).pin_memory()
            _status_mirrors[idx] = h
        return h


def _mirror_ptr(device: torch.device) -> int:
    """Address of the host mirror, or 0 where the library refused it (pinned
    memory that is not mapped into the device's address space); failures are
    then found by check_status() / check=True only."""
    if _dev_index(device) in _mirror_refused:
        return 0
    return _status_mirror(device).data_ptr()


def read_status(device: torch.device | None = None, reset: bool = True) -> int:
    """Synchronously read (and by default clear) the device status word."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    w = status_word(device)
    val = int(w.item())
    if reset:
        if val:
            w.zero_()
        _status_mirror(device).zero_()
    return val


def _raise_device_failure(device: torch.device, bits: int) -> None:
    what = "; ".join(n for b, n in _STATUS_NAMES.items() if bits & b) or f"bits {bits:#x}"
    raise _lib.MonarchAttentionError(
        _lib.MA_ERR_DEVICE,
        f"monarch attention: a kernel on {device} reported a device-side failure ({what}, "
        f"status {bits:#x}); the output of that call is not valid")


def check_status(device: torch.device | None = None) -> None:
    """Wait for the device, then raise MonarchAttentionError (code
    MA_ERR_DEVICE) if a kernel on it reported a failure since the last check;
    the status is cleared either way."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    torch.cuda.synchronize(device)
    bits = read_status(device)
    if bits:
        _raise_device_failure(device, bits)


def _check_previous(device: torch.device) -> None:
    """Lazy check at the start of every call: a failure of an earlier call on
    this device shows in the host mirror (a host read, no synchronisation)."""
    if _dev_index(device) in _mirror_refused:
        return
    h = _status_mirror(device)
    if int(h[0]) != 0:
        torch.cuda.synchronize(device)
        bits = read_status(device) or int(h[0])
        h.zero_()
        _raise_device_failure(device, bits)


def _impl_code(impl) -> int:
    env = os.environ.get("MA_IMPL")
    if env:
        impl = env
    if impl not in _IMPL_ARG:
        raise ValueError(f"impl must be one of {sorted(k for k in _IMPL_ARG if k)}; got {impl!r}")
    return _IMPL_ARG[impl]


def _mask_arg(attn_mask: Tensor | None, E: int, N: int, device) -> tuple:
    if attn_mask is None:
        return None, (0, 0), _lib.MASK_NONE, None
    if attn_mask.shape != (E, N):
        raise ValueError(f"attention_mask must have shape (E, N) = {(E, N)}; "
                         f"got {tuple(attn_mask.shape)}")
    if attn_mask.device != device:
        raise ValueError("attention_mask must be on the same device as the inputs")
    keep = attn_mask
    code = _MASK_DTYPES.get(attn_mask.dtype)
    if code is None:  # any other dtype: nonzero = valid
        keep = attn_mask != 0
        code = _lib.MASK_BOOL
    return keep.data_ptr(), tuple(keep.stride()), code, keep


def build_params(q: Tensor, k: Tensor, v: Tensor, out: Tensor, attn_mask: Tensor | None,
                 T: int, B: int, pre_pad: bool, impl: int = _lib.IMPL_AUTO,
                 scales: tuple | None = None) -> tuple[_lib.MaFwdParams, list]:
    """Fill an ``ma_fwd_params`` block; returns it and the tensors it points into."""
    E, H, N, D = q.shape
    Dv = v.shape[-1]
    mptr, mstride, mcode, mkeep = _mask_arg(attn_mask, E, N, q.device)
    p = _lib.MaFwdParams()
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    for name, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", out)):
        arr = getattr(p, name)
        for i, s in enumerate(t.stride()):
            arr[i] = s
    p.mask = mptr
    p.mask_stride[0], p.mask_stride[1] = mstride
    p.mask_dtype = mcode
    p.E, p.H, p.N, p.D, p.Dv = E, H, N, D, Dv
    p.block_size, p.num_steps, p.pre_pad = int(B), int(T), int(bool(pre_pad))
    p.dtype = _TORCH_TO_MA[q.dtype]
    p.out_dtype = _TORCH_TO_MA[out.dtype]
    # fp32 values with 16-bit q / k (the reference's get_matrix)
    p.v_f32 = int(v.dtype == torch.float32 and q.dtype in (torch.float16, torch.bfloat16))
    keep = [q, k, v, out, mkeep]
    if scales is not None:
        qs, ks, vs = (s.to(device=q.device, dtype=torch.float32).contiguous() for s in scales)
        p.q_scale, p.k_scale, p.v_scale = qs.data_ptr(), ks.data_ptr(), vs.data_ptr()
        keep += [qs, ks, vs]
    p.impl = impl
    return p, keep


def _check_inputs(q: Tensor, k: Tensor, v: Tensor) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("query, key and value must be 4-D (batch, heads, tokens, head_dim)")
    if k.shape != q.shape:
        raise ValueError(f"key shape {tuple(k.shape)} != query shape {tuple(q.shape)}")
    if v.shape[:3] != q.shape[:3]:
        raise ValueError(f"value shape {tuple(v.shape)} does not match query {tuple(q.shape)}")
    mixed = v.dtype == torch.float32 and q.dtype in (torch.float16, torch.bfloat16)
    if not (q.dtype == k.dtype and (v.dtype == q.dtype or mixed)):
        raise TypeError(f"query/key/value dtypes differ: {q.dtype}, {k.dtype}, {v.dtype} "
                        "(fp32 values with fp16 / bf16 queries and keys are accepted)")
    if q.dtype not in _TORCH_TO_MA:
        raise TypeError(f"unsupported dtype {q.dtype}")
    for t in (q, k, v):
        if t.device.type != "cuda":
            raise RuntimeError("MonarchAttention (B200) runs on CUDA tensors only; "
                               f"got a tensor on {t.device}")
    if not (q.device == k.device == v.device):
        raise ValueError("query/key/value are on different devices")


def _needs_grad(q: Tensor, k: Tensor, v: Tensor) -> bool:
    return torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)


def monarch_attention(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None, T: int,
                      B: int, pre_pad: bool, *, impl=None, scales: tuple | None = None,
                      out: Tensor | None = None, check: bool = False) -> Tensor:
    """MonarchAttention forward on the current CUDA stream.

    Same arguments and result as ``monarch_attention_torch``
    (ma/ma_torch.py:65-108): q, k (E, H, N, D), v (E, H, N, Dv), optional
    (E, N) mask (nonzero = valid), T alternating steps, block size B, and
    pre_pad selecting front padding.  Returns a new contiguous (E, H, N, Dv)
    tensor in v.dtype (bf16 for float8_e4m3fn inputs, which also need
    ``scales=(q_scale, k_scale, v_scale)``, each (E, H) fp32).

    ``out`` (optional) receives the result instead of a new tensor: an
    (E, H, N, Dv) tensor of the output dtype with any strides, e.g. the
    ``(E, N, H, Dv)`` buffer of the next projection seen through
    ``.permute(0, 2, 1, 3)``; with q, k, v passed as the same kind of views
    of the (E, N, H*D) projections, no layout copy is made on either side.

    Device-side failures (a bounded wait in a kernel that ran out) raise
    ``MonarchAttentionError`` with code MA_ERR_DEVICE: at the latest at the
    next call on the same device (the kernel writes a page-locked host word,
    so this costs no synchronisation), immediately with ``check=True`` (which
    waits for the device), or from ``check_status()``.
    """
    _check_inputs(q, k, v)
    if _needs_grad(q, k, v):
        if q.dtype == torch.float8_e4m3fn or scales is not None:
            raise RuntimeError("gradients through float8 e4m3 inputs are not supported")
        if out is not None:
            raise ValueError("out= cannot be used when gradients are required")
        res = training.MonarchAttentionFunction.apply(q, k, v, attn_mask, T, B, pre_pad, impl,
                                                      _kernel_forward, _kernel_backward)
    else:
        res = _kernel_forward(q, k, v, attn_mask, T, B, pre_pad, impl, scales, out)
    if check:
        check_status(q.device)
    return res


def _kernel_forward(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None, T: int, B: int,
                    pre_pad: bool, impl=None, scales: tuple | None = None,
                    out: Tensor | None = None) -> Tensor:
    """One ``ma_fwd`` call on the current stream (inputs already checked)."""
    E, H, N, _ = q.shape
    Dv = v.shape[-1]
    out_dtype = torch.bfloat16 if q.dtype == torch.float8_e4m3fn else v.dtype
    if q.dtype == torch.float8_e4m3fn and scales is None:
        raise ValueError("float8_e4m3fn inputs need scales=(q_scale, k_scale, v_scale)")
    if out is None:
        out = torch.empty((E, H, N, Dv), dtype=out_dtype, device=q.device)
    else:
        if tuple(out.shape) != (E, H, N, Dv):
            raise ValueError(f"out shape {tuple(out.shape)} != {(E, H, N, Dv)}")
        if out.dtype != out_dtype:
            raise TypeError(f"out dtype {out.dtype} != {out_dtype}")
        if out.device != q.device:
            raise ValueError("out is on a different device than the inputs")
    lib = _lib.load()
    _check_previous(q.device)
    p, keep = build_params(q, k, v, out, attn_mask, T, B, pre_pad, _impl_code(impl), scales)
    nbytes = lib.ma_workspace_bytes(ctypes.byref(p))
    if nbytes == 0:
        _lib.check(lib.ma_fwd(ctypes.byref(p), None))  # raises with the reason
    with torch.cuda.device(q.device):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
        p.status = status_word(q.device).data_ptr()
        p.status_host = _mirror_ptr(q.device)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        nvtx = os.environ.get("MA_NVTX") == "1"
        if nvtx:
            torch.cuda.nvtx.range_push(f"monarch_attention E{E} H{H} N{N} B{B} T{T}")
        rc = lib.ma_fwd(ctypes.byref(p), ctypes.c_void_p(stream))
        if rc == _lib.MA_ERR_BAD_PARAMS and p.status_host and \
                b"status_host" in lib.ma_last_error_detail():
            _mirror_refused.add(_dev_index(q.device))
            p.status_host = None
            rc = lib.ma_fwd(ctypes.byref(p), ctypes.c_void_p(stream))
        if nvtx:
            torch.cuda.nvtx.range_pop()
    _lib.check(rc)
    del keep
    return out


def _kernel_backward(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None, T: int, B: int,
                     pre_pad: bool, g: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """One ``ma_bwd`` call on the current stream: d<out, g>/d(q, k, v)."""
    _check_previous(q.device)
    lib = _lib.load()
    g = g.to(v.dtype)
    fp, keep = build_params(q, k, v, g, attn_mask, T, B, pre_pad)
    bp = _lib.MaBwdParams()
    bp.fwd = fp
    bp.dout = g.data_ptr()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    for name, t in (("dout_stride", g), ("dq_stride", dq), ("dk_stride", dk), ("dv_stride", dv)):
        arr = getattr(bp, name)
        for i, st in enumerate(t.stride()):
            arr[i] = st
    bp.dq, bp.dk, bp.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    nbytes = lib.ma_bwd_workspace_bytes(ctypes.byref(bp))
    if nbytes == 0:
        _lib.check(lib.ma_bwd(ctypes.byref(bp), None))  # raises with the reason
    with torch.cuda.device(q.device):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        bp.workspace, bp.workspace_bytes = ws.data_ptr(), nbytes
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = lib.ma_bwd(ctypes.byref(bp), ctypes.c_void_p(stream))
    _lib.check(rc)
    del keep
    return dq, dk, dv


def selected_impl(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None, T: int, B: int,
                  pre_pad: bool, impl=None) -> str:
    """Name of the kernel family ``monarch_attention`` would run
    ("generic" / "tc" / "small")."""
    lib = _lib.load()
    out = torch.empty((1,), device=q.device)
    p, _keep = build_params(q, k, v, out, attn_mask, T, B, pre_pad, _impl_code(impl))
    p.out_dtype = (_lib.DTYPE_F32 if p.v_f32 else
                   p.dtype if p.dtype != _lib.DTYPE_E4M3 else _lib.DTYPE_BF16)
    for i, s in enumerate((q.shape[1] * q.shape[2] * v.shape[-1], q.shape[2] * v.shape[-1],
                           v.shape[-1], 1)):
        p.o_stride[i] = s
    rc = lib.ma_select_impl(ctypes.byref(p))
    if rc < 0:
        _lib.check(-rc)
    return _lib.IMPL_NAMES[rc]


class MonarchAttention(nn.Module):
    """MonarchAttention (ma/monarch_attention.py:17-70) on B200 CUDA kernels.

    ``impl``: None / "auto" (default) picks the fastest kernel for the shape;
    "generic", "tc" or "small" force a kernel family; the reference's "torch" and
    "triton" are accepted and mean "auto".  The MA_IMPL environment variable
    overrides it (for tests).
    """

    def __init__(self, block_size: int, num_steps: int, pad_type: PadType,
                 impl: str | None = None):
        super().__init__()
        self.block_size = block_size
        self.num_steps = num_steps
        self.pad_type = pad_type
        _impl_code(impl)  # validate early
        self.impl = impl

    def forward(self, query: Tensor, key: Tensor, value: Tensor,
                attention_mask: Tensor | None = None) -> Tensor:
        return monarch_attention(query, key, value, attention_mask, self.num_steps,
                                 self.block_size, self.pad_type == PadType.pre, impl=self.impl)

    def get_matrix(self, query: Tensor, key: Tensor,
                   attention_mask: Tensor | None = None) -> Tensor:
        """Dense (E, H, N, N) attention matrix: the forward with V = I.

        As in the reference (ma/monarch_attention.py:60-70) the identity is
        fp32 whatever the query dtype, so with 16-bit queries the R / L steps
        run in the query dtype and y and the output step in fp32; the result
        is fp32.
        """
        batch_size, num_heads, seq_len, _ = query.shape
        value = torch.eye(seq_len, device=query.device, dtype=torch.float32).expand(
            batch_size, num_heads, seq_len, seq_len)
        return self.forward(query, key, value, attention_mask)

    def extra_repr(self) -> str:
        return (f"block_size={self.block_size}, num_steps={self.num_steps}, "
                f"pad_type={self.pad_type}, impl={self.impl}")
