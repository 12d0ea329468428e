"""CPU oracle for the MonarchAttention forward pass -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may
import it.  The shipped path (``monarch_attention_b200``) runs hand-written
sm_100a CUDA and raises when its extension is missing.

It restates, in numpy, the reference's PyTorch implementation
``ma/ma_torch.py`` of djmmoss/monarch-attention:

  * ``_r_step``      <- ``al_cl_ref`` (ma/ma_torch.py:10-23) and
                        ``al_y_cl_ref`` (ma/ma_torch.py:38-52)
  * ``_l_step``      <- ``ar_cr_ref`` (ma/ma_torch.py:26-35)
  * ``_z_step``      <- ``z_ref``     (ma/ma_torch.py:55-62)
  * ``monarch_attention_oracle`` <- ``monarch_attention_torch``
                        (ma/ma_torch.py:65-108)

Reduced precision is emulated exactly where the reference rounds: every
matmul of 16-bit operands accumulates in fp32 and rounds its output to the
input dtype, softmax statistics stay fp32, and a weight matrix is cast to the
input dtype before it becomes a matmul operand (ma/ma_torch.py:11, 21, 27, 34,
39, 50-51, 56, 60).  ``dtype="f32"`` applies no rounding.

Parity is pinned against the reference itself: ``tests/golden/gen_golden.py``
ran ``ma/ma_torch.py`` on seeded inputs and committed the outputs as fixtures,
and ``tests/test_oracle.py`` checks this module against every fixture.
"""
from __future__ import annotations

import math

import numpy as np

EPS = 1e-12  # ma/ma_torch.py:10, 38 (eps default of the R-step helpers)
TINY = np.finfo(np.float32).tiny  # torch.finfo(float32).tiny, ma/ma_torch.py:18

DTYPES = ("f32", "f16", "bf16")


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the precision of ``dtype`` (returned as float32).

    bf16 uses round-to-nearest-even on the top 16 bits of the float32 pattern,
    which is what a float32 -> bfloat16 cast does; NaN/Inf pass through.
    """
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        out = rounded.astype(np.uint32).view(np.float32)
        special = ~np.isfinite(x)
        if special.any():
            out = np.where(special, x, out)
        return out.astype(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def _mm(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Batched matmul with fp32 accumulation, output rounded to ``dtype``."""
    return round_to(np.matmul(a, b, dtype=np.float32), dtype)


def _softmax(x: np.ndarray, axis: int) -> np.ndarray:
    """F.softmax in fp32: exp(x - max) / sum along ``axis``."""
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def _r_step(ar, k, v, cr, sm_scale, mask, dtype, want_y, v_dtype=None):
    """R-step for every key block (ma/ma_torch.py:10-23, 38-52).

    ar, k: (..., M, B, D); v: (..., M, B, Dv) or None; cr: (..., M, B) fp32;
    mask: broadcastable to (..., M, B) bool (key validity).
    Returns al (..., B, M, D), cl (..., B, M), y (..., B, M, Dv) or None.
    ``v_dtype`` (default ``dtype``): the value dtype, in which y = r.to(v.dtype)
    @ v is computed (:51).
    """
    r_hat = np.float32(sm_scale) * _mm(ar, np.swapaxes(k, -1, -2), dtype)
    r_hat = r_hat / (cr[..., :, None] + np.float32(EPS))
    r_hat = r_hat + np.where(mask[..., None, :], np.float32(0.0), np.float32(-np.inf))
    mx = np.maximum(np.max(r_hat, axis=-1, keepdims=True), np.float32(EPS))
    r_hat = np.exp(r_hat - mx)
    r = r_hat / (np.sum(r_hat, axis=-1, keepdims=True) + np.float32(EPS))
    r = np.maximum(r, TINY).astype(np.float32)

    cl = np.swapaxes(np.sum(r * np.log(r), axis=-1), -1, -2)
    r_op = round_to(r, dtype)
    al = round_to(np.float32(sm_scale) * _mm(r_op, k, dtype), dtype)
    al = np.swapaxes(al, -2, -3)
    y = None
    if want_y:
        vd = v_dtype or dtype
        y = np.swapaxes(_mm(round_to(r, vd), v, vd), -2, -3)
    return al, cl.astype(np.float32), y


def _l_step(al, q_t, cl, mask_t, dtype):
    """L-step for every intra-block index j (ma/ma_torch.py:26-35).

    al: (..., B, M, D); q_t: (..., B, M, D); cl: (..., B, M);
    mask_t: broadcastable to (..., B, M) (query validity, 0/1).
    Returns ar (..., M, B, D) and cr (..., M, B).
    """
    l_hat = _mm(al, np.swapaxes(q_t, -1, -2), dtype)
    l_hat = l_hat - cl[..., :, None]
    l = _softmax(l_hat, axis=-2)
    l = mask_t[..., None, :].astype(np.float32) * l
    cr = np.swapaxes(np.sum(l, axis=-1), -1, -2)
    ar = np.swapaxes(_mm(round_to(l, dtype), q_t, dtype), -2, -3)
    return ar, cr.astype(np.float32)


def _z_step(al, q_t, cl, y, dtype, v_dtype=None):
    """Output step (ma/ma_torch.py:55-62): softmax over key blocks, times y
    (in the value dtype ``v_dtype``, default ``dtype``: l.to(y.dtype) @ y)."""
    l_hat = _mm(q_t, np.swapaxes(al, -1, -2), dtype)
    l_hat = l_hat - cl[..., None, :]
    l = _softmax(l_hat, axis=-1)
    vd = v_dtype or dtype
    z = _mm(round_to(l, vd), y, vd)
    return np.swapaxes(z, -2, -3)


def validity_mask(E: int, N: int, B: int, pre_pad: bool, attn_mask=None) -> np.ndarray:
    """Token validity of the padded sequence, shape (E or 1, M, B) bool.

    ma/ma_torch.py:92-98: pad positions are invalid (the front ones when
    ``pre_pad``), and ``attn_mask`` (E, N), nonzero = valid, is padded on the
    same side and AND-ed in.
    """
    M = (N + B - 1) // B
    Np = M * B
    pad = Np - N
    rng = np.arange(Np).reshape(M, B)
    mask = rng >= pad if pre_pad else rng < N
    mask = mask[None]
    if attn_mask is not None:
        am = np.asarray(attn_mask) != 0
        am = np.pad(am, ((0, 0), (pad, 0) if pre_pad else (0, pad)))
        mask = np.logical_and(mask, am.reshape(am.shape[0], M, B))
    return mask


def monarch_attention_oracle(q, k, v, attn_mask, T: int, B: int, pre_pad: bool,
                             dtype: str = "f32", v_dtype: str | None = None) -> np.ndarray:
    """MonarchAttention forward (ma/ma_torch.py:65-108) on CPU.

    q, k: (E, H, N, D); v: (E, H, N, Dv) float arrays whose values are already
    representable in ``dtype``.  attn_mask: None or (E, N), nonzero = valid.
    ``v_dtype`` (default ``dtype``): a different value dtype, as in the
    reference's ``get_matrix`` (fp32 identity values with 16-bit queries,
    ma/monarch_attention.py:60-70): y and z are then computed in it.
    Returns (E, H, N, Dv) float32 (values rounded to the value dtype).
    """
    if dtype not in DTYPES or (v_dtype is not None and v_dtype not in DTYPES):
        raise ValueError(f"dtype must be one of {DTYPES}")
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    E, H, N, D = q.shape
    Dv = v.shape[-1]
    M = (N + B - 1) // B
    Np = M * B
    sm_scale = 1.0 / math.sqrt(D)
    pad = ((Np - N, 0) if pre_pad else (0, Np - N))
    padw = ((0, 0), (0, 0), pad, (0, 0))
    qb = np.pad(q, padw).reshape(E, H, M, B, D)
    kb = np.pad(k, padw).reshape(E, H, M, B, D)
    vb = np.pad(v, padw).reshape(E, H, M, B, Dv)

    ar = qb
    cr = np.ones((E, H, M, B), dtype=np.float32)
    q_t = np.swapaxes(qb, -2, -3)

    mask = validity_mask(E, N, B, pre_pad, attn_mask)[:, None]  # (E|1, 1, M, B)
    mask_t = np.swapaxes(mask, -1, -2)

    for _ in range(T - 1):
        al, cl, _ = _r_step(ar, kb, None, cr, sm_scale, mask, dtype, False)
        ar, cr = _l_step(al, q_t, cl, mask_t, dtype)
    al, cl, y = _r_step(ar, kb, vb, cr, sm_scale, mask, dtype, True, v_dtype)
    z = _z_step(al, q_t, cl, y, dtype, v_dtype).reshape(E, H, Np, Dv)
    return z[:, :, Np - N:, :] if pre_pad else z[:, :, :N, :]


def monarch_attention_oracle_heads(q, k, v, attn_mask, T, B, pre_pad, dtype="f32",
                                   v_dtype=None):
    """Same as :func:`monarch_attention_oracle`, one (e, h) at a time.

    Heads and batch rows never interact (ma/ma_torch.py mixes neither), so
    this is exact; it bounds peak memory on long sequences.
    """
    q = np.asarray(q)
    E, H, N, _ = q.shape
    out = np.empty((E, H, N, np.asarray(v).shape[-1]), dtype=np.float32)
    for e in range(E):
        am = None if attn_mask is None else np.asarray(attn_mask)[e:e + 1]
        for h in range(H):
            out[e, h] = monarch_attention_oracle(
                q[e:e + 1, h:h + 1], k[e:e + 1, h:h + 1], v[e:e + 1, h:h + 1],
                am, T, B, pre_pad, dtype, v_dtype)[0, 0]
    return out


def flops(E, H, N, D, Dv, B, T) -> float:
    """Algorithmic FLOPs of one forward, counted on the padded length.

    (T-1) rounds of R-step (2 GEMMs of B x B x D per block) and L-step
    (2 GEMMs of M x M x D per index), a final R-step with the extra y GEMM
    (B x B x Dv) and the output step (M x M x D and M x M x Dv).
    """
    M = (N + B - 1) // B
    Np = M * B
    per_head = ((T - 1) * (4 * Np * B * D + 4 * Np * M * D)
                + 4 * Np * B * D + 2 * Np * B * Dv
                + 2 * Np * M * D + 2 * Np * M * Dv)
    return float(E * H * per_head)


def hbm_bytes(E, H, N, D, Dv, in_bytes, out_bytes, mask_bytes=0) -> float:
    """Algorithmic HBM bytes: Q, K, V read once, O written once (+ the mask)."""
    return float(E * H * N * (2 * D + Dv) * in_bytes + E * H * N * Dv * out_bytes
                 + mask_bytes)
