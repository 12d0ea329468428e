"""Gradients of the MonarchAttention forward.

The reference trains MonarchAttention (BART fine-tuning,
bart/run_summarization.py) through PyTorch autograd over its torch
implementation, ma/ma_torch.py.  Here the forward pass runs on the CUDA
kernels, and the backward pass recomputes the forward with autograd over
``torch_forward`` -- a restatement of ma/ma_torch.py:10-108 with the same
operations, casts and rounding points -- and differentiates that, so the
gradients are the reference's own.  The recomputation materialises the
(E, H, M, b, b) and (E, H, b, M, M) weights like the reference does.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

_EPS = 1e-12  # ma_torch.py:10, 38


def _key_block_step(ar: Tensor, k: Tensor, cr: Tensor, scale: float, valid: Tensor,
                    v: Tensor | None = None):
    """R-step (ma_torch.py:10-23; with ``v`` the final one, :38-52).

    For every key block m, row j: a row softmax of sm_scale * ar[m] k[m]^T
    (rounded to the input dtype, then fp32) divided by cr[m][j] + eps, over
    the valid keys, with the max clamped at eps, the sum offset by eps and r
    clamped at the smallest normal.  Returns al [.., j, m, :], cl [.., j, m]
    and, with ``v``, y [.., j, m, :].
    """
    logits = scale * (ar @ k.transpose(-1, -2)).to(torch.float)
    logits = logits / (cr.unsqueeze(-1) + _EPS)
    logits = logits + torch.where(valid.unsqueeze(-2), 0.0, -float("inf"))
    shift = torch.clamp(torch.max(logits, dim=-1, keepdim=True).values, min=_EPS)
    e = torch.exp(logits - shift)
    r = e / (torch.sum(e, dim=-1, keepdim=True) + _EPS)
    r = torch.clamp(r, min=torch.finfo(r.dtype).tiny)
    cl = torch.sum(torch.special.xlogy(r, r), dim=-1).transpose(-1, -2)
    al = (scale * (r.to(k.dtype) @ k)).transpose(-2, -3)
    y = None if v is None else (r.to(v.dtype) @ v).transpose(-2, -3)
    return al, cl, y


def _index_step(al: Tensor, qt: Tensor, cl: Tensor, valid_t: Tensor):
    """L-step (ma_torch.py:26-35): for every intra-block index j, a softmax
    over key blocks (dim -2) of al_j q_j^T - cl, times the query mask; returns
    ar [.., m, j, :] and cr [.., m, j]."""
    logits = (al @ qt.transpose(-1, -2)).to(torch.float) - cl.unsqueeze(-1)
    p = F.softmax(logits, dim=-2) * valid_t.unsqueeze(-2)
    cr = torch.sum(p, dim=-1).transpose(-1, -2)
    ar = (p.to(qt.dtype) @ qt).transpose(-2, -3)
    return ar, cr


def _output_step(al: Tensor, qt: Tensor, cl: Tensor, y: Tensor) -> Tensor:
    """Output (ma_torch.py:55-62): softmax over key blocks of q_j al_j^T - cl
    (no mask), applied to y_j."""
    logits = (qt @ al.transpose(-1, -2)).to(torch.float) - cl.unsqueeze(-2)
    p = F.softmax(logits, dim=-1)
    return (p.to(y.dtype) @ y).transpose(-2, -3).contiguous()


def torch_forward(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None, T: int, B: int,
                  pre_pad: bool) -> Tensor:
    """The MonarchAttention forward of ma/ma_torch.py:65-108 in torch ops
    (any device); differentiable."""
    E, H, N, D = q.shape
    Dv = v.shape[-1]
    M = (N + B - 1) // B
    Np = M * B
    pad = Np - N
    scale = 1 / math.sqrt(D)
    side = (pad, 0) if pre_pad else (0, pad)
    qb = F.pad(q, (0, 0) + side).view(E, H, M, B, D)
    kb = F.pad(k, (0, 0) + side).view(E, H, M, B, D)
    vb = F.pad(v, (0, 0) + side).view(E, H, M, B, Dv)
    idx = torch.arange(Np, device=q.device).view(M, B)
    valid = idx >= pad if pre_pad else idx < N
    if attn_mask is not None:
        valid = torch.logical_and(valid, F.pad(attn_mask, side).view(E, 1, M, B))
    ar = qb
    cr = torch.ones(E, H, M, B, device=q.device, dtype=torch.float)
    qt = qb.transpose(-2, -3)
    for _ in range(T - 1):
        al, cl, _ = _key_block_step(ar, kb, cr, scale, valid)
        ar, cr = _index_step(al, qt, cl, valid.mT)
    al, cl, y = _key_block_step(ar, kb, cr, scale, valid, vb)
    z = _output_step(al, qt, cl, y).view(E, H, Np, Dv)
    return z[..., pad:, :] if pre_pad else z[..., :N, :]


class MonarchAttentionFunction(torch.autograd.Function):
    """Forward on the CUDA kernels, backward by recomputation (see module
    docstring).  Arguments after q, k, v are not differentiable."""

    @staticmethod
    def forward(ctx, q, k, v, attn_mask, T, B, pre_pad, impl, kernel_forward):
        ctx.save_for_backward(q, k, v)
        ctx.attn_mask = attn_mask
        ctx.args = (T, B, pre_pad)
        with torch.no_grad():
            return kernel_forward(q.detach(), k.detach(), v.detach(), attn_mask, T, B, pre_pad,
                                  impl)

    @staticmethod
    def backward(ctx, g):
        q, k, v = ctx.saved_tensors
        need = ctx.needs_input_grad[:3]
        with torch.enable_grad():
            leaves = [t.detach().requires_grad_(n) for t, n in zip((q, k, v), need)]
            out = torch_forward(*leaves, ctx.attn_mask, *ctx.args)
            wrt = [t for t in leaves if t.requires_grad]
            grads = iter(torch.autograd.grad(out, wrt, g.to(out.dtype)))
        dq, dk, dv = (next(grads) if n else None for n in need)
        return dq, dk, dv, None, None, None, None, None, None
