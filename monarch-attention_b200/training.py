"""Gradients of the MonarchAttention forward on the CUDA kernels.

The reference trains MonarchAttention (BART fine-tuning,
bart/run_summarization.py) through PyTorch autograd over ma/ma_torch.py.
Here inputs that require gradients go through ``MonarchAttentionFunction``:
the forward runs on the forward kernels (``ma_fwd``) and the backward on the
backward kernels (``ma_bwd``, include/ma_api.h), which recompute the forward
with every step's intermediates kept and differentiate each phase in
reverse order -- the same gradients as autograd over the reference.
"""
from __future__ import annotations

import torch


class MonarchAttentionFunction(torch.autograd.Function):
    """Forward on ``ma_fwd``, backward on ``ma_bwd``.  Arguments after q, k,
    v are not differentiable."""

    @staticmethod
    def forward(ctx, q, k, v, attn_mask, T, B, pre_pad, impl, kernel_forward, kernel_backward):
        ctx.save_for_backward(q, k, v)
        ctx.attn_mask = attn_mask
        ctx.args = (T, B, pre_pad)
        ctx.kernel_backward = kernel_backward
        with torch.no_grad():
            return kernel_forward(q.detach(), k.detach(), v.detach(), attn_mask, T, B, pre_pad,
                                  impl)

    @staticmethod
    def backward(ctx, g):
        q, k, v = ctx.saved_tensors
        need = ctx.needs_input_grad[:3]
        dq, dk, dv = ctx.kernel_backward(q.detach(), k.detach(), v.detach(), ctx.attn_mask,
                                         *ctx.args, g)
        grads = [t if n else None for t, n in zip((dq, dk, dv), need)]
        return (*grads, None, None, None, None, None, None, None)
