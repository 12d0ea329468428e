"""Generate gradient fixtures by running the reference implementation itself.

Run once, in a checkout that has the reference repository available:

    python tests/golden/grad/gen_grad_golden.py --reference <path to djmmoss/monarch-attention>

The reference trains MonarchAttention (BART fine-tuning) through PyTorch
autograd over ``monarch_attention_torch`` (ma/ma_torch.py:65-108).  For every
case this draws seeded inputs and a seeded upstream gradient g, runs the
reference forward on CPU with autograd and writes the output and
dq, dk, dv = d<out, g>/d(q, k, v) to ``tests/golden/grad/<case>.npz``.  The
fixtures pin the library's backward; tests never need the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from gen_golden import TORCH_DT, make_inputs, pack  # noqa: E402

# name: (E, H, N, D, Dv, B, T, pad, dtype, scaled, mask_kind, seed)
CASES = {
    # two alternating steps, no padding, no mask
    "grad_t2_f32": (1, 2, 64, 16, 16, 8, 2, "post", "f32", True, None, 2001),
    # T = 3, pre-padding, Dv != D, a key-padding mask with an empty tail
    "grad_t3_prepad_mask_f32": (2, 1, 45, 16, 24, 8, 3, "pre", "f32", True, "one_empty", 2002),
    # T = 1 (final R-step and output only), post-padding
    "grad_t1_postpad_f32": (1, 2, 30, 8, 8, 4, 1, "post", "f32", True, None, 2003),
    # bf16 with the reference's rounding points
    "grad_t2_bf16": (1, 2, 64, 32, 32, 16, 2, "post", "bf16", True, None, 2004),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from ma.ma_torch import monarch_attention_torch  # noqa: E402  (reference)

    torch.set_num_threads(os.cpu_count() or 1)
    for name, (E, H, N, D, Dv, B, T, pad, dtype, scaled, mk, seed) in CASES.items():
        q, k, v, mask = make_inputs(E, H, N, D, Dv, dtype, scaled, mk, seed)
        gen = torch.Generator(device="cpu").manual_seed(seed + 77)
        g = torch.randn(E, H, N, Dv, generator=gen).to(TORCH_DT[dtype])
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
        out = monarch_attention_torch(*leaves, mask, T, B, pad == "pre")
        dq, dk, dv = torch.autograd.grad(out, leaves, g)
        meta = dict(E=E, H=H, N=N, D=D, Dv=Dv, B=B, T=T, pre_pad=pad == "pre", dtype=dtype,
                    scaled=scaled, mask=mk, seed=seed)
        arrays = dict(q=pack(q), k=pack(k), v=pack(v), g=pack(g), out=pack(out.detach()),
                      dq=pack(dq), dk=pack(dk), dv=pack(dv), meta=np.array(json.dumps(meta)))
        if mask is not None:
            arrays["mask"] = mask.numpy()
        path = os.path.join(args.out, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{name}: max|dq|={dq.float().abs().max():.4g} max|dk|={dk.float().abs().max():.4g} "
              f"max|dv|={dv.float().abs().max():.4g} -> {path}")


if __name__ == "__main__":
    main()
