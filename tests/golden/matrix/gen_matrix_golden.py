"""Generate the get_matrix fixtures by running the reference itself.

    python tests/golden/matrix/gen_matrix_golden.py --reference <path to djmmoss/monarch-attention>

The reference's ``MonarchAttention.get_matrix`` (ma/monarch_attention.py:60-70)
runs the forward with an fp32 identity as the values, whatever the query
dtype: with 16-bit queries its R / L logits and ``al`` are rounded to the
query dtype while y and z stay fp32.  Each case draws seeded 16-bit q, k
(and a mask), runs ``get_matrix`` on CPU and writes
``tests/golden/matrix/<case>.npz`` with the inputs and the (E, H, N, N) fp32
matrix.  Tests never need the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (E, H, N, D, B, T, pad_type, dtype, mask_len, seed)
CASES = {
    "matrix_bf16": (1, 2, 64, 32, 8, 2, "post", "bf16", None, 2001),
    "matrix_f16_prepad_mask": (2, 1, 60, 16, 8, 3, "pre", "f16", 41, 2002),
}
TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from ma.monarch_attention import MonarchAttention, PadType  # the reference itself

    for name, (E, H, N, D, B, T, pad, dt, mlen, seed) in CASES.items():
        g = torch.Generator(device="cpu").manual_seed(seed)
        q = (torch.randn(E, H, N, D, generator=g) / np.sqrt(D)).to(TORCH_DT[dt])
        k = (torch.randn(E, H, N, D, generator=g) / np.sqrt(D)).to(TORCH_DT[dt])
        mask = None
        if mlen is not None:
            mask = torch.ones(E, N, dtype=torch.bool)
            mask[0, mlen:] = False
        attn = MonarchAttention(B, T, PadType(pad))
        with torch.no_grad():
            mat = attn.get_matrix(q, k, mask)
        meta = dict(E=E, H=H, N=N, D=D, B=B, T=T, pre_pad=pad == "pre", dtype=dt,
                    out_dtype=str(mat.dtype))
        arrs = dict(q=q.float().numpy(), k=k.float().numpy(), matrix=mat.float().numpy(),
                    meta=np.array(json.dumps(meta)))
        if mask is not None:
            arrs["mask"] = mask.numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, meta, float(mat.float().abs().max()))


if __name__ == "__main__":
    main()
