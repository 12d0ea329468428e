"""Generate the golden fixtures by running the reference implementation itself.

Run once, in a checkout that has the reference repository available:

    python tests/golden/gen_golden.py --reference <path to djmmoss/monarch-attention>

For every case it draws seeded inputs, runs the reference's
``monarch_attention_torch`` (ma/ma_torch.py:65-108) on CPU in the case's dtype
and again in fp32 on the same (already rounded) inputs, and writes
``tests/golden/<case>.npz``.  The fixtures are what pins the CPU oracle
(``oracle/ma_oracle.py``) to the reference; tests never need the reference.

Input distribution follows the benchmark configs: iid N(0, 1), scaled by
1/sqrt(d) unless the case is "unscaled" (the long-sequence sweep).  Masks are
key-padding masks with a per-sequence valid length.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (E, H, N, D, Dv, B, T, pad, dtype, scaled, mask_kind, seed)
CASES = {
    # config 0 (fp32 B=2 H=12 N=256 d=64 b=16 T=3), reduced to 2 heads
    "cfg0_f32": (1, 2, 256, 64, 64, 16, 3, "post", "f32", True, None, 1000),
    # ViT-B/16 shape (N=196 = 14 x 14), reduced batch
    "vit_bf16": (1, 2, 196, 64, 64, 14, 2, "post", "bf16", True, None, 1001),
    # RoBERTa shape with a key-padding mask, valid length uniform in [128, 512]
    "roberta_mask_bf16": (2, 2, 512, 64, 64, 32, 2, "post", "bf16", True, "len128", 1002),
    # DiT-XL/2 shape: d = 72, T = 3
    "dit_bf16": (1, 1, 1024, 72, 72, 32, 3, "post", "bf16", True, None, 1003),
    # long-sequence sweep distribution (unscaled), shortened
    "long_bf16": (1, 1, 512, 128, 128, 32, 2, "post", "bf16", False, None, 1004),
    # real ViT sequence (197 tokens incl. CLS) pre-padded to 14 x 15, fp16, mask
    "vit197_prepad_f16": (2, 1, 197, 64, 64, 14, 2, "pre", "f16", True, "len64", 1005),
    # post-padding, Dv != D, one fully masked sequence, fp32
    "postpad_dv_f32": (2, 2, 100, 32, 48, 8, 2, "post", "f32", True, "one_empty", 1006),
    # T = 1: no alternating rounds, only the final R-step and the output
    "t1_f32": (1, 2, 64, 16, 16, 8, 1, "post", "f32", True, None, 1007),
    # pre-padding without a mask, T = 3, bf16
    "prepad_t3_bf16": (1, 2, 90, 32, 32, 16, 3, "pre", "bf16", True, None, 1008),
    # a mask that empties whole key blocks (blocks 1 and 2 of 4), fp32
    "masked_blocks_f32": (1, 1, 64, 16, 16, 16, 2, "post", "f32", True, "blocks", 1009),
}

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def make_inputs(E, H, N, D, Dv, dtype, scaled, mask_kind, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(E, H, N, D, generator=g)
    k = torch.randn(E, H, N, D, generator=g)
    v = torch.randn(E, H, N, Dv, generator=g)
    if scaled:
        q, k, v = q / math.sqrt(D), k / math.sqrt(D), v / math.sqrt(D)
    q, k, v = (t.to(TORCH_DT[dtype]) for t in (q, k, v))
    mask = None
    if mask_kind == "len128":
        lens = torch.randint(128, N + 1, (E,), generator=g)
        mask = torch.arange(N)[None, :] < lens[:, None]
    elif mask_kind == "len64":
        lens = torch.randint(64, N + 1, (E,), generator=g)
        mask = torch.arange(N)[None, :] < lens[:, None]
    elif mask_kind == "one_empty":
        mask = torch.ones(E, N, dtype=torch.bool)
        mask[0, N // 2:] = False
        mask[1, :] = False
    elif mask_kind == "blocks":
        mask = torch.ones(E, N, dtype=torch.bool)
        mask[:, 16:48] = False
    return q, k, v, mask


def pack(t: torch.Tensor) -> np.ndarray:
    """16-bit tensors are stored as their raw uint16 bit patterns (see load_case)."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def load_case(path: str) -> dict:
    """Load a fixture; 16-bit tensors come back as exactly-representable float32."""
    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    out = {"meta": meta}
    for key in z.files:
        if key == "meta":
            continue
        a = z[key]
        if a.dtype == np.uint16:
            if meta["dtype"] == "bf16":
                a = (a.astype(np.uint32) << 16).view(np.float32)
            else:
                a = a.view(np.float16).astype(np.float32)
        out[key] = a
    return out


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
        pre = pad == "pre"
        out = monarch_attention_torch(q, k, v, mask, T, B, pre)
        out32 = monarch_attention_torch(q.float(), k.float(), v.float(), mask, T, B, pre)
        meta = dict(E=E, H=H, N=N, D=D, Dv=Dv, B=B, T=T, pre_pad=pre, dtype=dtype,
                    scaled=scaled, mask=mk, seed=seed)
        arrays = dict(q=pack(q), k=pack(k), v=pack(v), out_ref=pack(out),
                      out_ref_f32=out32.numpy(), meta=np.array(json.dumps(meta)))
        if mask is not None:
            arrays["mask"] = mask.numpy()
        path = os.path.join(args.out, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{name}: {tuple(out.shape)} max|out|={out.float().abs().max():.4g} -> {path}")


if __name__ == "__main__":
    main()
