"""Benchmark / parity configurations and seeded synthetic inputs.

The shapes are the attention layers the reference evaluates MonarchAttention
in: a fp32 CPU-checkable case, ViT-B/16 (vit/benchmark.py), RoBERTa-base with
a key-padding mask (roberta/benchmark.py), DiT-XL/2 at 512 px
(dit/sample_fid.py, head_dim 72 per dit/model.py:20) and a long-sequence
sweep with b = sqrt(N) (perfbench/bench.py:427-445).  The datasets and model
weights behind them are not used: inputs are iid N(0, 1) from a seeded
generator, scaled by 1/sqrt(d) where the config says so, and masks draw a
per-sequence valid length.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Config:
    name: str
    E: int
    H: int
    N: int
    D: int
    B: int
    T: int
    dtype: str  # "f32" | "bf16" | "f16" | "e4m3"
    scaled: bool = True
    mask_min_len: int | None = None  # key-padding mask: valid length in [min, N]
    pre_pad: bool = False
    Dv: int | None = None
    seed: int = 1000

    @property
    def dv(self) -> int:
        return self.Dv or self.D

    @property
    def M(self) -> int:
        return (self.N + self.B - 1) // self.B

    def with_(self, **kw) -> "Config":
        d = dict(self.__dict__)
        d.update(kw)
        return Config(**d)


CONFIGS = {
    c.name: c
    for c in [
        Config("cfg0_f32", 2, 12, 256, 64, 16, 3, "f32", seed=1000),
        Config("vit_bf16", 64, 12, 196, 64, 14, 2, "bf16", seed=1001),
        # the ViT pipeline itself: 197 tokens (CLS + 14 x 14 patches), fp16,
        # padded at the front to 15 blocks of 14 (vit/benchmark.py:19-25)
        Config("vit_n197_f16", 64, 12, 197, 64, 14, 2, "f16", pre_pad=True, seed=1005),
        Config("roberta_bf16", 32, 12, 512, 64, 32, 2, "bf16", mask_min_len=128, seed=1002),
        Config("dit_bf16", 32, 16, 1024, 72, 32, 3, "bf16", seed=1003),
        # the DiT pipeline's default precision (dit/pipeline.py:147-159 loads
        # the model without a dtype): fp32 inputs, fused FFMA kernel
        Config("dit_f32", 32, 16, 1024, 72, 32, 3, "f32", seed=1003),
        Config("long4k_bf16", 4, 16, 4096, 128, 64, 2, "bf16", scaled=False, seed=1004),
        Config("long16k_bf16", 4, 16, 16384, 128, 128, 2, "bf16", scaled=False, seed=1004),
        Config("long64k_bf16", 4, 16, 65536, 128, 256, 2, "bf16", scaled=False, seed=1004),
        # BART-base encoder layers at the lengths bart/benchmark.py:42 evaluates
        # (batch 4, 12 heads of 64, (b, T) per length), with a float key-padding
        # mask (bart/model.py:145-152): valid length uniform in [N/2, N]
        Config("bart1k_bf16", 4, 12, 1024, 64, 32, 3, "bf16", mask_min_len=512, seed=1006),
        Config("bart2k_bf16", 4, 12, 2048, 64, 32, 2, "bf16", mask_min_len=1024, seed=1007),
        Config("bart4k_bf16", 4, 12, 4096, 64, 64, 2, "bf16", mask_min_len=2048, seed=1008),
        Config("bart8k_bf16", 4, 12, 8192, 64, 64, 2, "bf16", mask_min_len=4096, seed=1009),
        Config("long4k_e4m3", 4, 16, 4096, 128, 64, 2, "e4m3", scaled=False, seed=1004),
        Config("long16k_e4m3", 4, 16, 16384, 128, 128, 2, "e4m3", scaled=False, seed=1004),
        Config("long64k_e4m3", 4, 16, 65536, 128, 256, 2, "e4m3", scaled=False, seed=1004),
    ]
}

# the configuration BASELINE's headline metric is quoted on
NORTH_STAR = "long16k_bf16"

TORCH_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16,
                "e4m3": torch.float8_e4m3fn}
E4M3_MAX = 448.0


def make_inputs(cfg: Config, device="cpu", seed: int | None = None):
    """Seeded q, k, v (E, H, N, D) in cfg.dtype, the mask, and e4m3 scales.

    Returns (q, k, v, mask, scales); ``scales`` is None except for e4m3, where
    it is (q_scale, k_scale, v_scale), each (E, H) fp32 = absmax / 448 per
    head, and q/k/v hold the quantised values.
    """
    g = torch.Generator(device=device).manual_seed(cfg.seed if seed is None else seed)
    shape = (cfg.E, cfg.H, cfg.N, cfg.D)
    q = torch.randn(shape, generator=g, device=device)
    k = torch.randn(shape, generator=g, device=device)
    v = torch.randn((cfg.E, cfg.H, cfg.N, cfg.dv), generator=g, device=device)
    if cfg.scaled:
        s = 1.0 / math.sqrt(cfg.D)
        q, k, v = q * s, k * s, v * s
    mask = None
    if cfg.mask_min_len is not None:
        lens = torch.randint(cfg.mask_min_len, cfg.N + 1, (cfg.E,), generator=g, device=device)
        mask = torch.arange(cfg.N, device=device)[None, :] < lens[:, None]
    if cfg.dtype == "e4m3":
        qq, qs = quantize_e4m3(q)
        kq, ks = quantize_e4m3(k)
        vq, vs = quantize_e4m3(v)
        return qq, kq, vq, mask, (qs, ks, vs)
    dt = TORCH_DTYPES[cfg.dtype]
    return q.to(dt), k.to(dt), v.to(dt), mask, None


def quantize_e4m3(x: torch.Tensor):
    """Per-(e, h) absmax scaling into float8 e4m3: x ~= q.float() * scale."""
    amax = x.abs().amax(dim=(-1, -2)).clamp_min(1e-12)
    scale = (amax / E4M3_MAX).float()
    q = (x / scale[..., None, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q, scale


def dequantize_e4m3(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale[..., None, None]
