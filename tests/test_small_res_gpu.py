"""Head-resident small-block kernel (csrc/ma_small_res.cu: the head's
intermediates in shared memory, q / k / v staged per item) against the fp32
oracle, over every (R-item rows, L-item rows) tile pair of 16 / 32, head dims
64 and 128, masks, front / back padding, T = 1 / 2 / 3, bf16 and fp16, and
b * M both even and odd (the shared-memory layout's alignment).  Each case
also runs the workspace small-block kernel (MA_DISABLE_SMALL_RES=1) on the
same inputs, whose result must agree within the same tolerance.
Tolerances as in test_parity_gpu.py (bf16 / fp16 within 2e-2 * max|ref| of
the fp32 reference on the same rounded inputs)."""
import numpy as np
import pytest
import torch

import monarch_attention_b200 as mab
from monarch_attention_b200 import monarch_attention
from monarch_attention_b200.configs import CONFIGS, make_inputs
from oracle.ma_oracle import monarch_attention_oracle_heads

pytestmark = pytest.mark.gpu

LP_TOL = 2e-2

# (name, base config, overrides)
CASES = [
    ("vit", "vit_bf16", dict(E=2, H=3)),
    ("vit197_prepad_f16", "vit_n197_f16", dict(E=2, H=2)),              # front padding
    ("vit_T1", "vit_bf16", dict(E=1, H=2, T=1)),                        # final R-step first
    ("vit_T3_mask", "vit_bf16", dict(E=2, H=2, T=3, mask_min_len=100)),
    ("roberta", "roberta_bf16", dict(E=2, H=2)),
    ("roberta_T3_f16", "roberta_bf16", dict(E=1, H=2, T=3, dtype="f16")),
    ("b16_M32", "roberta_bf16", dict(E=1, H=2, N=512, B=16, mask_min_len=200)),
    ("b17_M17_odd", "roberta_bf16", dict(E=1, H=2, N=280, B=17, mask_min_len=140)),
    ("b17_M12", "roberta_bf16", dict(E=2, H=2, N=204, B=17, mask_min_len=100)),
    ("d128_N60", "long4k_bf16", dict(E=2, H=2, N=60, B=16, scaled=True)),
    ("d128_N240", "long4k_bf16", dict(E=1, H=2, N=240, B=16, scaled=True)),
    ("ragged_postpad", "vit_bf16", dict(E=2, H=2, N=190)),
]


def _oracle(q, k, v, mask, cfg):
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    mn = None if mask is None else mask.cpu().numpy()
    return monarch_attention_oracle_heads(qn, kn, vn, mn, cfg.T, cfg.B, cfg.pre_pad, "f32")


@pytest.mark.parametrize("name,base,over", CASES, ids=[c[0] for c in CASES])
def test_small_res_against_oracle(name, base, over, cuda_device, monkeypatch):
    cfg = CONFIGS[base].with_(**over)
    assert cfg.B <= 32 and cfg.M <= 32
    q, k, v, mask, _ = make_inputs(cfg, device="cpu")
    dev = [t.to(cuda_device) for t in (q, k, v)]
    m = None if mask is None else mask.to(cuda_device)
    assert mab.selected_impl(*dev, m, cfg.T, cfg.B, cfg.pre_pad, impl="small") == "small"
    out = monarch_attention(*dev, m, cfg.T, cfg.B, cfg.pre_pad, impl="small")
    torch.cuda.synchronize()
    assert mab.read_status(cuda_device) == 0
    ref = _oracle(q, k, v, mask, cfg)
    tol = LP_TOL * float(np.abs(ref).max())
    got = out.float().cpu().numpy()
    err = np.abs(got - ref).max()
    assert np.isfinite(got).all()
    assert err <= tol, f"{name}: max|err|={err:.3g} > {tol:.3g}"
    # the workspace kernel on the same inputs
    monkeypatch.setenv("MA_DISABLE_SMALL_RES", "1")
    out_ws = monarch_attention(*dev, m, cfg.T, cfg.B, cfg.pre_pad, impl="small")
    torch.cuda.synchronize()
    d = (out_ws.float() - out.float()).abs().max().item()
    assert d <= tol, f"{name}: resident vs workspace kernel differ by {d:.3g}"


def test_small_res_strided_views(cuda_device):
    """Inputs as permuted (E, N, H, D) views and the output written into a
    permuted view: the same result as contiguous tensors, bit for bit."""
    g = torch.Generator(device="cpu").manual_seed(5)
    E, N, H, D, b = 2, 196, 3, 64, 14
    proj = [(torch.randn(E, N, H * D, generator=g) / 8).to(cuda_device, torch.bfloat16)
            for _ in range(3)]
    q, k, v = (t.view(E, N, H, D).permute(0, 2, 1, 3) for t in proj)
    o_buf = torch.full((E, N, H * D), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    o_view = o_buf.view(E, N, H, D).permute(0, 2, 1, 3)
    monarch_attention(q, k, v, None, 2, b, False, impl="small", out=o_view)
    ref = monarch_attention(q.contiguous(), k.contiguous(), v.contiguous(), None, 2, b, False,
                            impl="small")
    torch.cuda.synchronize()
    assert torch.equal(o_buf.view(E, N, H, D).permute(0, 2, 1, 3), ref)


def test_small_res_deterministic(cuda_device):
    cfg = CONFIGS["roberta_bf16"].with_(E=2, H=2)
    q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)
    a = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl="small")
    b = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl="small")
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("name,base,over", [
    ("roberta", "roberta_bf16", dict(E=2, H=3)),
    ("roberta_T3_f16", "roberta_bf16", dict(E=1, H=2, T=3, dtype="f16")),
    ("b17_M12", "roberta_bf16", dict(E=2, H=2, N=204, B=17, mask_min_len=100)),
    ("b20_M10_prepad", "roberta_bf16", dict(E=1, H=2, N=195, B=20, pre_pad=True)),
], ids=lambda x: x if isinstance(x, str) else None)
def test_small_res_warp_pairs_match_single_warps(name, base, over, cuda_device, monkeypatch):
    """The 16-warp layout (a warp pair shares the staged k / v / q tiles of
    an R item and takes one 16-row half each) computes every row exactly as
    the 8-warp layout does: the same bits."""
    cfg = CONFIGS[base].with_(**over)
    q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)

    def run():
        return monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl="small")

    pairs = run()
    monkeypatch.setenv("MA_SMALL_RES_PAIRS", "0")
    single = run()
    torch.cuda.synchronize()
    assert mab.read_status(cuda_device) == 0
    assert torch.equal(pairs, single)
