"""Parity of the CUDA path (through the C ABI) with the CPU oracle and with the
reference's own outputs (golden fixtures).

Tolerances (from the task's north star): fp32 within 1e-4 max-abs of the
fp32 reference; bf16 / fp16 within 2e-2 * max|ref| of the fp32 reference run
on the same (rounded) inputs; e4m3 against the fp32 oracle on the
dequantised inputs within E4M3_TOL * max|ref| (stated bound).
"""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import golden_paths
from gen_golden import load_case
import monarch_attention_b200 as mab
from monarch_attention_b200 import MonarchAttention, PadType, monarch_attention
from monarch_attention_b200.configs import CONFIGS, dequantize_e4m3, make_inputs
from oracle.ma_oracle import monarch_attention_oracle, monarch_attention_oracle_heads

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
LP_TOL = 2e-2
E4M3_TOL = 6e-2
TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def tol_for(dtype, ref):
    scale = float(np.abs(ref).max())
    return F32_TOL if dtype == "f32" else LP_TOL * scale


def to_dev(a, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(TORCH_DT[dtype])


def check_status(dev):
    assert mab.read_status(dev) == 0


# ---------------------------------------------------------------------------
# golden fixtures (outputs of the reference itself)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("impl", ["auto", "generic", "small"])
@pytest.mark.parametrize("path", golden_paths(), ids=lambda p: os.path.basename(p)[:-4])
def test_golden(path, impl, cuda_device):
    c = load_case(path)
    m = c["meta"]
    dt = m["dtype"]
    if impl == "small" and not (m["B"] <= 32 and -(-m["N"] // m["B"]) <= 32
                                and m["D"] == m["Dv"] and m["D"] % 8 == 0):
        pytest.skip("outside the small-block kernel's shapes")
    q, k, v = (to_dev(c[n], dt, cuda_device) for n in ("q", "k", "v"))
    mask = None if "mask" not in c else torch.from_numpy(c["mask"]).to(cuda_device)
    out = monarch_attention(q, k, v, mask, m["T"], m["B"], m["pre_pad"], impl=impl)
    torch.cuda.synchronize()
    check_status(cuda_device)
    got = out.float().cpu().numpy()
    ref32 = c["out_ref_f32"]
    assert out.dtype == q.dtype and out.shape == (m["E"], m["H"], m["N"], m["Dv"])
    assert np.isfinite(got).all()
    err = np.abs(got - ref32).max()
    assert err <= tol_for(dt, ref32), f"max|err|={err:.3g}"


# ---------------------------------------------------------------------------
# the benchmark configs, reduced to a few heads (oracle in seconds)
# ---------------------------------------------------------------------------
SMALL = {
    "cfg0_f32": dict(),
    "vit_bf16": dict(E=2, H=2),
    "vit_n197_f16": dict(E=2, H=2),
    "roberta_bf16": dict(E=3, H=2),
    "dit_bf16": dict(E=1, H=2),
    "dit_f32": dict(E=1, H=2),
    "long4k_bf16": dict(E=1, H=2),
    "long16k_bf16": dict(E=1, H=1),
    "long64k_bf16": dict(E=1, H=1),
}


def oracle_for(q, k, v, mask, cfg, dt):
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    mn = None if mask is None else mask.cpu().numpy()
    return monarch_attention_oracle_heads(qn, kn, vn, mn, cfg.T, cfg.B, cfg.pre_pad, dt)


@pytest.mark.parametrize("impl", ["auto", "generic", "small"])
@pytest.mark.parametrize("name", list(SMALL))
def test_config_small(name, impl, cuda_device):
    cfg = CONFIGS[name].with_(**SMALL[name])
    if impl == "small" and (cfg.B > 32 or cfg.M > 32):
        pytest.skip("outside the small-block kernel's shapes")
    q, k, v, mask, _ = make_inputs(cfg, device="cpu")
    out = monarch_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                            None if mask is None else mask.to(cuda_device),
                            cfg.T, cfg.B, cfg.pre_pad, impl=impl)
    torch.cuda.synchronize()
    check_status(cuda_device)
    ref = oracle_for(q, k, v, mask, cfg, "f32")
    got = out.float().cpu().numpy()
    err = np.abs(got - ref).max()
    assert err <= tol_for(cfg.dtype, ref), f"{name}/{impl}: max|err|={err:.3g}"


# ---------------------------------------------------------------------------
# full-size configs: every head computed, a sample of heads checked exactly
# ---------------------------------------------------------------------------
FULL = ["cfg0_f32", "dit_f32", "vit_bf16", "vit_n197_f16", "roberta_bf16", "dit_bf16", "long4k_bf16",
        "long16k_bf16", "long64k_bf16", "bart1k_bf16", "bart2k_bf16", "bart4k_bf16",
        "bart8k_bf16"]


@pytest.mark.parametrize("name", FULL)
def test_config_full_size(name, cuda_device):
    cfg = CONFIGS[name]
    q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)
    out = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert torch.isfinite(out).all()
    # heads are independent: check the first and the last (e, h) exactly
    for e, h in ((0, 0), (cfg.E - 1, cfg.H - 1)):
        sl = (slice(e, e + 1), slice(h, h + 1))
        m = None if mask is None else mask[e:e + 1]
        ref = oracle_for(q[sl], k[sl], v[sl], m, cfg, "f32")
        got = out[sl].float().cpu().numpy()
        err = np.abs(got - ref).max()
        assert err <= tol_for(cfg.dtype, ref), f"{name} head ({e},{h}): max|err|={err:.3g}"


# ---------------------------------------------------------------------------
# interface behaviour
# ---------------------------------------------------------------------------
def test_permuted_views_match_contiguous(cuda_device):
    """Hooks pass permute(0, 2, 1, 3) views of (E, N, H, D) projections."""
    g = torch.Generator(device="cpu").manual_seed(7)
    E, N, H, D = 2, 96, 3, 32
    x = [torch.randn(E, N, H, D, generator=g).to(cuda_device, torch.bfloat16) for _ in range(3)]
    views = [t.permute(0, 2, 1, 3) for t in x]
    a = monarch_attention(*views, None, 2, 16, False)
    b = monarch_attention(*[t.contiguous() for t in views], None, 2, 16, False)
    assert torch.equal(a, b)
    assert a.is_contiguous()


@pytest.mark.parametrize("impl,shape", [("small", (2, 3, 196, 64, 14)),
                                        ("generic", (2, 3, 196, 64, 14)),
                                        ("tc", (1, 2, 16384, 128, 128)),
                                        ("tc", (1, 2, 4096, 128, 64))])
def test_caller_layout_in_and_out(impl, shape, cuda_device):
    """Projections in the callers' (E, N, H*D) layout are read through
    permuted views and the result is written straight into an (E, N, H*Dv)
    buffer (vit/model.py:93-101): no layout copy on either side."""
    E, H, N, D, b = shape
    g = torch.Generator(device="cpu").manual_seed(21)
    proj = [torch.randn(E, N, H * D, generator=g).to(cuda_device, torch.bfloat16)
            for _ in range(3)]
    if D == 64:
        proj = [t / 8 for t in proj]
    q, k, v = (t.view(E, N, H, D).permute(0, 2, 1, 3) for t in proj)
    o_buf = torch.full((E, N, H * D), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    o_view = o_buf.view(E, N, H, D).permute(0, 2, 1, 3)
    assert mab.selected_impl(q, k, v, None, 2, b, False, impl=impl) == impl
    res = monarch_attention(q, k, v, None, 2, b, False, impl=impl, out=o_view)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert res.data_ptr() == o_buf.data_ptr()
    ref = monarch_attention(q.contiguous(), k.contiguous(), v.contiguous(), None, 2, b, False,
                            impl=impl)
    assert torch.equal(o_buf.view(E, N, H, D).permute(0, 2, 1, 3), ref)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("csize", ["1", "2", "4", "8"])
def test_small_kernel_cluster_sizes(csize, dtype, cuda_device, monkeypatch):
    """The small-block kernels (mma.sync 16-bit, FFMA fp32) split a head over a
    cluster of 1, 2 or 4 CTAs; every split gives the oracle's result (masked
    RoBERTa shape, T = 3).  The head-resident kernel, which takes this shape
    in 16 bits, is switched off so the workspace kernel runs."""
    monkeypatch.setenv("MA_SMALL_CLUSTER", csize)
    monkeypatch.setenv("MA_DISABLE_SMALL_RES", "1")
    cfg = CONFIGS["roberta_bf16"].with_(E=2, H=2, T=3, dtype=dtype)
    q, k, v, mask, _ = make_inputs(cfg, device="cpu")
    out = monarch_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                            mask.to(cuda_device), cfg.T, cfg.B, cfg.pre_pad, impl="small")
    torch.cuda.synchronize()
    check_status(cuda_device)
    ref = oracle_for(q, k, v, mask, cfg, "f32")
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= tol_for(cfg.dtype, ref), f"cluster {csize}: max|err|={err:.3g}"


@pytest.mark.parametrize("T,dtype,views", [(1, "bf16", False), (3, "bf16", False),
                                           (2, "f16", True)])
def test_block256_kernel_variants(T, dtype, views, cuda_device):
    """The b = 256 tcgen05 kernel (one launch per phase; L-step split into a
    log-sum-exp pass and an accumulation pass) for T = 1 (final R-step and
    output only), T = 3 (two L rounds), fp16, and permuted (E, N, H, D)
    views in and out; one head against the oracle."""
    cfg = CONFIGS["long64k_bf16"].with_(E=1, H=1, T=T, dtype=dtype)
    q, k, v, mask, _ = make_inputs(cfg, device="cpu")
    dq, dk, dv = (t.to(cuda_device) for t in (q, k, v))
    out = None
    if views:
        E, H, N, D = dq.shape
        dq, dk, dv = (t.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3) for t in (dq, dk, dv))
        out = torch.empty(E, N, H, D, dtype=dq.dtype, device=cuda_device).permute(0, 2, 1, 3)
    assert mab.selected_impl(dq, dk, dv, None, cfg.T, cfg.B, cfg.pre_pad) == "tc"
    res = monarch_attention(dq, dk, dv, None, cfg.T, cfg.B, cfg.pre_pad, out=out)
    torch.cuda.synchronize()
    check_status(cuda_device)
    ref = oracle_for(q, k, v, None, cfg, "f32")
    err = np.abs(res.float().cpu().numpy() - ref).max()
    assert err <= tol_for(dtype, ref), f"T={T} {dtype}: max|err|={err:.3g}"


# Shapes the reference accepts that the tensor-core kernels do not take (fp32,
# Dv != D, ragged N with front padding): the automatic choice must fall back
# to a kernel that gets them right.
FALLBACK = [
    ("f32_b64", dict(E=1, H=1, N=4096, D=128, B=64, T=2, dtype="f32", scaled=False), None),
    ("dv64_b64", dict(E=1, H=1, N=4096, D=128, B=64, T=2, dtype="bf16", scaled=False, Dv=64), None),
    ("ragged_prepad_b64", dict(E=1, H=2, N=4000, D=128, B=64, T=2, dtype="bf16", scaled=False,
                               pre_pad=True), None),
]


# The persistent tcgen05 kernel's other shapes: head dim 64, b != M (tiles
# packing 4 R items of b = 32, or 2 of b = 64 next to 1 L item of M = 128),
# and key-padding masks (BART, bart/model.py:145-152: a float (E, N) mask).
# Batch row 1 of the masked cases is fully masked, batch row 0 partly.
TC_SHAPES = [
    ("mask_b128", dict(N=16384, D=128, B=128, T=2, dtype="bf16", scaled=False), "part+full"),
    ("mask_b64_d128", dict(N=4096, D=128, B=64, T=2, dtype="bf16", scaled=False), "part+full"),
    ("d64_b64_f16", dict(N=4096, D=64, B=64, T=2, dtype="f16"), None),
    ("d64_b128", dict(N=16384, D=64, B=128, T=2, dtype="bf16"), None),
    ("bart2k_b32_m64", dict(N=2048, D=64, B=32, T=2, dtype="bf16"), "part+full"),
    ("bart2k_b32_m64_t3", dict(N=2048, D=64, B=32, T=3, dtype="bf16"), "part"),
    ("bart4k_b64", dict(N=4096, D=64, B=64, T=2, dtype="bf16"), "part+full"),
    ("bart8k_b64_m128", dict(N=8192, D=64, B=64, T=2, dtype="bf16"), "part+full"),
    ("bart8k_b64_m128_f16", dict(N=8192, D=64, B=64, T=2, dtype="f16"), "part"),
]


@pytest.mark.parametrize("name,shape,masking", TC_SHAPES, ids=[c[0] for c in TC_SHAPES])
def test_tc_kernel_shapes_and_masks(name, shape, masking, cuda_device):
    cfg = CONFIGS["long4k_bf16"].with_(E=2, H=1, **shape)
    q, k, v, _m, _s = make_inputs(cfg, device="cpu")
    mask = None
    if masking is not None:
        g = torch.Generator(device="cpu").manual_seed(17)
        mask = torch.ones(cfg.E, cfg.N, dtype=torch.float32)  # float, as the BART hook passes
        n_valid = int(torch.randint(cfg.N // 4, cfg.N - 1, (1,), generator=g))
        mask[0, n_valid:] = 0.0
        mask[0, torch.randint(0, n_valid, (cfg.N // 16,), generator=g)] = 0.0  # holes
        if masking == "part+full":
            mask[1] = 0.0
    dq, dk, dv = (t.to(cuda_device) for t in (q, k, v))
    dm = None if mask is None else mask.to(cuda_device)
    assert mab.selected_impl(dq, dk, dv, dm, cfg.T, cfg.B, cfg.pre_pad) == "tc"
    out = monarch_attention(dq, dk, dv, dm, cfg.T, cfg.B, cfg.pre_pad)
    torch.cuda.synchronize()
    check_status(cuda_device)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref = oracle_for(q, k, v, mask, cfg, "f32")
    err = np.abs(got - ref).max()
    assert err <= tol_for(cfg.dtype, ref), f"{name}: max|err|={err:.3g}"


@pytest.mark.parametrize("name,shape,_", FALLBACK, ids=[c[0] for c in FALLBACK])
def test_shapes_outside_the_tensor_core_kernels(name, shape, _, cuda_device):
    """(f32 b = 64 has M = 64 > 32: neither fused kernel takes it; the
    generic kernels do.)"""
    cfg = CONFIGS["long4k_bf16"].with_(**shape)
    q, k, v, mask, _s = make_inputs(cfg, device="cpu")
    assert mab.selected_impl(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                             None if mask is None else mask.to(cuda_device),
                             cfg.T, cfg.B, cfg.pre_pad) != "tc"
    out = monarch_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                            None if mask is None else mask.to(cuda_device),
                            cfg.T, cfg.B, cfg.pre_pad)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert out.shape == (cfg.E, cfg.H, cfg.N, cfg.dv)
    ref = oracle_for(q, k, v, mask, cfg, "f32")
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= tol_for(cfg.dtype, ref), f"{name}: max|err|={err:.3g}"


def test_out_argument_is_checked(cuda_device):
    q = torch.randn(1, 2, 32, 16, device=cuda_device)
    with pytest.raises(ValueError, match="out shape"):
        monarch_attention(q, q, q, None, 2, 8, False, out=torch.empty(1, 2, 32, 8, device=cuda_device))
    with pytest.raises(TypeError, match="out dtype"):
        monarch_attention(q, q, q, None, 2, 8, False,
                          out=torch.empty(1, 2, 32, 16, dtype=torch.float16, device=cuda_device))


def test_mask_dtypes_agree(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(8)
    E, H, N, D = 2, 2, 80, 16
    q, k, v = (torch.randn(E, H, N, D, generator=g).to(cuda_device) for _ in range(3))
    mb = torch.ones(E, N, dtype=torch.bool)
    mb[0, 50:] = False
    mb[1, :7] = False
    mb = mb.to(cuda_device)
    outs = [monarch_attention(q, k, v, mb.to(dt), 2, 16, False)
            for dt in (torch.bool, torch.int64, torch.int32, torch.float32, torch.float16,
                       torch.bfloat16, torch.uint8)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = monarch_attention_oracle(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(),
                                   mb.cpu().numpy(), 2, 16, False)
    assert np.abs(outs[0].cpu().numpy() - ref).max() <= F32_TOL


def test_get_matrix_rows_sum_to_one(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(9)
    E, H, N, D = 1, 2, 64, 32
    q, k = (torch.randn(E, H, N, D, generator=g).to(cuda_device) / 4 for _ in range(2))
    A = MonarchAttention(8, 2, PadType.post).get_matrix(q, k)
    assert A.shape == (E, H, N, N) and A.dtype == torch.float32
    assert (A.sum(-1) - 1).abs().max().item() < 1e-5
    ref = monarch_attention_oracle(q.cpu().numpy(), k.cpu().numpy(),
                                   np.broadcast_to(np.eye(N, dtype=np.float32), (E, H, N, N)),
                                   None, 2, 8, False)
    assert np.abs(A.cpu().numpy() - ref).max() <= F32_TOL


def test_get_matrix_is_monarch_and_ascends(cuda_device):
    """The CUDA path's matrix has the Monarch structure (every (j, k) block
    over (l, i) is rank 1) and the variational objective does not decrease
    with the number of steps (same properties as the oracle's tests)."""
    from test_oracle import monarch_blocks, objective
    g = torch.Generator(device="cpu").manual_seed(12)
    E, H, N, D, B = 1, 4, 256, 64, 16
    q, k = (torch.randn(E, H, N, D, generator=g).to(cuda_device) / 2 for _ in range(2))
    qn, kn = q.cpu().numpy(), k.cpu().numpy()
    fs = []
    for T in (1, 2, 3, 4):
        A = MonarchAttention(B, T, PadType.post).get_matrix(q, k).cpu().numpy()
        sv = np.linalg.svd(monarch_blocks(A, B).astype(np.float64), compute_uv=False)
        assert (sv[..., 1] <= 1e-4 * sv[..., 0]).all(), T
        fs.append(objective(A, qn, kn))
    for a, b in zip(fs, fs[1:]):
        assert (b >= a - 1e-4 * np.abs(a)).all(), (a, b)


@pytest.mark.parametrize("name", ["long4k_bf16", "long16k_bf16", "long64k_bf16"])
def test_full_size_properties(name, cuda_device):
    """Size-independent checks over every head of the full-size tensor-core
    workloads: the output is linear in V (A depends on q and k only), and
    heads are independent (permuting the (e, h) heads permutes the output
    bit for bit, whatever wavefront order and workspace slots they get)."""
    cfg = CONFIGS[name]
    q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)

    def f(q_, k_, v_):
        return monarch_attention(q_, k_, v_, mask, cfg.T, cfg.B, cfg.pre_pad)

    g = torch.Generator(device=cuda_device).manual_seed(11)
    v2 = torch.randn(v.shape, generator=g, device=cuda_device).to(v.dtype)
    o1 = f(q, k, v)
    o2 = f(q, k, v2)
    o3 = f(q, k, (v.float() + v2.float()).to(v.dtype))
    torch.cuda.synchronize()
    check_status(cuda_device)
    scale = o3.float().abs().max().item()
    err = (o3.float() - o1.float() - o2.float()).abs().max().item()
    assert err <= LP_TOL * scale, f"linearity: max|err|={err:.3g} (max|out|={scale:.3g})"
    E, H = q.shape[:2]
    perm = torch.randperm(E * H, generator=torch.Generator().manual_seed(5)).to(cuda_device)

    def shuf(t):
        return t.reshape(E * H, *t.shape[2:])[perm].reshape(t.shape)

    o4 = f(shuf(q), shuf(k), shuf(v))
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert torch.equal(o4, shuf(o1))
    # a shard of a few heads (the multi-GPU split: 8 or 16 heads per GPU)
    # runs with another wavefront group size and slot count: same bits
    if mask is None:
        for lo, hi in ((0, 8), (16, 32)):
            def sl(t):
                return t.reshape(E * H, 1, *t.shape[2:])[lo:hi]

            o5 = f(sl(q), sl(k), sl(v))
            torch.cuda.synchronize()
            check_status(cuda_device)
            assert torch.equal(o5, sl(o1)), (lo, hi)


def test_module_forward_matches_function(cuda_device):
    cfg = CONFIGS["vit_bf16"].with_(E=1, H=2)
    q, k, v, _, _ = make_inputs(cfg, device=cuda_device)
    mod = MonarchAttention(cfg.B, cfg.T, PadType.post)
    assert torch.equal(mod(q, k, v), monarch_attention(q, k, v, None, cfg.T, cfg.B, False))


def test_deterministic(cuda_device):
    cfg = CONFIGS["roberta_bf16"].with_(E=2, H=2)
    q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)
    a = monarch_attention(q, k, v, mask, cfg.T, cfg.B, False)
    b = monarch_attention(q, k, v, mask, cfg.T, cfg.B, False)
    assert torch.equal(a, b)


def test_fully_masked_rows_are_finite(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(10)
    E, H, N, D = 2, 1, 64, 16
    q, k, v = (torch.randn(E, H, N, D, generator=g) for _ in range(3))
    mask = torch.ones(E, N, dtype=torch.bool)
    mask[1] = False
    mask[0, 16:32] = False
    out = monarch_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                            mask.to(cuda_device), 3, 16, False)
    ref = monarch_attention_oracle(q.numpy(), k.numpy(), v.numpy(), mask.numpy(), 3, 16, False)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= F32_TOL


def test_missing_library_fails_loudly(monkeypatch, cuda_device):
    from monarch_attention_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libmonarch_attn.so")
    q = torch.randn(1, 1, 16, 8, device=cuda_device)
    with pytest.raises(RuntimeError, match="not built"):
        monarch_attention(q, q, q, None, 2, 4, False)


# ---------------------------------------------------------------------------
# float8 e4m3 inputs with per-(e, h) scales: compared with the fp32 oracle run
# on the dequantised inputs (the quantisation error itself is not counted)
# ---------------------------------------------------------------------------
E4M3_CASES = [("long4k_e4m3", dict(E=1, H=2), "auto"),
              ("long16k_e4m3", dict(E=1, H=1), "auto"),
              ("long16k_e4m3", dict(E=1, H=1), "generic"),
              ("long16k_e4m3", dict(E=1, H=3), "tc"),
              ("long64k_e4m3", dict(E=1, H=1), "tc"),
              ("vit_bf16", dict(E=2, H=2, dtype="e4m3"), "small"),
              ("roberta_bf16", dict(E=2, H=2, dtype="e4m3"), "small")]


@pytest.mark.parametrize("name,shape,impl", E4M3_CASES,
                         ids=[f"{n}-{i}-{sh.get('H')}" for n, sh, i in E4M3_CASES])
def test_e4m3_against_dequantised_oracle(name, shape, impl, cuda_device):
    cfg = CONFIGS[name].with_(**shape)
    q, k, v, mask, scales = make_inputs(cfg, device=cuda_device)
    out = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, scales=scales, impl=impl)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert out.dtype == torch.bfloat16
    deq = [dequantize_e4m3(t, s) for t, s in zip((q, k, v), scales)]
    ref = oracle_for(*deq, mask, cfg, "f32")
    got = out.float().cpu().numpy()
    err = np.abs(got - ref).max()
    assert np.isfinite(got).all()
    assert err <= E4M3_TOL * float(np.abs(ref).max()), f"max|err|={err:.3g}"


def test_e4m3_routes_to_tensor_core_kernels(cuda_device):
    """e4m3 inputs run on the tensor-core kernels (directly, or after a bf16
    conversion for the shapes the e4m3 build does not take)."""
    for name, shape, want in [("long16k_e4m3", dict(E=1, H=1), "tc"),
                              ("long4k_bf16", dict(E=1, H=1), "tc"),
                              ("long64k_bf16", dict(E=1, H=1), "tc"),
                              ("vit_bf16", dict(E=1, H=1, dtype="e4m3"), "small"),
                              ("long4k_e4m3", dict(E=1, H=1), "tc")]:
        cfg = CONFIGS[name].with_(**shape)
        q, k, v, mask, _ = make_inputs(cfg, device=cuda_device)
        assert mab.selected_impl(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad) == want, name


@pytest.mark.parametrize("name,shape", [("long16k_e4m3", dict(E=1, H=3)),
                                        ("long4k_e4m3", dict(E=2, H=3)),
                                        ("long4k_e4m3", dict(E=2, H=2, mask_min_len=1500))])
def test_e4m3_direct_matches_conversion_route(name, shape, cuda_device, monkeypatch):
    """The persistent kernel reads e4m3 tiles itself (converted to f16 in
    shared memory, scales folded into the softmax and epilogue); the result
    agrees with the route through bf16 copies and with the oracle."""
    cfg = CONFIGS[name].with_(**shape)
    q, k, v, mask, scales = make_inputs(cfg, device=cuda_device)
    direct = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, scales=scales)
    torch.cuda.synchronize()
    check_status(cuda_device)
    monkeypatch.setenv("MA_FP8_CONVERT", "1")
    conv = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, scales=scales)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert direct.dtype == torch.bfloat16 and torch.isfinite(direct.float()).all()
    scale = float(conv.float().abs().max())
    assert float((direct.float() - conv.float()).abs().max()) <= 3e-2 * scale
    deq = [dequantize_e4m3(t, s_).cpu() for t, s_ in zip((q, k, v), scales)]
    ref = oracle_for(*deq, None if mask is None else mask.cpu(), cfg, "f32")
    err = np.abs(direct.float().cpu().numpy() - ref).max()
    assert err <= E4M3_TOL * float(np.abs(ref).max()), f"max|err|={err:.3g}"


def test_e4m3_full_size_tc(cuda_device):
    """long16k e4m3 at full size on the persistent kernel (e4m3 read directly)."""
    cfg = CONFIGS["long16k_e4m3"]
    q, k, v, mask, scales = make_inputs(cfg, device=cuda_device)
    out = monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, scales=scales)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert torch.isfinite(out.float()).all()
    for e, h in ((0, 0), (cfg.E - 1, cfg.H - 1)):
        sl = (slice(e, e + 1), slice(h, h + 1))
        deq = [dequantize_e4m3(t[sl], s_[sl]) for t, s_ in zip((q, k, v), scales)]
        ref = oracle_for(*deq, None, cfg, "f32")
        got = out[sl].float().cpu().numpy()
        err = np.abs(got - ref).max()
        assert err <= E4M3_TOL * float(np.abs(ref).max()), f"head ({e},{h}): max|err|={err:.3g}"


MATRIX_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "matrix")


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(MATRIX_DIR, "*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_get_matrix_16bit_queries_match_reference(path, cuda_device):
    """get_matrix with fp16 / bf16 queries: fp32 identity values, so y and
    the output step run in fp32 like the reference's (fixtures of the
    reference's own get_matrix, tests/golden/matrix)."""
    import json
    c = np.load(path)
    m = json.loads(str(c["meta"]))
    dt = TORCH_DT[m["dtype"]]
    q, k = (torch.from_numpy(c[n]).to(cuda_device, dt) for n in ("q", "k"))
    mask = None if "mask" not in c else torch.from_numpy(c["mask"]).to(cuda_device)
    attn = MonarchAttention(m["B"], m["T"], PadType.pre if m["pre_pad"] else PadType.post)
    A = attn.get_matrix(q, k, mask)
    torch.cuda.synchronize()
    check_status(cuda_device)
    assert A.dtype == torch.float32
    ref = c["matrix"]
    err = np.abs(A.cpu().numpy() - ref).max()
    # the same rounding points; only fp32 summation order differs
    assert err <= 1e-3 * np.abs(ref).max(), f"max|err|={err:.3g}"
