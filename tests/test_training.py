"""Backward pass.  The gradient checker -- a torch restatement of the
reference forward (oracle/ma_grad_oracle.py) -- is pinned to the reference's
own outputs and gradients (tests/golden, tests/golden/grad); the CUDA
backward (ma_bwd, through MonarchAttentionFunction) is compared with the
reference fixtures and with autograd over the checker on the GPU."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_paths
from gen_golden import load_case
import monarch_attention_b200 as mab
from monarch_attention_b200 import MonarchAttention, PadType, monarch_attention
from oracle.ma_grad_oracle import torch_forward

GRAD_DIR = os.path.join(GOLDEN, "grad")
TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def grad_paths():
    return sorted(glob.glob(os.path.join(GRAD_DIR, "*.npz")))


def tensors(c, dev="cpu"):
    dt = TORCH_DT[c["meta"]["dtype"]]
    q, k, v = (torch.from_numpy(c[n]).to(dev, dt) for n in ("q", "k", "v"))
    mask = None if "mask" not in c else torch.from_numpy(c["mask"]).to(dev)
    return q, k, v, mask


@pytest.mark.parametrize("path", golden_paths(), ids=lambda p: os.path.basename(p)[:-4])
def test_torch_forward_matches_reference_output(path):
    """Same operations and rounding points as ma/ma_torch.py: on CPU the
    restatement reproduces the reference's own output (16-bit: within 2
    output ulps)."""
    c = load_case(path)
    m = c["meta"]
    q, k, v, mask = tensors(c)
    out = torch_forward(q, k, v, mask, m["T"], m["B"], m["pre_pad"]).float().numpy()
    ref = c["out_ref"]
    scale = float(np.abs(ref).max())
    tol = 1e-6 * scale if m["dtype"] == "f32" else 2 * 2.0 ** -8 * scale
    assert np.abs(out - ref).max() <= tol


@pytest.mark.parametrize("path", grad_paths(), ids=lambda p: os.path.basename(p)[:-4])
def test_torch_forward_gradients_match_reference(path):
    """d<out, g>/d(q, k, v) of the restatement equals the reference's
    autograd gradients (fixtures generated from the reference itself)."""
    c = load_case(path)
    m = c["meta"]
    q, k, v, mask = tensors(c)
    dt = TORCH_DT[m["dtype"]]
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    out = torch_forward(*leaves, mask, m["T"], m["B"], m["pre_pad"])
    g = torch.from_numpy(c["g"]).to(dt)
    grads = torch.autograd.grad(out, leaves, g)
    for name, got in zip(("dq", "dk", "dv"), grads):
        ref = c[name]
        scale = float(np.abs(ref).max())
        tol = 1e-5 * scale if m["dtype"] == "f32" else 2e-2 * scale
        err = np.abs(got.float().numpy() - ref).max()
        assert np.isfinite(got.float().numpy()).all()
        assert err <= tol, f"{name}: max|err|={err:.3g} (max|ref|={scale:.3g})"


def test_torch_forward_directional_derivative():
    """<grad, d> against a central difference along a random direction d.
    The algorithm casts matmul outputs to fp32 (ma_torch.py:11, 27, 39, 56),
    so the check runs in fp32 with a step well above its rounding."""
    g = torch.Generator().manual_seed(3)
    E, H, N, D, B = 1, 2, 30, 8, 4
    x = [torch.randn(E, H, N, D, generator=g) / 2 for _ in range(3)]
    d = [torch.randn(E, H, N, D, generator=g) for _ in range(3)]
    w = torch.randn(E, H, N, D, generator=g)
    mask = torch.ones(E, N, dtype=torch.bool)
    mask[0, 23:] = False

    def f(q, k, v):
        return (torch_forward(q, k, v, mask, 3, B, True) * w).sum()

    leaves = [t.clone().requires_grad_(True) for t in x]
    grads = torch.autograd.grad(f(*leaves), leaves)
    analytic = sum((gr * dd).sum() for gr, dd in zip(grads, d)).item()
    h = 1e-2
    with torch.no_grad():
        fp = f(*[a + h * b for a, b in zip(x, d)]).item()
        fm = f(*[a - h * b for a, b in zip(x, d)]).item()
    numeric = (fp - fm) / (2 * h)
    assert abs(analytic - numeric) <= 1e-2 * max(abs(numeric), 1e-3), (analytic, numeric)


@pytest.mark.gpu
@pytest.mark.parametrize("path", grad_paths(), ids=lambda p: os.path.basename(p)[:-4])
def test_cuda_forward_and_backward_match_reference(path, cuda_device):
    """Inputs that require gradients: the forward runs on the kernels (same
    result as without gradients) and the gradients equal the reference's."""
    c = load_case(path)
    m = c["meta"]
    dt = TORCH_DT[m["dtype"]]
    q, k, v, mask = tensors(c, cuda_device)
    with torch.no_grad():
        plain = monarch_attention(q, k, v, mask, m["T"], m["B"], m["pre_pad"])
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    out = monarch_attention(*leaves, mask, m["T"], m["B"], m["pre_pad"])
    assert out.requires_grad and torch.equal(out.detach(), plain)
    out.backward(torch.from_numpy(c["g"]).to(cuda_device, dt))
    assert mab.read_status(cuda_device) == 0
    for name, t in zip(("dq", "dk", "dv"), leaves):
        ref = c[name]
        scale = float(np.abs(ref).max())
        tol = 1e-4 * scale if m["dtype"] == "f32" else 2e-2 * scale
        err = np.abs(t.grad.float().cpu().numpy() - ref).max()
        assert err <= tol, f"{name}: max|err|={err:.3g} (max|ref|={scale:.3g})"


@pytest.mark.gpu
def test_module_trains(cuda_device):
    """A few SGD steps through the module lower a regression loss (the BART
    fine-tuning use: gradients reach the projections feeding q, k, v)."""
    torch.manual_seed(5)
    E, N, H, D = 2, 64, 2, 16
    x = torch.randn(E, N, H * D, device=cuda_device)
    target = torch.randn(E, N, H * D, device=cuda_device)
    proj = torch.nn.Linear(H * D, 3 * H * D, device=cuda_device)
    attn = MonarchAttention(8, 2, PadType.post)
    opt = torch.optim.SGD(proj.parameters(), lr=0.5)
    losses = []
    for _ in range(5):
        q, k, v = (t.view(E, N, H, D).permute(0, 2, 1, 3) for t in proj(x).chunk(3, dim=-1))
        o = attn(q, k, v).permute(0, 2, 1, 3).reshape(E, N, H * D)
        loss = ((o - target) ** 2).mean()
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in proj.parameters())


@pytest.mark.gpu
def test_gradients_refuse_out_argument(cuda_device):
    q = torch.randn(1, 1, 16, 8, device=cuda_device, requires_grad=True)
    with pytest.raises(ValueError, match="out="):
        monarch_attention(q, q, q, None, 2, 4, False, out=torch.empty(1, 1, 16, 8, device=cuda_device))


# The CUDA backward against autograd over the checker (same device, same
# inputs): masks (bool, float), front and back padding, T = 1, 2, 3, Dv != D,
# and the BART / RoBERTa / long shapes reduced to a few heads.
BWD_CASES = [
    ("t2_b16_f32", dict(E=2, H=2, N=256, D=64, Dv=64, B=16, T=2, pre=False, mask=None), "f32"),
    ("t3_prepad_mask_f32", dict(E=2, H=1, N=197, D=64, Dv=64, B=14, T=3, pre=True,
                                mask="bool"), "f32"),
    ("t1_postpad_dv_f32", dict(E=1, H=2, N=100, D=32, Dv=48, B=16, T=1, pre=False, mask=None),
     "f32"),
    ("roberta_mask_f32", dict(E=2, H=2, N=512, D=64, Dv=64, B=32, T=2, pre=False,
                              mask="float"), "f32"),
    ("bart2k_mask_f32", dict(E=1, H=2, N=2048, D=64, Dv=64, B=32, T=2, pre=False,
                             mask="float"), "f32"),
    ("long4k_f32", dict(E=1, H=1, N=4096, D=128, Dv=128, B=64, T=2, pre=False, mask=None),
     "f32"),
    ("roberta_mask_bf16", dict(E=2, H=2, N=512, D=64, Dv=64, B=32, T=2, pre=False,
                               mask="float"), "bf16"),
    ("dit_f16", dict(E=1, H=2, N=1024, D=72, Dv=72, B=32, T=3, pre=False, mask=None), "f16"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("name,sh,dt", BWD_CASES, ids=[c[0] for c in BWD_CASES])
def test_cuda_backward_matches_autograd_of_the_checker(name, sh, dt, cuda_device):
    g = torch.Generator(device="cpu").manual_seed(31)
    E, H, N, D, Dv = sh["E"], sh["H"], sh["N"], sh["D"], sh["Dv"]
    s = 1.0 / np.sqrt(D)
    q, k = (torch.randn(E, H, N, D, generator=g) * s for _ in range(2))
    v = torch.randn(E, H, N, Dv, generator=g) * s
    w = torch.randn(E, H, N, Dv, generator=g)
    mask = None
    if sh["mask"] is not None:
        lens = torch.randint(N // 3, N, (E,), generator=g)
        mask = torch.arange(N)[None, :] < lens[:, None]
        if sh["mask"] == "float":
            mask = mask.float()
        mask = mask.to(cuda_device)
    tdt = TORCH_DT[dt]
    q, k, v, w = (t.to(cuda_device, tdt) for t in (q, k, v, w))
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    out = monarch_attention(*leaves, mask, sh["T"], sh["B"], sh["pre"])
    out.backward(w)
    assert mab.read_status(cuda_device) == 0
    ref_leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    ref_out = torch_forward(*ref_leaves, mask, sh["T"], sh["B"], sh["pre"])
    ref = torch.autograd.grad(ref_out, ref_leaves, w)
    for gname, got, r in zip(("dq", "dk", "dv"), leaves, ref):
        r = r.float()
        scale = float(r.abs().max())
        tol = (1e-4 if dt == "f32" else 3e-2) * scale
        err = float((got.grad.float() - r).abs().max())
        assert torch.isfinite(got.grad).all()
        assert err <= tol, f"{name} {gname}: max|err|={err:.3g} (max|ref|={scale:.3g})"


def test_backward_abi_rejects_on_the_host():
    """ma_bwd refuses bad parameters before any CUDA call (no GPU needed)."""
    import ctypes
    from monarch_attention_b200 import _lib
    lib = mab.load_library()
    bp = _lib.MaBwdParams()
    assert lib.ma_bwd(ctypes.byref(bp), None) != 0  # forward block unset: invalid
    f = bp.fwd
    f.E, f.H, f.N, f.D, f.Dv = 1, 1, 64, 32, 32
    f.block_size, f.num_steps = 8, 2
    f.dtype = f.out_dtype = _lib.DTYPE_E4M3
    f.out_dtype = _lib.DTYPE_BF16
    assert lib.ma_bwd(ctypes.byref(bp), None) == 3  # e4m3: no gradients
    f.dtype = f.out_dtype = _lib.DTYPE_BF16
    assert lib.ma_bwd_workspace_bytes(ctypes.byref(bp)) > 0
    assert lib.ma_bwd(ctypes.byref(bp), None) == 1  # NULL tensors
    bp.struct_size = 4
    assert lib.ma_bwd(ctypes.byref(bp), None) == 9
