"""The allocation-free entry point ma_fwd_noalloc against ma_fwd.

ma_fwd_noalloc exists for callers that cannot allocate device memory on the
path that runs the attention (a runtime that owns the memory pool, a serving
loop with a fixed device-memory budget): it takes only q / k / v / out and runs
the tcgen05 kernel on a scratch array compiled into the library.  This file
calls it through the C ABI, twice in a row on different inputs, and checks
each result against the regular entry point on the same inputs, and one head
of the second call against the CPU oracle, within the bf16 tolerance the
other parity tests use (2e-2 * max|ref|).

It is collected last (file name) so that a run stopping at the first failure
has run every other test before it; it passes alone in a fresh process too.
"""
import ctypes

import pytest
import torch

import monarch_attention_b200 as mab
from monarch_attention_b200 import _lib
from monarch_attention_b200.configs import CONFIGS, make_inputs
from monarch_attention_b200.monarch_attention import build_params

LP_TOL = 2e-2


def noalloc_fn():
    lib = mab.load_library()
    fn = lib.ma_fwd_noalloc
    fn.argtypes = [ctypes.POINTER(_lib.MaFwdParams), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return lib, fn


@pytest.mark.gpu
@pytest.mark.parametrize("H", [3, 8])
def test_noalloc_matches_ma_fwd_twice(H, cuda_device):
    """H = 8 heads is more than the 2T + 1 = 5 slots the scratch holds: the
    kernel must then cycle through those 5 slots only."""
    lib, fn = noalloc_fn()
    cfg = CONFIGS["long16k_bf16"].with_(E=1, H=H)
    stream = torch.cuda.current_stream(cuda_device)
    for call, seed in enumerate((11, 12)):
        q, k, v, mask, _ = make_inputs(cfg, device=cuda_device, seed=seed)
        ref = mab.monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl="tc")
        out = torch.full_like(ref, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        p, keep = build_params(q, k, v, out, mask, cfg.T, cfg.B, cfg.pre_pad, _lib.IMPL_AUTO)
        p.status = status.data_ptr()
        rc = fn(ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, (rc, lib.ma_last_error_detail())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.isfinite(out.float()).all()
        scale = ref.float().abs().max().item()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= LP_TOL * scale, f"call {call}: max|err|={err:.3g}"
        if call == 1:
            # and one head directly against the CPU oracle (fp32 reference)
            from oracle.ma_oracle import monarch_attention_oracle_heads
            h = H - 1
            o = monarch_attention_oracle_heads(
                *(t[:, h:h + 1].float().cpu().numpy() for t in (q, k, v)), None, cfg.T, cfg.B,
                cfg.pre_pad, "f32")
            got = out[:, h:h + 1].float().cpu().numpy()
            oerr = float(abs(got - o).max())
            assert oerr <= LP_TOL * float(abs(o).max()), f"oracle: max|err|={oerr:.3g}"


@pytest.mark.gpu
def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    lib, fn = noalloc_fn()
    # T = 3 cycles 7 workspace slots of 12 MiB: more than the 64 MiB array
    cfg = CONFIGS["long16k_bf16"].with_(E=1, H=8, T=3)
    q = torch.empty(cfg.E, cfg.H, cfg.N, cfg.D, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty_like(q)
    p, keep = build_params(q, q, q, out, None, cfg.T, cfg.B, False, _lib.IMPL_AUTO)
    rc = fn(ctypes.byref(p), None)
    assert rc == 7  # MA_ERR_UNSUPPORTED, nothing launched
    assert b"static array holds" in lib.ma_last_error_detail()
