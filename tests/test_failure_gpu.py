"""Device-side failure detection on the GPU without a fault.

The persistent tcgen05 kernel bounds every wait.  MA_TEST_STALL_DEP=head,phase
makes one (head, phase) dependency need one more completed tile than its
producer phase has, so that wait runs out after MA_WAIT_TIMEOUT_NS; the kernel
must then set MA_STATUS_WAIT_TIMEOUT, stop every role (nothing traps, nothing
hangs: every other wait sees the abort flag), free its tensor memory and
return, and the Python layer must raise MonarchAttentionError (MA_ERR_DEVICE)
-- immediately with check=True, lazily at the next call, or from
check_status().  The next normal call on the same device must pass parity.
"""
import numpy as np
import pytest
import torch

import monarch_attention_b200 as mab
from monarch_attention_b200 import _lib
from monarch_attention_b200.configs import CONFIGS, make_inputs
from oracle.ma_oracle import monarch_attention_oracle_heads

pytestmark = pytest.mark.gpu

LP_TOL = 2e-2
STALL_NS = "20000000"  # 20 ms per bounded wait


def _inputs(dev, H=2, name="long16k_bf16"):
    cfg = CONFIGS[name].with_(E=1, H=H)
    q, k, v, mask, _ = make_inputs(cfg, device=dev)
    return cfg, q, k, v


def _stalled(monkeypatch, head, phase):
    monkeypatch.setenv("MA_TEST_STALL_DEP", f"{head},{phase}")
    monkeypatch.setenv("MA_WAIT_TIMEOUT_NS", STALL_NS)


@pytest.mark.parametrize("name,head,phase", [("long16k_bf16", 1, 1), ("long4k_bf16", 0, 3)])
def test_expired_wait_raises_with_check(name, head, phase, cuda_device, monkeypatch):
    mab.read_status(cuda_device)  # start clean
    cfg, q, k, v = _inputs(cuda_device, name=name)
    _stalled(monkeypatch, head, phase)
    with pytest.raises(mab.MonarchAttentionError) as ei:
        mab.monarch_attention(q, k, v, None, cfg.T, cfg.B, False, impl="tc", check=True)
    assert ei.value.code == _lib.MA_ERR_DEVICE
    assert "bounded device wait" in str(ei.value)
    # the status was cleared by the check
    assert mab.read_status(cuda_device) == 0


def test_expired_wait_raises_lazily_at_next_call(cuda_device, monkeypatch):
    mab.read_status(cuda_device)
    cfg, q, k, v = _inputs(cuda_device)
    _stalled(monkeypatch, 1, 2)
    mab.monarch_attention(q, k, v, None, cfg.T, cfg.B, False, impl="tc")  # enqueued, returns
    torch.cuda.synchronize(cuda_device)  # the kernel returned (bounded waits)
    monkeypatch.delenv("MA_TEST_STALL_DEP")
    monkeypatch.delenv("MA_WAIT_TIMEOUT_NS")
    with pytest.raises(mab.MonarchAttentionError) as ei:
        mab.monarch_attention(q, k, v, None, cfg.T, cfg.B, False, impl="tc")
    assert ei.value.code == _lib.MA_ERR_DEVICE
    # after the error the device works normally
    out = mab.monarch_attention(q, k, v, None, cfg.T, cfg.B, False, impl="tc", check=True)
    ref = monarch_attention_oracle_heads(q[:, :1].float().cpu().numpy(),
                                         k[:, :1].float().cpu().numpy(),
                                         v[:, :1].float().cpu().numpy(), None, cfg.T, cfg.B,
                                         False, "f32")
    err = float(np.abs(out[:, :1].float().cpu().numpy() - ref).max())
    assert err <= LP_TOL * float(np.abs(ref).max()), err


def test_status_bits_and_recovery_through_the_c_abi(cuda_device, monkeypatch):
    """The raw ABI: the status word holds MA_STATUS_WAIT_TIMEOUT after the
    stalled call, and the next call (same workspace, same stream) is exact."""
    import ctypes
    lib = mab.load_library()
    cfg, q, k, v = _inputs(cuda_device)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    p, keep = mab.build_params(q, k, v, out, None, cfg.T, cfg.B, False, _lib.IMPL_TC)
    nbytes = lib.ma_workspace_bytes(ctypes.byref(p))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    p.workspace, p.workspace_bytes, p.status = ws.data_ptr(), nbytes, status.data_ptr()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    _stalled(monkeypatch, 0, 1)
    assert lib.ma_fwd(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) & _lib.MA_STATUS_WAIT_TIMEOUT
    monkeypatch.delenv("MA_TEST_STALL_DEP")
    monkeypatch.delenv("MA_WAIT_TIMEOUT_NS")
    status.zero_()
    assert lib.ma_fwd(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    ref = mab.monarch_attention(q, k, v, None, cfg.T, cfg.B, False, impl="tc", check=True)
    assert torch.equal(out, ref)
