"""Host-side behaviour of the MonarchAttention module (no GPU needed)."""
import pytest
import torch

from monarch_attention_b200 import MonarchAttention, PadType, monarch_attention


def test_padtype_values_match_reference():
    assert PadType("pre") == "pre" and PadType("post") == "post"
    assert [p.value for p in PadType] == ["pre", "post"]


def test_constructor_surface():
    m = MonarchAttention(14, 2, PadType.pre)
    assert (m.block_size, m.num_steps, m.pad_type) == (14, 2, "pre")
    # the reference's impl names are accepted
    MonarchAttention(14, 2, PadType.pre, impl="torch")
    MonarchAttention(14, 2, PadType.pre, impl="triton")
    with pytest.raises(ValueError):
        MonarchAttention(14, 2, PadType.pre, impl="bogus")


def test_cpu_tensors_are_rejected_not_computed():
    q = torch.randn(1, 2, 32, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        MonarchAttention(8, 2, PadType.post)(q, q, q)


def test_shape_and_dtype_checks():
    q = torch.randn(1, 2, 32, 16)
    with pytest.raises(ValueError):
        monarch_attention(q, q[:, :1], q, None, 2, 8, False)
    with pytest.raises(TypeError):
        monarch_attention(q, q.half(), q, None, 2, 8, False)
    with pytest.raises(ValueError):
        monarch_attention(q[0], q[0], q[0], None, 2, 8, False)
