"""B200-native MonarchAttention forward.

Importable as ``monarch_attention_b200`` (the repository-root module of that
name loads this directory as the package).  Public surface mirrors the
reference's ``ma/monarch_attention.py`` and ``ma/ma_torch.py``.
"""
from ._lib import MonarchAttentionError, lib_path, load as load_library
from .monarch_attention import (
    MonarchAttention,
    PadType,
    build_params,
    check_status,
    monarch_attention,
    read_status,
    selected_impl,
    status_word,
)

__all__ = [
    "MonarchAttention",
    "MonarchAttentionError",
    "PadType",
    "build_params",
    "check_status",
    "lib_path",
    "load_library",
    "monarch_attention",
    "read_status",
    "selected_impl",
    "status_word",
]
