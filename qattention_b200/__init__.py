"""qattention_b200 — B200 (sm_100a) tree-verification attention.

Drop-in for QAttention's operator API (``src.ragged_attn`` / ``src.tree_mask``):

    from qattention_b200.ragged_attn import pack_inputs, ragged_attention

Kernels live in ``libqattn_b200.so`` (C ABI in ``include/qattn_b200.h``),
built in-tree by ``python -m qattention_b200.build``.
"""
from . import tree_mask  # noqa: F401
from .host_pipeline import ragged_attention_with_lse_host  # noqa: F401
from .ragged_attn import (  # noqa: F401
    build_paged_kv,
    fused_lse_merge,
    pack_inputs,
    ragged_attention,
    ragged_attention_paged,
    ragged_attention_sibling,
    ragged_attention_sibling_with_lse,
    ragged_attention_with_lse,
    ragged_attention_with_parents,
)

__version__ = "0.1.0"
