"""Verify-step host logic on the CPU: RoPE frequencies against HF transformers' Llama-3
implementation (the rotary code the reference's Llama-3.1 model runs), tree positions,
and the C ABI's argument checks of the elementwise kernels (no GPU work)."""
import ctypes

import pytest
import torch

from qattention_b200 import _lib
from qattention_b200 import verify as vf


def test_llama31_inv_freq_matches_transformers():
    tr = pytest.importorskip("transformers")
    from transformers import modeling_rope_utils as mru
    cfg = vf.LlamaConfig()
    hf_cfg = tr.LlamaConfig(hidden_size=cfg.hidden, num_attention_heads=cfg.heads, rope_theta=cfg.rope_theta,
                            max_position_embeddings=131072,
                            rope_scaling={"rope_type": "llama3", "factor": cfg.rope_factor,
                                          "low_freq_factor": cfg.rope_low_freq_factor,
                                          "high_freq_factor": cfg.rope_high_freq_factor,
                                          "original_max_position_embeddings": cfg.rope_original_max_pos})
    ref, scaling = mru._compute_llama3_parameters(hf_cfg, "cpu")
    ours = vf.llama31_inv_freq(cfg)
    assert scaling == 1.0
    assert ours.shape == ref.shape == (cfg.head_dim // 2,)
    assert torch.allclose(ours.double(), ref.double(), rtol=1e-6, atol=0)


def test_tree_depths_bfs_levels():
    assert vf.tree_depths(2, 3).tolist() == [0, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 3]
    d = vf.tree_depths(4, 5)
    assert d.numel() == 1365 and int(d.max()) == 5 and int((d == 5).sum()) == 1024
    # parent rule of the walk: parent(a) = (a-1)//b is exactly one level up
    for b, dep in ((2, 9), (3, 4), (8, 3)):
        dd = vf.tree_depths(b, dep)
        for a in range(1, dd.numel()):
            assert dd[a] == dd[(a - 1) // b] + 1


def test_elementwise_entry_points_validate_arguments():
    L = _lib.lib()
    assert L.qa_add_rmsnorm(None, None, None, None, 4, 64, 1e-5, None) == -1       # null pointers
    assert L.qa_add_rmsnorm(16, None, 16, 16, 4, 60, 1e-5, None) == -1            # hidden % 8
    assert L.qa_add_rmsnorm(8, None, 16, 16, 4, 64, 1e-5, None) == -3             # misaligned
    assert L.qa_silu_mul(16, 16, 4, 12, None) == -1                               # F % 8
    assert L.qa_silu_mul(16, 24, 4, 16, None) == -3                               # misaligned
    assert L.qa_rope_qkv(16, 16, 16, 16, 16, 4, 2, 4, 2, 63, 0, 0, 0, None) == -1  # odd head_dim
    assert L.qa_rope_qkv(16, 16, 16, 16, 16, 4, 0, 4, 2, 64, 0, 0, 0, None) == -1  # n_per_seq
    # zero rows: valid, nothing launched
    assert L.qa_add_rmsnorm(16, None, 16, 16, 0, 64, 1e-5, None) == 0
    assert L.qa_silu_mul(16, 16, 0, 16, None) == 0
