"""Model-integration hook on CPU: the parent extractor and the attention switch.

parents_from_tree_mask restates the reference's extraction from EAGLE's
[1, 1, N, N] tree mask (scripts/w4a16_e2e.py:999-1019); it is checked against
the golden pruned trees the reference generated and against complete trees.
The context manager is checked for switching a transformers Llama model's
attention implementation and back, and for passing through to the previous
implementation outside a verify step (no GPU needed for that path).
"""
import numpy as np
import pytest
import torch

from qattention_b200 import hf_hook
from qattention_b200 import tree_mask as tm


def _depths(parents):
    d = np.zeros(len(parents), dtype=np.int64)
    for i in range(1, len(parents)):
        d[i] = d[parents[i]] + 1
    return d


@pytest.mark.parametrize("b,d", [(1, 4), (2, 3), (3, 3), (4, 2)])
def test_parents_from_complete_tree_masks(b, d):
    mask = torch.from_numpy(tm.tree_attention_mask(b, d)).float()[None, None]
    par = hf_hook.parents_from_tree_mask(mask)
    expect = [0] + [(i - 1) // b for i in range(1, tm.num_tree_nodes(b, d))]
    assert par.dtype == torch.int32 and par.tolist() == expect


def test_parents_from_golden_pruned_trees(golden):
    # the masks are the reference's own tree_attention_mask_pruned outputs
    g = golden["tree_topology"]
    names = [k for k in g.files if k.startswith("pruned_b")]
    assert len(names) == 5
    for k in names:
        tree = g[k]
        mask = torch.from_numpy(g[k.replace("pruned_", "pruned_mask_")])
        kp = tm.kernel_parents(tree)
        depths = torch.from_numpy(_depths(kp))
        assert hf_hook.parents_from_tree_mask(mask[None, None].float()).tolist() == kp.tolist()
        assert hf_hook.parents_from_tree_mask(mask, depths[None]).tolist() == kp.tolist()


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=32, vocab_size=100)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_context_switches_attention_and_restores_it():
    model = _tiny_llama()
    ids = torch.randint(0, 100, (1, 12))
    ref = model(ids).logits
    flag = {"in_tree_verify": False}
    with hf_hook.ragged_tree_context(model, 2, 3, verify_flag=flag) as stats:
        assert model.config._attn_implementation == hf_hook.ATTN_NAME
        out = model(ids).logits        # outside a verify step: the previous (eager) attention
    assert model.config._attn_implementation == "eager"
    assert torch.equal(out, ref) and stats["n"] == 0
