"""Model-integration hook on the GPU: a transformers Llama verifies a draft tree.

A random-init tiny Llama (fp16) prefills a prompt into its KV cache, then runs
one verify step over N tree tokens twice from the same cache: once with its
own eager attention under the equivalent 4-D mask (prefix visible, tree
ancestors visible, positions L + depth), and once inside ragged_tree_context,
where every attention layer runs this library's tree-verify attention. The
logits must agree within the 1e-2 regime of the reference's tests. This is the
reference's EAGLE verify hook (scripts/w4a16_e2e.py:1370-1610) with the parents
recovered from the tree mask (:999-1019).
"""
import copy

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qattention_b200 import hf_hook  # noqa: E402
from qattention_b200 import tree_mask as tm  # noqa: E402


def _model(D=64):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=D, vocab_size=512, max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).half().cuda().eval()


def _depths(parents):
    d = np.zeros(len(parents), dtype=np.int64)
    for i in range(1, len(parents)):
        d[i] = d[parents[i]] + 1
    return d


@pytest.mark.parametrize("B,L,kind", [(1, 40, "complete"), (2, 37, "complete"), (2, 50, "pruned"), (1, 0, "pruned")])
@torch.no_grad()
def test_llama_verify_step_matches_eager_masked_attention(B, L, kind):
    from transformers import DynamicCache
    model = _model()
    if kind == "complete":
        b, d = 3, 3
        tree = tm.build_tree(b, d)
    else:
        b, d = 3, 4
        tree = tm.build_pruned_tree(b, d, rng=np.random.default_rng(7))
    kp = tm.kernel_parents(tree)
    N = len(kp)
    tmask = torch.from_numpy(tm.tree_attention_mask_pruned(tree))           # [N, N] ancestors incl. self
    depth = torch.from_numpy(_depths(kp))
    g = torch.Generator().manual_seed(B * 100 + L)
    cache = DynamicCache(config=model.config)
    if L:
        model(torch.randint(0, 512, (B, L), generator=g).cuda(), past_key_values=cache, use_cache=True)
    tokens = torch.randint(0, 512, (B, N), generator=g).cuda()
    pos = (L + depth).cuda()[None].expand(B, N)

    mask = torch.full((B, 1, N, L + N), float("-inf"), dtype=torch.float16, device="cuda")
    mask[..., :L] = 0
    mask[..., L:] = torch.where(tmask, 0.0, float("-inf")).half().cuda()
    ref = model(tokens, attention_mask=mask, position_ids=pos, past_key_values=copy.deepcopy(cache),
                use_cache=True).logits.float()

    parents = None
    if kind == "pruned":  # recovered from the EAGLE-style mask, as the reference's hook does
        parents = hf_hook.parents_from_tree_mask(tmask[None, None].float().cuda(), depth.cuda())
        assert parents.tolist() == kp.tolist()
    flag = {"in_tree_verify": True}
    with hf_hook.ragged_tree_context(model, b, d, tree_parents=parents, verify_flag=flag) as stats:
        out = model(tokens, position_ids=pos, past_key_values=copy.deepcopy(cache), use_cache=True).logits.float()
    assert stats["n"] == model.config.num_hidden_layers
    assert model.config._attn_implementation == "eager"
    assert torch.isfinite(out).all()
    err = (out - ref).abs().max().item()
    assert torch.allclose(out, ref, atol=1e-2, rtol=1e-2), f"max |logit diff| {err:.3e}"
