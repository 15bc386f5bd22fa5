"""Model integration: tree-verify attention inside a Hugging Face Llama model.

The reference verifies EAGLE draft trees by patching ``LlamaAttention.forward``
for the duration of a verify step (``ragged_eagle_context``,
scripts/w4a16_e2e.py:1370-1610): the patched forward projects q/k/v, applies
RoPE, appends to the KV cache, expands K/V with ``repeat_kv`` and runs the
prefix pass (aten flash SDPA) plus the ancestor pass merged by log-sum-exp.
It recovers the tree's parent array from EAGLE's ``[1, 1, N, N]`` tree mask and
the tokens' depths (scripts/w4a16_e2e.py:999-1019).

Here the same hook is an attention function registered with transformers'
attention interface (``ALL_ATTENTION_FUNCTIONS``), so the model's own forward
(projections, RoPE, cache update, o_proj) is untouched and only the attention
call changes: :func:`tree_verify_attention` on the query and the cache-updated
``[B, Hkv, L+N, D]`` keys/values, without ``repeat_kv`` and without layout
copies. :func:`ragged_tree_context` switches a model to it for the verify step
and back afterwards; outside a verify step (``verify_flag["in_tree_verify"]``
false) the model's previous attention implementation runs.

Functions:
  parents_from_tree_mask(tree_mask, depths=None)  EAGLE mask -> int32 parents
  ragged_tree_context(model, branching_factor, max_depth, ...)  context manager
"""
from __future__ import annotations

import contextlib
import math
from typing import Dict, Optional

import torch

ATTN_NAME = "qattention_tree"

# per-process verify state read by the registered attention function
_STATE: Dict[str, object] = {"active": False}


def parents_from_tree_mask(tree_mask: torch.Tensor, depths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Parent array (int32 ``[N]``, root self-loop) of a draft tree given its ancestor mask.

    ``tree_mask``: ``[1, 1, N, N]`` or ``[N, N]``, nonzero where token i may attend to
    token j (itself and its ancestors: EAGLE's convention, read with ``.bool()`` as in
    scripts/w4a16_e2e.py:1001). ``depths``: depth of every token (EAGLE's
    ``tree_position_ids``, any shape with N leading entries after squeezing); when
    omitted, a token's depth is its number of ancestors (row sum - 1).
    parents[i] = the visible j with depth[j] = depth[i] - 1; parents[0] = 0.
    """
    m = tree_mask
    while m.dim() > 2:
        m = m[0]
    m = m.bool()
    N = m.shape[0]
    if depths is None:
        d = m.sum(1).to(torch.int64) - 1
    else:
        d = depths.reshape(-1)[:N].to(device=m.device, dtype=torch.int64)
    match = (d.unsqueeze(0) == (d - 1).unsqueeze(1)) & m
    parents = match.to(torch.int32).argmax(dim=1).to(torch.int32)
    if N:
        parents[0] = 0
    return parents


def _tree_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """Attention-interface function: tree-verify attention, or the saved implementation
    outside a verify step. Returns ``([B, N, Hq, D], None)`` like the interface's others."""
    st = _STATE
    flag = st.get("verify_flag")
    if not st["active"] or (flag is not None and not flag.get("in_tree_verify", False)):
        return st["fallback"](module, query, key, value, attention_mask, scaling=scaling, dropout=dropout, **kwargs)
    from .ragged_attn import tree_verify_attention

    D = query.shape[-1]
    if scaling is not None and not math.isclose(float(scaling), D ** -0.5, rel_tol=1e-6):
        raise ValueError(f"tree-verify attention uses scale 1/sqrt(D); the model asked for {scaling}")
    parents = st.get("tree_parents")
    if flag is not None and flag.get("tree_parents") is not None:
        parents = flag["tree_parents"]
    plan = None
    if parents is not None:
        # every layer of the step shares the tree: plan its tiles once (per tensor and version)
        from .ragged_attn import plan_tree_parents
        B, N = query.shape[0], query.shape[2]
        pk = (id(parents), parents._version, B, N, str(query.device))
        plans = st.setdefault("plans", {})
        if pk not in plans:
            plans.clear()
            plans[pk] = plan_tree_parents(parents, B, st["max_depth"], device=query.device)
        plan = plans[pk]
    out = tree_verify_attention(query, key, value, st["branching"], st["max_depth"], tree_parents=parents,
                                plan=plan)
    st["stats"]["n"] += 1
    return out.transpose(1, 2), None  # [B, N, Hq, D] (contiguous underneath)


def _register() -> None:
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    if ATTN_NAME not in ALL_ATTENTION_FUNCTIONS:
        ALL_ATTENTION_FUNCTIONS.register(ATTN_NAME, _tree_attention)


def _interface(name: str):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    if name in (None, "eager"):
        from transformers.models.llama.modeling_llama import eager_attention_forward
        return eager_attention_forward
    return ALL_ATTENTION_FUNCTIONS[name]


@contextlib.contextmanager
def ragged_tree_context(model, branching_factor: int, max_depth: int,
                        tree_parents: Optional[torch.Tensor] = None,
                        verify_flag: Optional[Dict[str, object]] = None):
    """Run the model's attention as tree-verify attention inside the ``with`` block.

    Counterpart of the reference's ``ragged_eagle_context`` (scripts/w4a16_e2e.py:1370).
    During the block every attention layer of ``model`` attends with this library:
    each query sees all cached prefix keys plus its tree ancestors (complete
    ``branching_factor``-ary BFS tree of ``max_depth``, or ``tree_parents`` ``[N]``
    int32 with root self-loop, e.g. from :func:`parents_from_tree_mask`). The
    block's forward must feed exactly the N tree tokens after an L-token cache, with
    the tokens' positions (L + depth) as ``position_ids``; the attention mask is not
    read (the tree defines visibility). ``verify_flag`` (optional dict) gates it like
    the reference's: only when ``verify_flag["in_tree_verify"]`` is true, and
    ``verify_flag["tree_parents"]``, when set, overrides ``tree_parents``.
    Yields a dict whose ``"n"`` counts the attention calls served.
    """
    _register()
    cfg = model.config
    prev = getattr(cfg, "_attn_implementation", None)
    if prev == ATTN_NAME:
        raise RuntimeError("ragged_tree_context is already active on this model")
    saved = dict(_STATE)
    _STATE.clear()
    _STATE.update(active=True, branching=int(branching_factor), max_depth=int(max_depth),
                  tree_parents=tree_parents, verify_flag=verify_flag, fallback=_interface(prev),
                  stats={"n": 0})
    # the model builds its attention mask for the implementation name it runs under;
    # build the one the previous implementation expects (its fallback reads it)
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_NAME, ALL_MASK_ATTENTION_FUNCTIONS[prev or "eager"])
    cfg._attn_implementation = ATTN_NAME
    try:
        yield _STATE["stats"]
    finally:
        cfg._attn_implementation = prev
        _STATE.clear()
        _STATE.update(saved)
