"""Drop-in replacement for QAttention's ``src.ragged_attn`` operator API on B200.

Same function names, arguments, return values and error behaviour as the
reference module (``src/ragged_attn.py``); the work runs in the hand-written
sm_100a kernels of ``libqattn_b200.so`` through its C ABI. There is no Triton,
no dispatch to other backends and no CPU path: CPU tensors raise.

Reference entry points mirrored here (file:line in the reference project):
  pack_inputs                        src/ragged_attn.py:1054-1077
  ragged_attention                   src/ragged_attn.py:1080-1166
  ragged_attention_with_lse          src/ragged_attn.py:499-572
  ragged_attention_with_parents      src/ragged_attn.py:716-795
  ragged_attention_sibling(_with_lse) src/ragged_attn.py:1423-1556 (same math)
  fused_lse_merge                    src/ragged_attn.py:1619-1653
  ragged_attention_hybrid            src/ragged_attn.py:1851-1888
  ragged_attention_paged             src/ragged_attn.py:827-1004
  build_paged_kv                     src/ragged_attn.py:1007-1047
"""
from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Tuple

import torch

from . import _lib

_SUPPORTED = (torch.float16, torch.bfloat16)


def _dtype_code(dt: torch.dtype) -> int:
    return _lib.QA_DTYPE_F16 if dt == torch.float16 else _lib.QA_DTYPE_BF16


def _check_qkv(Q, K, V) -> None:
    # Same assertion and message as the reference (src/ragged_attn.py:1113-1116).
    assert Q.dtype in _SUPPORTED and Q.dtype == K.dtype == V.dtype, (
        f"Inputs must be fp16 or bf16 (got {Q.dtype})"
    )
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor: this library has no CPU path")
        if t.dim() != 3:
            raise ValueError(f"{name} must be [tokens, heads, head_dim], got shape {tuple(t.shape)}")


def _rowable(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` if its rows are 16-byte vectors at 16-byte aligned addresses, else a copy.

    The kernels take arbitrary token/head strides but need stride 1 along
    head_dim, token/head strides that are multiples of 8 elements and a
    16-byte aligned base pointer.
    """
    ok = (t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1])
          and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cu_and_max(cu_seqlens: torch.Tensor, max_seqlen: Optional[int], device) -> Tuple[torch.Tensor, int]:
    """cu_seqlens on the device as int32, and max_seqlen (derived on the host when None).

    Mirrors src/ragged_attn.py:1136-1142: with ``max_seqlen=None`` the offsets
    are read on the host (a device->host copy if the caller passed a CUDA
    tensor); pass ``max_seqlen`` and a device ``cu_seqlens`` to stay
    asynchronous and CUDA-graph capturable.
    """
    B = int(cu_seqlens.shape[0]) - 1
    if max_seqlen is None:
        cu_cpu = cu_seqlens.cpu()
        sl = cu_cpu.tolist()
        max_seqlen = int(max(sl[i + 1] - sl[i] for i in range(B))) if B else 1
        cu_dev = cu_cpu.to(device=device, dtype=torch.int32, non_blocking=True)
    else:
        cu_dev = cu_seqlens.to(device=device, dtype=torch.int32, non_blocking=True)
    return cu_dev.contiguous(), int(max_seqlen)


def pack_inputs(
    qs: List[torch.Tensor],
    ks: List[torch.Tensor],
    vs: List[torch.Tensor],
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Concatenate per-sequence ``[L_i, H, D]`` tensors into the packed ragged layout.

    Returns ``(Q, K, V, cu_seqlens)`` with ``cu_seqlens`` a CPU int32 tensor,
    ``cu[0] = 0`` and ``cu[i+1] = cu[i] + L_i`` (src/ragged_attn.py:1071-1077).
    """
    assert len(qs) == len(ks) == len(vs)
    B = len(qs)
    cu_seqlens = torch.zeros(B + 1, dtype=torch.int32)
    if B:
        lens = torch.tensor([q.shape[0] for q in qs], dtype=torch.int64)
        cu_seqlens[1:] = torch.cumsum(lens, 0).to(torch.int32)
    return torch.cat(qs, 0), torch.cat(ks, 0), torch.cat(vs, 0), cu_seqlens


def _ancestor(Q, K, V, cu_dev, max_seqlen, *, branching=1, max_depth=0, parents=None,
              want_lse=False, cu_kv=None, kv_offset=0, prefix_o=None, prefix_lse=None,
              out=None, lse_out=None, q_batched=None, plan=None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Launch ``qa_ancestor_attn`` on torch's current stream; returns (O, LSE or None).

    ``q_batched``: the queries as a ``[B, N, Hq, D]`` view read in place through its
    batch stride (``Q`` then only gives the packed shape ``[B*N, Hq, D]``).
    """
    total, Hq, D = Q.shape
    Hkv = K.shape[1]
    if K.shape[2] != D or V.shape[1:] != K.shape[1:]:
        raise ValueError("K/V must be [tokens, kv_heads, head_dim] matching Q's head_dim")
    if Hq % Hkv != 0:
        raise ValueError(f"query heads {Hq} must be a multiple of kv heads {Hkv}")
    if max_depth < 0:
        raise ValueError(f"max_depth must be >= 0, got {max_depth}")
    if parents is None and branching < 1:
        raise ValueError(f"branching_factor must be >= 1, got {branching}")
    Q, K, V = _rowable(Q), _rowable(K), _rowable(V)
    O = out if out is not None else torch.empty_like(Q, memory_format=torch.contiguous_format)
    LSE = lse_out
    if want_lse and LSE is None:
        LSE = torch.empty(total, Hq, dtype=torch.float32, device=Q.device)
    B = int(cu_dev.shape[0]) - 1
    a = _lib.AncestorArgs()
    a.q, a.k, a.v, a.o = Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr()
    a.lse = LSE.data_ptr() if LSE is not None else None
    a.cu_seqlens_q = cu_dev.data_ptr()
    a.cu_seqlens_kv = cu_kv.data_ptr() if cu_kv is not None else None
    a.parents = parents.data_ptr() if parents is not None else None
    a.q_stride_t, a.q_stride_h = Q.stride(0), Q.stride(1)
    if q_batched is not None:
        a.q = q_batched.data_ptr()
        a.q_stride_b, a.q_stride_t, a.q_stride_h = q_batched.stride(0), q_batched.stride(1), q_batched.stride(2)
    a.k_stride_t, a.k_stride_h = K.stride(0), K.stride(1)
    a.v_stride_t, a.v_stride_h = V.stride(0), V.stride(1)
    a.o_stride_t, a.o_stride_h = O.stride(0), O.stride(1)
    if LSE is not None:
        a.lse_stride_t, a.lse_stride_h = LSE.stride(0), LSE.stride(1)
    if prefix_o is not None:
        prefix_o = _rowable(prefix_o)
        a.prefix_o, a.prefix_lse = prefix_o.data_ptr(), prefix_lse.data_ptr()
        a.prefix_o_stride_t, a.prefix_o_stride_h = prefix_o.stride(0), prefix_o.stride(1)
        a.prefix_lse_stride_t, a.prefix_lse_stride_h = prefix_lse.stride(0), prefix_lse.stride(1)
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = B, Hq, Hkv, D
    a.kv_offset, a.branching, a.max_depth, a.max_seqlen = kv_offset, branching, max_depth, max_seqlen
    a.scale = 1.0 / math.sqrt(D)
    a.dtype = _dtype_code(Q.dtype)
    ws = None
    if plan is not None:  # plans made once for these parents (plan_parents)
        plan._check(B, max_depth, max_seqlen)
        a.workspace, a.workspace_bytes, a.workspace_planned = plan.workspace.data_ptr(), plan.nbytes, 1
    elif parents is not None:  # plan scratch of the tensor-core explicit-parent path
        need = ctypes.c_int64(0)
        _lib.check(_lib.lib().qa_ancestor_workspace_bytes(a, ctypes.byref(need)), "qa_ancestor_workspace_bytes")
        if need.value > 0:
            ws = torch.empty(need.value, dtype=torch.uint8, device=Q.device)
            a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
    _lib.check(_lib.lib().qa_ancestor_attn(a, _stream_ptr(Q.device)), "qa_ancestor_attn")
    return O, LSE


def ragged_attention(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    cu_seqlens: torch.Tensor,
    branching_factor: int,
    max_depth: int,
    max_seqlen: int = None,
) -> torch.Tensor:
    """Ancestor-sparse attention for BFS-ordered complete b-ary draft trees.

    Each query token q attends to {parent^0(q), ..., parent^max_depth(q)} with
    parent(k) = max(k-1, 0) // b, softmax scale 1/sqrt(D), fp32 accumulation.
    Q, K, V: packed ``[sum L_i, H, D]`` fp16/bf16 CUDA tensors; returns O like Q.
    """
    _check_qkv(Q, K, V)
    cu_dev, ms = _cu_and_max(cu_seqlens, max_seqlen, Q.device)
    O, _ = _ancestor(Q, K, V, cu_dev, ms, branching=branching_factor, max_depth=max_depth)
    return O


def ragged_attention_with_lse(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    cu_seqlens: torch.Tensor,
    branching_factor: int,
    max_depth: int,
    max_seqlen: int = None,
) -> tuple:
    """As :func:`ragged_attention`, also returning ``lse`` fp32 ``[sum L_i, H]``
    (natural log of the softmax denominator in scaled-score units)."""
    _check_qkv(Q, K, V)
    cu_dev, ms = _cu_and_max(cu_seqlens, max_seqlen, Q.device)
    return _ancestor(Q, K, V, cu_dev, ms, branching=branching_factor, max_depth=max_depth,
                     want_lse=True)


class ParentsPlan:
    """Tile plans of explicit-parent trees, made once by :func:`plan_parents` and
    reused by every call on the same trees (e.g. all layers of one verify step).

    Holds the device workspace with the plans, the int32 parents and cu_seqlens
    they were made from, and the batch, max_depth and max_seqlen they cover.
    """

    def __init__(self, workspace, nbytes, parents, cu, batch, max_depth, max_seqlen):
        self.workspace, self.nbytes = workspace, nbytes
        self.parents, self.cu_seqlens = parents, cu
        self.batch, self.max_depth, self.max_seqlen = batch, max_depth, max_seqlen

    def _check(self, batch, max_depth, max_seqlen):
        if (batch, max_depth, max_seqlen) != (self.batch, self.max_depth, self.max_seqlen):
            raise ValueError(f"plan made for (batch, max_depth, max_seqlen) = "
                             f"{(self.batch, self.max_depth, self.max_seqlen)}, "
                             f"called with {(batch, max_depth, max_seqlen)}")


def plan_parents(cu_seqlens: torch.Tensor, parents: torch.Tensor, max_depth: int, max_seqlen: int = None,
                 device=None) -> Optional[ParentsPlan]:
    """Plans every (sequence, 64-query tile) of explicit-parent trees on the device
    (one kernel) for reuse by :func:`ragged_attention_with_parents` /
    :func:`tree_verify_attention` calls with ``plan=``. Returns None when the
    tensor-core path does not apply (sequences over 16384 tokens, walks over 31
    steps): those calls then take the per-query walk. The plan stays valid while
    ``parents`` and ``cu_seqlens`` keep their values.
    """
    dev = torch.device(device) if device is not None else parents.device
    if dev.type != "cuda":
        raise RuntimeError("plan_parents needs a CUDA device: this library has no CPU path")
    cu_dev, ms = _cu_and_max(cu_seqlens, max_seqlen, dev)
    par = parents.to(device=dev, dtype=torch.int32).contiguous()
    a = _lib.AncestorArgs()
    a.cu_seqlens_q, a.parents = cu_dev.data_ptr(), par.data_ptr()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = int(cu_dev.shape[0]) - 1, 1, 1, 128
    a.max_depth, a.max_seqlen, a.dtype = max_depth, ms, _lib.QA_DTYPE_F16
    need = ctypes.c_int64(0)
    _lib.check(_lib.lib().qa_ancestor_workspace_bytes(a, ctypes.byref(need)), "qa_ancestor_workspace_bytes")
    if need.value == 0:
        return None
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().qa_ancestor_plan(a, _stream_ptr(dev)), "qa_ancestor_plan")
    return ParentsPlan(ws, need.value, par, cu_dev, a.batch, max_depth, ms)


def ragged_attention_with_parents(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    cu_seqlens: torch.Tensor,
    parents: torch.Tensor,
    max_depth: int,
    max_seqlen: int = None,
    plan: Optional[ParentsPlan] = None,
) -> tuple:
    """Ancestor-sparse attention over explicit (pruned / EAGLE-style) trees.

    ``parents[global_pos]`` is the sequence-local parent index; roots carry a
    self-loop ``parents[root] = root``. The walk stops at the first self-loop or
    after ``max_depth`` parent steps. A parent outside ``[0, L_i)`` also ends
    the walk (the reference reads out of bounds there). Returns (O, lse).
    ``plan``: optional :func:`plan_parents` result for these parents (skips planning).
    """
    _check_qkv(Q, K, V)
    if plan is not None:
        cu_dev, ms, par = plan.cu_seqlens, plan.max_seqlen, plan.parents
        if max_seqlen is not None and max_seqlen != ms:
            raise ValueError(f"plan made for max_seqlen {ms}, called with {max_seqlen}")
    else:
        cu_dev, ms = _cu_and_max(cu_seqlens, max_seqlen, Q.device)
        par = parents.to(device=Q.device, dtype=torch.int32, non_blocking=True).contiguous()
    if par.shape[0] != Q.shape[0]:
        raise ValueError(f"parents must have one entry per token ({Q.shape[0]}), got {par.shape[0]}")
    return _ancestor(Q, K, V, cu_dev, ms, parents=par, max_depth=max_depth, want_lse=True, plan=plan)


def ragged_attention_paged(
    Q: torch.Tensor,
    K_cache: torch.Tensor,
    V_cache: torch.Tensor,
    page_table: torch.Tensor,
    cu_seqlens: torch.Tensor,
    branching_factor: int,
    max_depth: int,
) -> torch.Tensor:
    """Ancestor-walk attention with a paged K/V cache (vLLM PagedAttention layout).

    Q: packed ``[total_tokens, H, D]``; K_cache / V_cache: ``[pages, page_size, H_kv, D]``;
    page_table: ``[B, max_pages]`` int32 (CPU or GPU), ``page_table[b, p]`` = physical page
    of sequence b's logical page p; token n of sequence b (its BFS node n) is slot
    ``n % page_size`` of page ``page_table[b, n // page_size]``. Returns O like ``Q``.
    Mirrors src/ragged_attn.py:934-1004; the walk, the duplicate rule and the result
    are those of :func:`ragged_attention`. Complete trees (b >= 2) look a page up once
    per staged row of a tile in the tensor-core kernel; chains (b = 1) take the per-query
    walk, which looks up each row it stages or reads.
    """
    assert K_cache.shape == V_cache.shape, "K and V cache shapes must match"
    assert Q.dtype in _SUPPORTED and Q.dtype == K_cache.dtype == V_cache.dtype, (
        f"Inputs must be fp16 or bf16 (got {Q.dtype})"
    )
    for name, t in (("Q", Q), ("K_cache", K_cache), ("V_cache", V_cache)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor: this library has no CPU path")
    if Q.dim() != 3 or K_cache.dim() != 4:
        raise ValueError("Q must be [tokens, heads, D] and the caches [pages, page_size, kv_heads, D]")
    total, Hq, D = Q.shape
    _, page_size, Hkv, Dk = K_cache.shape
    if Dk != D or Hq % Hkv != 0:
        raise ValueError(f"cache [.., {Hkv}, {Dk}] does not match Q [.., {Hq}, {D}]")
    if branching_factor < 1:
        raise ValueError(f"branching_factor must be >= 1, got {branching_factor}")
    if max_depth < 0:
        raise ValueError(f"max_depth must be >= 0, got {max_depth}")
    cu_dev, ms = _cu_and_max(cu_seqlens, None, Q.device)
    pt = page_table.to(device=Q.device, dtype=torch.int32).contiguous()
    Q, Kc, Vc = _rowable(Q), _rowable(K_cache), _rowable(V_cache)
    O = torch.empty_like(Q, memory_format=torch.contiguous_format)
    B = int(cu_dev.shape[0]) - 1
    a = _lib.AncestorArgs()
    a.q, a.k, a.v, a.o = Q.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr()
    a.cu_seqlens_q = cu_dev.data_ptr()
    a.q_stride_t, a.q_stride_h = Q.stride(0), Q.stride(1)
    a.k_stride_t, a.k_stride_h, a.k_stride_page = Kc.stride(1), Kc.stride(2), Kc.stride(0)
    a.v_stride_t, a.v_stride_h, a.v_stride_page = Vc.stride(1), Vc.stride(2), Vc.stride(0)
    a.o_stride_t, a.o_stride_h = O.stride(0), O.stride(1)
    a.page_table, a.page_table_stride, a.page_size = pt.data_ptr(), pt.stride(0), page_size
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = B, Hq, Hkv, D
    a.branching, a.max_depth, a.max_seqlen = branching_factor, max_depth, ms
    a.scale = 1.0 / math.sqrt(D)
    a.dtype = _dtype_code(Q.dtype)
    _lib.check(_lib.lib().qa_ancestor_attn(a, _stream_ptr(Q.device)), "qa_ancestor_attn (paged)")
    return O


def build_paged_kv(ks: List[torch.Tensor], vs: List[torch.Tensor], page_size: int = 16):
    """Per-sequence K/V ``[L_b, H, D]`` -> ``(K_cache, V_cache, page_table)``: caches
    ``[total_pages, page_size, H, D]`` (zero-padded last pages) on the inputs' device and
    a CPU int32 ``[B, max_pages]`` table, sequence b's pages numbered consecutively after
    those of sequences < b (src/ragged_attn.py:1007-1047)."""
    B = len(ks)
    H, D = ks[0].shape[1], ks[0].shape[2]
    pages = [(k.shape[0] + page_size - 1) // page_size for k in ks]
    total, max_pages = sum(pages), max(pages)
    K_cache = torch.zeros(total, page_size, H, D, device=ks[0].device, dtype=ks[0].dtype)
    V_cache = torch.zeros_like(K_cache)
    page_table = torch.zeros(B, max_pages, dtype=torch.int32)
    phys = 0
    for b, (k, v) in enumerate(zip(ks, vs)):
        L = k.shape[0]
        for pg in range(pages[b]):
            lo, hi = pg * page_size, min(pg * page_size + page_size, L)
            K_cache[phys, : hi - lo] = k[lo:hi]
            V_cache[phys, : hi - lo] = v[lo:hi]
            page_table[b, pg] = phys
            phys += 1
    return K_cache, V_cache, page_table


def ragged_attention_sibling(Q, K, V, cu_seqlens, branching_factor, max_depth, max_seqlen=None):
    """Alias of :func:`ragged_attention`. The reference's sibling kernel
    (src/ragged_attn.py:1211-1420) only reorders loads of the same math; the
    B200 kernel already shares ancestor rows between siblings."""
    return ragged_attention(Q, K, V, cu_seqlens, branching_factor, max_depth, max_seqlen)


def ragged_attention_sibling_with_lse(Q, K, V, cu_seqlens, branching_factor, max_depth,
                                      max_seqlen=None):
    """Alias of :func:`ragged_attention_with_lse` (see :func:`ragged_attention_sibling`)."""
    return ragged_attention_with_lse(Q, K, V, cu_seqlens, branching_factor, max_depth, max_seqlen)


def fused_lse_merge(
    lse_pre: torch.Tensor,
    lse_tree: torch.Tensor,
    out_pre: torch.Tensor,
    out_tree: torch.Tensor,
) -> torch.Tensor:
    """Merge two partial attention results by log-sum-exp.

    ``lse_*``: ``[B, H, N_q]`` fp32; ``out_*``: ``[B, H, N_q, D]`` fp16/bf16, any
    strides with a unit head_dim stride (permuted views need no copy).
    Returns a new contiguous ``[B, H, N_q, D]`` tensor of ``out_pre``'s dtype.
    """
    B, H, N_q, D = out_pre.shape
    for t in (lse_pre, lse_tree, out_pre, out_tree):
        if not t.is_cuda:
            raise RuntimeError("fused_lse_merge needs CUDA tensors: this library has no CPU path")
    if out_tree.dtype != out_pre.dtype:
        out_tree = out_tree.to(out_pre.dtype)
    lp, lt = lse_pre.float(), lse_tree.float()
    op = out_pre if (out_pre.stride(-1) == 1 and out_pre.data_ptr() % 16 == 0
                     and all(s % 8 == 0 for s in out_pre.stride()[:3])) else out_pre.contiguous()
    ot = out_tree if (out_tree.stride(-1) == 1 and out_tree.data_ptr() % 16 == 0
                      and all(s % 8 == 0 for s in out_tree.stride()[:3])) else out_tree.contiguous()
    res = torch.empty(B, H, N_q, D, dtype=out_pre.dtype, device=out_pre.device)
    L = _lib.lib()
    st = L.qa_lse_merge(lp.data_ptr(), lt.data_ptr(), op.data_ptr(), ot.data_ptr(), res.data_ptr(),
                        B, H, N_q, D,
                        _lib.i64_array(lp.stride()), _lib.i64_array(lt.stride()),
                        _lib.i64_array(op.stride()[:3]), _lib.i64_array(ot.stride()[:3]),
                        _lib.i64_array(res.stride()[:3]), _dtype_code(res.dtype),
                        _stream_ptr(res.device))
    _lib.check(st, "qa_lse_merge")
    return res


def prefix_attention_with_lse(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float = None):
    """Dense attention of tree queries over a shared KV prefix (tensor cores).

    Q: ``[B, N, Hq, D]``; K, V: ``[B, L, Hkv, D]`` (any batch/token/head strides
    with unit stride along D). Every prefix key is visible to every query; GQA
    query head h reads KV head ``h // (Hq // Hkv)``. Returns ``O`` like Q
    (contiguous) and ``LSE`` fp32 ``[B, N, Hq]`` in natural-log units. This is
    the prefix phase of the reference's ``_ragged_tree_attn``
    (scripts/w4a16_e2e.py:1236-1253), without materialising ``repeat_kv``.
    """
    # checked in place: flattening permuted cache views would copy them
    assert Q.dtype in _SUPPORTED and Q.dtype == K.dtype == V.dtype, (
        f"Inputs must be fp16 or bf16 (got {Q.dtype})"
    )
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor: this library has no CPU path")
        if t.dim() != 4:
            raise ValueError(f"{name} must be [batch, tokens, heads, head_dim], got shape {tuple(t.shape)}")
    B, N, Hq, D = Q.shape
    L, Hkv = K.shape[1], K.shape[2]
    O = torch.empty(B, N, Hq, D, dtype=Q.dtype, device=Q.device)
    LSE = torch.empty(B, N, Hq, dtype=torch.float32, device=Q.device)
    if B == 0 or N == 0:
        return O, LSE
    if L == 0:
        O.zero_()
        LSE.fill_(-math.inf)
        return O, LSE
    def fix(t):
        ok = (t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:3]) and t.data_ptr() % 16 == 0)
        return t if ok else t.contiguous()
    Q, K, V = fix(Q), fix(K), fix(V)
    a = _lib.PrefixArgs()
    a.q, a.k, a.v, a.o, a.lse = Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), LSE.data_ptr()
    a.q_stride_b, a.q_stride_t, a.q_stride_h = Q.stride(0), Q.stride(1), Q.stride(2)
    a.k_stride_b, a.k_stride_t, a.k_stride_h = K.stride(0), K.stride(1), K.stride(2)
    a.v_stride_b, a.v_stride_t, a.v_stride_h = V.stride(0), V.stride(1), V.stride(2)
    a.o_stride_b, a.o_stride_t, a.o_stride_h = O.stride(0), O.stride(1), O.stride(2)
    a.lse_stride_b, a.lse_stride_t, a.lse_stride_h = LSE.stride(0), LSE.stride(1), LSE.stride(2)
    a.batch, a.num_queries, a.prefix_len = B, N, L
    a.num_q_heads, a.num_kv_heads, a.head_dim = Hq, Hkv, D
    a.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    a.dtype = _dtype_code(Q.dtype)
    _lib.check(_lib.lib().qa_prefix_attn(a, _stream_ptr(Q.device)), "qa_prefix_attn")
    return O, LSE


def ragged_attention_hybrid(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    prefix_length: int,
    tree_size: int,
    branching_factor: int,
    max_depth: int,
) -> torch.Tensor:
    """Prefix + tree attention in the reference's hybrid layout.

    Q: ``[B*N, H, D]``; K, V: ``[B*(L+N), H(kv), D]`` with each sequence's L
    prefix rows first, then its N tree rows (src/ragged_attn.py:1851-1888).
    Every query sees all L prefix keys plus its tree ancestors. Runs the
    tensor-core prefix pass, then the ancestor pass with the log-sum-exp merge
    fused into it.
    """
    _check_qkv(Q, K, V)
    total, H, D = Q.shape
    N, L = int(tree_size), int(prefix_length)
    B = total // N
    Hkv = K.shape[1]
    cu_q = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device=Q.device)
    cu_kv = torch.arange(0, (B + 1) * (L + N), L + N, dtype=torch.int32, device=Q.device)
    if L == 0:
        O, _ = _ancestor(Q, K, V, cu_q, N, branching=branching_factor, max_depth=max_depth,
                         cu_kv=cu_kv, kv_offset=0)
        return O
    Kb = K.view(B, L + N, Hkv, D)[:, :L]
    Vb = V.view(B, L + N, Hkv, D)[:, :L]
    Op, Lp = prefix_attention_with_lse(Q.view(B, N, H, D), Kb, Vb)
    O, _ = _ancestor(Q, K, V, cu_q, N, branching=branching_factor, max_depth=max_depth,
                     cu_kv=cu_kv, kv_offset=L, prefix_o=Op.view(B * N, H, D),
                     prefix_lse=Lp.view(B * N, H), out=Op.view(B * N, H, D))
    return O


def tree_verify_attention(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    branching_factor: int,
    max_depth: int,
    tree_parents: Optional[torch.Tensor] = None,
    plan: Optional[ParentsPlan] = None,
) -> torch.Tensor:
    """Verify-step attention in the E2E caller's layout (``_ragged_tree_attn``,
    scripts/w4a16_e2e.py:1201-1309).

    Q: ``[B, Hq, N, D]`` (post-RoPE tree queries); K, V: ``[B, Hkv, L+N, D]``
    (prefix then tree). Tree queries see every prefix key and their tree
    ancestors (complete b-ary BFS tree, or ``tree_parents`` ``[N]`` int32 with
    root self-loop, shared by the batch). Returns ``[B, Hq, N, D]`` (a permuted
    view of a ``[B, N, Hq, D]`` buffer). GQA without ``repeat_kv``; no layout
    copies of Q/K/V (the kernels take the strides). ``plan``: a
    :func:`plan_tree_parents` result for this tree and batch (every layer of a
    verify step can share it).
    """
    B, Hq, N, D = Q.shape
    Hkv, LN = K.shape[1], K.shape[2]
    L = LN - N
    Qt = Q.permute(0, 2, 1, 3)                              # [B, N, Hq, D] view
    Kt, Vt = K.permute(0, 2, 1, 3), V.permute(0, 2, 1, 3)  # [B, L+N, Hkv, D] views
    if L > 0:
        out, lse = prefix_attention_with_lse(Qt, Kt[:, :L], Vt[:, :L])
    else:
        out = torch.empty(B, N, Hq, D, dtype=Q.dtype, device=Q.device)
        lse = None
    par = None
    if plan is not None:
        par = plan.parents
    elif tree_parents is not None:
        par = tree_parents.to(device=Q.device, dtype=torch.int32).repeat(B).contiguous()
    # Queries are read in place: as packed rows when the batch pitch is N token rows (a
    # head slice of a fused qkv projection), else through the kernel's batch stride
    # (e.g. a contiguous [B, Hq, N, D] tensor); only a misaligned view is copied.
    q_batched = None
    if Qt.stride(3) != 1 or any(x % 8 for x in Qt.stride()[:3]) or Qt.data_ptr() % 16:
        Qr = Qt.contiguous().view(B * N, Hq, D)
    elif Qt.stride(0) == N * Qt.stride(1):
        Qr = Qt.as_strided((B * N, Hq, D), (Qt.stride(1), Qt.stride(2), 1), Qt.storage_offset())
    else:
        Qr, q_batched = out.view(B * N, Hq, D), Qt  # Qr only carries the packed shape
    Kr, Vr, kv_rows, kv_off = _tree_rows(Kt, Vt, L, N)
    cu_q = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device=Q.device)
    cu_kv = torch.arange(0, (B + 1) * kv_rows, kv_rows, dtype=torch.int32, device=Q.device)
    _ancestor(Qr, Kr, Vr, cu_q, N, branching=branching_factor, max_depth=max_depth, parents=par,
              cu_kv=cu_kv, kv_offset=kv_off,
              prefix_o=out.view(B * N, Hq, D) if L > 0 else None,
              prefix_lse=lse.view(B * N, Hq) if L > 0 else None,
              out=out.view(B * N, Hq, D), q_batched=q_batched, plan=plan)
    return out.permute(0, 2, 1, 3)


def plan_tree_parents(tree_parents: torch.Tensor, batch: int, max_depth: int, device=None) -> Optional[ParentsPlan]:
    """:func:`plan_parents` for :func:`tree_verify_attention`: one tree (``tree_parents``
    ``[N]``, root self-loop) shared by ``batch`` sequences of N queries."""
    N = int(tree_parents.shape[0])
    dev = torch.device(device) if device is not None else tree_parents.device
    cu = torch.arange(0, (batch + 1) * N, N, dtype=torch.int32)
    par = tree_parents.to(device=dev, dtype=torch.int32).repeat(batch).contiguous()
    return plan_parents(cu, par, max_depth, max_seqlen=N, device=dev)


def _tree_rows(Kt: torch.Tensor, Vt: torch.Tensor, L: int, N: int):
    """[B, L+N, Hkv, D] views -> ([B*R, Hkv, D] row tensors, R, offset of the tree rows).

    Uses the views directly when the batch stride is a whole number of token
    rows (the common contiguous [B, L+N, ...] or [B, Hkv, L+N, D] layouts give
    R = L+N or a larger pitch); otherwise copies the tree rows once.
    """
    B, LN, Hkv, D = Kt.shape
    def rows(t):
        sb, st = t.stride(0), t.stride(1)
        if st > 0 and sb % st == 0 and t.stride(3) == 1:
            R = sb // st
            # rows past the last sequence's L+N are never addressed
            base = t.as_strided(((B - 1) * R + LN, Hkv, D), (st, t.stride(2), 1), t.storage_offset())
            return base, R
        return None, None
    Kr, RK = rows(Kt)
    Vr, RV = rows(Vt)
    if Kr is not None and Vr is not None and RK == RV:
        return Kr, Vr, RK, L
    Kc = Kt[:, L:].contiguous().view(B * N, Hkv, D)
    Vc = Vt[:, L:].contiguous().view(B * N, Hkv, D)
    return Kc, Vc, N, 0
