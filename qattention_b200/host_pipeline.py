"""Ancestor attention from host buffers to host buffers, with the copies overlapped.

A caller whose Q/K/V live in host memory and who wants O and LSE back in host
memory pays three things per call: the host->device copy of the inputs, the
kernel, and the device->host copy of the outputs. On a B200 the kernel is a
small fraction of that (C3: ~0.11 ms against ~7 ms of PCIe traffic), and run
back to back the two copies add up. Trees never attend to each other, so the
packed batch splits into chunks of whole trees, and three CUDA streams overlap
chunk k+1's upload, chunk k's attention and chunk k-1's download: the call then
costs about its largest transfer (the upload) instead of the sum.

Every tree is computed by the same kernel on the same rows as in one
``ragged_attention_with_lse`` over the whole batch, so the results are
bit-identical to it. The reference has no host-buffer entry point; its callers
move tensors with ``.to(device)`` before ``ragged_attention`` (src/ragged_attn.py:1080).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from .ragged_attn import _SUPPORTED, _ancestor

_STREAMS: Dict[int, Tuple[torch.cuda.Stream, torch.cuda.Stream, torch.cuda.Stream]] = {}


def _streams(device: torch.device):
    """Upload, compute and download streams of a device (made once, reused)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        with torch.cuda.device(idx):
            _STREAMS[idx] = (torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream())
    return _STREAMS[idx]


def chunk_bounds(cu: list, chunks: int) -> list:
    """Tree indices that cut the batch into <= `chunks` non-empty contiguous groups
    of near-equal token counts (boundary k = the tree start nearest k/chunks of the tokens)."""
    B = len(cu) - 1
    total = cu[-1]
    n = max(1, min(chunks, B))  # fewer trees than chunks: one tree per chunk
    pts = [0]
    for k in range(1, n):
        goal = total * k / n
        j = next((i for i in range(B + 1) if cu[i] >= goal), B)
        if j > 0 and goal - cu[j - 1] < cu[j] - goal:
            j -= 1
        pts.append(j)
    pts.append(B)
    return sorted(set(pts))


def ragged_attention_with_lse_host(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    cu_seqlens: torch.Tensor,
    branching_factor: int,
    max_depth: int,
    *,
    device=None,
    out: Optional[torch.Tensor] = None,
    lse_out: Optional[torch.Tensor] = None,
    chunks: int = 8,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``ragged_attention_with_lse`` on host tensors, returning host tensors.

    Q, K, V: packed ``[T, H, D]`` host tensors (fp16/bf16; pinned memory makes the
    copies asynchronous and lets them overlap). ``cu_seqlens``: int32 offsets of
    the B trees (host). ``out`` / ``lse_out``: optional host outputs ``[T, H, D]``
    and fp32 ``[T, H]`` (allocated pinned when omitted). The batch is split into
    at most ``chunks`` groups of whole trees. Returns when the outputs are in
    host memory.
    """
    # the device path's dtype rule (src/ragged_attn.py:1113-1116)
    assert Q.dtype in _SUPPORTED and Q.dtype == K.dtype == V.dtype, (
        f"Inputs must be fp16 or bf16 (got {Q.dtype})")
    if Q.dim() != 3 or K.shape != Q.shape or V.shape != K.shape:
        raise ValueError(f"Q, K, V must be [tokens, heads, head_dim] of one shape, got {tuple(Q.shape)}, "
                         f"{tuple(K.shape)}, {tuple(V.shape)}")
    if Q.is_cuda or K.is_cuda or V.is_cuda:
        raise ValueError("ragged_attention_with_lse_host takes host tensors; use ragged_attention_with_lse")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    T, H, D = Q.shape
    cu = [int(x) for x in cu_seqlens.tolist()]
    if len(cu) < 1 or cu[0] != 0 or cu[-1] != T:
        raise ValueError("cu_seqlens must start at 0 and end at the packed token count")
    if out is None:
        out = torch.empty(T, H, D, dtype=Q.dtype).pin_memory()
    if lse_out is None:
        lse_out = torch.empty(T, H, dtype=torch.float32).pin_memory()
    if T == 0:
        return out, lse_out
    pts = chunk_bounds(cu, chunks)
    # every chunk's own cu_seqlens (starting at 0), uploaded once before the inputs
    local = []
    for a, b in zip(pts[:-1], pts[1:]):
        local.extend(c - cu[a] for c in cu[a:b + 1])
    cu_all_h = torch.tensor(local, dtype=torch.int32).pin_memory()
    up, comp, down = _streams(dev)
    cur = torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        dQ = torch.empty(T, H, D, dtype=Q.dtype, device=dev)
        dK = torch.empty_like(dQ, dtype=K.dtype)
        dV = torch.empty_like(dQ, dtype=V.dtype)
        dO = torch.empty(T, H, D, dtype=Q.dtype, device=dev)
        dL = torch.empty(T, H, dtype=torch.float32, device=dev)
        cu_all = torch.empty_like(cu_all_h, device=dev)
    for s in (up, comp, down):
        s.wait_stream(cur)  # the buffers were allocated on the caller's stream
    ev_in, ev_out = [], []
    with torch.cuda.stream(up):
        cu_all.copy_(cu_all_h, non_blocking=True)
        for a, b in zip(pts[:-1], pts[1:]):
            s = slice(cu[a], cu[b])
            dQ[s].copy_(Q[s], non_blocking=True)
            dK[s].copy_(K[s], non_blocking=True)
            dV[s].copy_(V[s], non_blocking=True)
            e = torch.cuda.Event()
            e.record(up)
            ev_in.append(e)
    off = 0
    with torch.cuda.stream(comp):
        for k, (a, b) in enumerate(zip(pts[:-1], pts[1:])):
            comp.wait_event(ev_in[k])
            s = slice(cu[a], cu[b])
            ms = max(cu[i + 1] - cu[i] for i in range(a, b))
            _ancestor(dQ[s], dK[s], dV[s], cu_all[off:off + b - a + 1], ms, branching=branching_factor,
                      max_depth=max_depth, want_lse=True, out=dO[s], lse_out=dL[s])
            off += b - a + 1
            e = torch.cuda.Event()
            e.record(comp)
            ev_out.append(e)
    with torch.cuda.stream(down):
        for k, (a, b) in enumerate(zip(pts[:-1], pts[1:])):
            down.wait_event(ev_out[k])
            s = slice(cu[a], cu[b])
            out[s].copy_(dO[s], non_blocking=True)
            lse_out[s].copy_(dL[s], non_blocking=True)
    # every upload and kernel precedes the last download: once it is done the
    # device buffers are idle and go back to the caller's stream's pool
    down.synchronize()
    return out, lse_out
