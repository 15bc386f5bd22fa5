"""W4A16 tree-verify step of a Llama-architecture model (bench config C5) on this package's kernels.

The reference's end-to-end script (scripts/w4a16_e2e.py) runs EAGLE-3 tree
verification on a GPTQ-int4 Llama-3.1-8B: every decoder layer projects the
tree tokens (W4A16 Marlin linears, :698-699), applies rotate-half RoPE at
position prefix_len + depth (:993, :1424-1431), attends to the cached prefix
and to the tokens' tree ancestors (`_ragged_tree_attn`, :1201-1309), and runs
the SwiGLU MLP. This module is that verify step, built from:

* ``quant.w4a16_linear`` — the B200 W4A16 GEMM, with q/k/v and gate/up fused
  along N as serving stacks load them;
* ``ragged_attn.tree_verify_attention`` — the tcgen05 prefix pass plus the
  ancestor pass with the LSE merge fused, reading the KV cache in place (GQA
  without ``repeat_kv``);
* ``qa_add_rmsnorm``, ``qa_rope_qkv``, ``qa_silu_mul`` (csrc/verify_ops.cu) for
  the elementwise work between them;
* the fp16 LM head through cuBLAS (a plain library GEMM: GPTQ leaves it
  unquantised).

Weights are random (no checkpoints here); the architecture and shapes are the
model's. ``VerifyModel.step`` returns the logits of every tree token.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, quant
from . import ragged_attn as ra


@dataclass
class LlamaConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    # Llama-3.1 long-context frequency scaling ("llama3" rope type)
    rope_factor: float = 8.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    rope_original_max_pos: int = 8192


def llama31_inv_freq(cfg: LlamaConfig) -> torch.Tensor:
    """RoPE inverse frequencies with the Llama-3.1 scaling rule (fp32, [head_dim/2])."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    if cfg.rope_factor == 1.0:
        return inv.float()
    low_wl = cfg.rope_original_max_pos / cfg.rope_low_freq_factor
    high_wl = cfg.rope_original_max_pos / cfg.rope_high_freq_factor
    wl = 2 * math.pi / inv
    smooth = (cfg.rope_original_max_pos / wl - cfg.rope_low_freq_factor) / (
        cfg.rope_high_freq_factor - cfg.rope_low_freq_factor)
    scaled = torch.where(wl > low_wl, inv / cfg.rope_factor, inv)
    mid = (wl <= low_wl) & (wl >= high_wl)
    scaled = torch.where(mid, (1 - smooth) * inv / cfg.rope_factor + smooth * inv, scaled)
    return scaled.float()


def tree_depths(b: int, d: int) -> torch.Tensor:
    """Depth of every node of a complete b-ary BFS tree of depth d (int64 [N])."""
    depth, out = 0, []
    width = 1
    for depth in range(d + 1):
        out += [depth] * width
        width *= b
    return torch.tensor(out, dtype=torch.int64)


class VerifyModel:
    """Random-init W4A16 Llama model for the tree-verify step (one GPU)."""

    def __init__(self, cfg: LlamaConfig, device, seed: int = 0, std: float = 0.02):
        self.cfg = cfg
        self.dev = torch.device(device)
        g = torch.Generator(device=self.dev).manual_seed(seed)
        H, D, Hq, Hkv, F = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.ffn

        def w4(K, N):
            W = torch.randn(K, N, generator=g, device=self.dev) * std
            return quant.quantize_w4a16(W)

        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "qkv": w4(H, (Hq + 2 * Hkv) * D), "o": w4(Hq * D, H),
                "gate_up": w4(H, 2 * F), "down": w4(F, H),
                "ln1": (1.0 + 0.1 * torch.randn(H, generator=g, device=self.dev)).half(),
                "ln2": (1.0 + 0.1 * torch.randn(H, generator=g, device=self.dev)).half(),
            })
        self.embed = (torch.randn(cfg.vocab, H, generator=g, device=self.dev) * std).half()
        self.norm = (1.0 + 0.1 * torch.randn(H, generator=g, device=self.dev)).half()
        self.lm_head = (torch.randn(H, cfg.vocab, generator=g, device=self.dev) * std).half()
        self.inv_freq = llama31_inv_freq(cfg).to(self.dev)
        self._pos = {}  # (prefix_len, branching, depth, B) -> int32 positions on the device

    def new_cache(self, batch: int, prefix_len: int, tree_len: int, seed: int = 1):
        """Per-layer K/V caches [B, Hkv, L+N, D]: the prefix filled (as after a prefill)."""
        c = self.cfg
        g = torch.Generator(device=self.dev).manual_seed(seed)
        cache = []
        for _ in range(c.layers):
            k = torch.zeros(batch, c.kv_heads, prefix_len + tree_len, c.head_dim, dtype=torch.float16, device=self.dev)
            v = torch.zeros_like(k)
            k[:, :, :prefix_len] = torch.randn(batch, c.kv_heads, prefix_len, c.head_dim, generator=g,
                                               device=self.dev).half()
            v[:, :, :prefix_len] = torch.randn(batch, c.kv_heads, prefix_len, c.head_dim, generator=g,
                                               device=self.dev).half()
            cache.append((k, v))
        return cache

    def step(self, tokens: torch.Tensor, cache, prefix_len: int, branching: int, depth: int) -> torch.Tensor:
        """Verify one complete ``branching``-ary tree of ``depth`` per sequence.

        tokens: int64 [B, N] on the device (BFS order). Returns fp16 logits [B*N, vocab].
        The tree's K/V are written into ``cache`` after the prefix.
        """
        c = self.cfg
        B, N = tokens.shape
        M = B * N
        H, D, Hq, Hkv, F = c.hidden, c.head_dim, c.heads, c.kv_heads, c.ffn
        L = _lib.lib()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        key = (prefix_len, branching, depth, B)
        pos = self._pos.get(key)
        if pos is None:  # made once, outside any graph capture (a host-to-device copy)
            pos = (prefix_len + tree_depths(branching, depth)).to(self.dev, torch.int32).repeat(B)
            self._pos[key] = pos
        h = self.embed[tokens.reshape(-1)]                       # residual stream [M, H]
        x = torch.empty(M, H, dtype=torch.float16, device=self.dev)
        qkv = torch.empty(M, (Hq + 2 * Hkv) * D, dtype=torch.float16, device=self.dev)
        attn_proj = torch.empty(M, H, dtype=torch.float16, device=self.dev)
        gu = torch.empty(M, 2 * F, dtype=torch.float16, device=self.dev)
        act = torch.empty(M, F, dtype=torch.float16, device=self.dev)
        mlp = torch.empty(M, H, dtype=torch.float16, device=self.dev)
        delta = None
        for li, lw in enumerate(self.layers):
            kc, vc = cache[li]
            _lib.check(L.qa_add_rmsnorm(h.data_ptr(), delta.data_ptr() if delta is not None else None,
                                        lw["ln1"].data_ptr(), x.data_ptr(), M, H, c.rms_eps, st), "qa_add_rmsnorm")
            quant.w4a16_linear(x, *lw["qkv"], out=qkv)
            _lib.check(L.qa_rope_qkv(qkv.data_ptr(), pos.data_ptr(), self.inv_freq.data_ptr(), kc.data_ptr(),
                                     vc.data_ptr(), M, N, Hq, Hkv, D, kc.stride(0), kc.stride(1), prefix_len, st),
                       "qa_rope_qkv")
            q = qkv.view(B, N, Hq + 2 * Hkv, D)[:, :, :Hq].permute(0, 2, 1, 3)
            o = ra.tree_verify_attention(q, kc, vc, branching, depth)    # [B, Hq, N, D] view
            o2 = o.permute(0, 2, 1, 3).reshape(M, Hq * D)               # contiguous underneath: no copy
            quant.w4a16_linear(o2, *lw["o"], out=attn_proj)
            _lib.check(L.qa_add_rmsnorm(h.data_ptr(), attn_proj.data_ptr(), lw["ln2"].data_ptr(), x.data_ptr(),
                                        M, H, c.rms_eps, st), "qa_add_rmsnorm")
            quant.w4a16_linear(x, *lw["gate_up"], out=gu)
            _lib.check(L.qa_silu_mul(gu.data_ptr(), act.data_ptr(), M, F, st), "qa_silu_mul")
            quant.w4a16_linear(act, *lw["down"], out=mlp)
            delta = mlp
        _lib.check(L.qa_add_rmsnorm(h.data_ptr(), delta.data_ptr(), self.norm.data_ptr(), x.data_ptr(), M, H,
                                    c.rms_eps, st), "qa_add_rmsnorm")
        return x @ self.lm_head

    def capture(self, tokens: torch.Tensor, cache, prefix_len: int, branching: int, depth: int):
        """Record one verify step in a CUDA graph (the reference captures its verify
        forward too: scripts/w4a16_e2e.py:1455-1575). ``tokens`` is the static input
        buffer (copy new tokens into it before a replay); returns ``(graph, logits)``
        where ``logits`` is the static output. Every launch of the step (GEMMs,
        attention, elementwise kernels, the LM head) is in the graph; the first call
        runs the step eagerly on a side stream to create its buffers and memos."""
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.step(tokens, cache, prefix_len, branching, depth)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits = self.step(tokens, cache, prefix_len, branching, depth)
        return graph, logits
