"""CPU oracle for the W4A16 path — TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench CPU arms).

PARITY UNPINNED: the reference's quantiser (GPTQModel, sym int4, group 128,
desc_act=False; scripts/quantize_llama31.py:41-59) and its Marlin GEMM
(scripts/w4a16_e2e.py:698-699) are third-party packages that are neither
vendored in the reference nor installed here, and the reference holds no
quantised fixture. This module restates the published symmetric GPTQ
round-to-nearest rule in numpy, independently of qattention_b200.quant:
scale = fp16(2*amax/15), zero 8, q = clamp(rint(w/scale) + 8, 0, 15),
w' = fp16((q - 8) * scale); and computes Y = X @ W' in fp32 (fp64 accumulate).
"""
from __future__ import annotations

import numpy as np

GROUP = 128


def quantize(W: np.ndarray):
    """W [K, N] float -> (q [K, N] uint8 in 0..15, scales [K/128, N] float16)."""
    K, N = W.shape
    Wg = W.astype(np.float32).reshape(K // GROUP, GROUP, N)
    amax = np.abs(Wg).max(axis=1)
    amax[amax == 0] = 1.0
    scales = (np.float32(2.0) * amax / np.float32(15.0)).astype(np.float16)
    q = np.rint(Wg / scales.astype(np.float32)[:, None, :]) + 8.0
    q = np.clip(q, 0, 15).astype(np.uint8).reshape(K, N)
    return q, scales


def pack(q: np.ndarray) -> np.ndarray:
    """q [K, N] 0..15 -> qweight [N/128, K/128, 4, 128, 4] int32 (the library's tile-major,
    chunk-plane layout: tile (n tile, k tile), 16-byte chunk c, row = output column, word w
    holds k = 32 c + 8 w .. + 7): 8 consecutive k per word, k%8 = 2i in nibble i and
    k%8 = 2i+1 in nibble i+4."""
    K, N = q.shape
    qt = q.T.reshape(N, K // 8, 8).astype(np.uint32)
    words = np.zeros((N, K // 8), dtype=np.uint32)
    for j in range(8):
        nibble = j // 2 if j % 2 == 0 else 4 + j // 2
        words |= qt[:, :, j] << np.uint32(4 * nibble)
    w = words.view(np.int32).reshape(N // 128, 128, K // 128, 4, 4)
    return np.ascontiguousarray(w.transpose(0, 2, 3, 1, 4))


def dequantize(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """-> W' [K, N] float16, each element fp16((q - 8) * scale) with one rounding."""
    K, N = q.shape
    s = np.repeat(scales.astype(np.float32), GROUP, axis=0)
    return ((q.astype(np.float32) - 8.0) * s).astype(np.float16)


def gemm(X: np.ndarray, q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Y = X @ dequantize(q, scales) in fp64 accumulation, returned as float32."""
    W = dequantize(q, scales).astype(np.float64)
    return (X.astype(np.float64) @ W).astype(np.float32)
