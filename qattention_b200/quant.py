"""W4A16 weight format: symmetric int4, group 128 along K, fp16 scales (host-side quantiser).

The reference quantises its verify-step linears with GPTQModel
``QuantizeConfig(bits=4, group_size=128, desc_act=False, sym=True)``
(scripts/quantize_llama31.py:41-59) and runs them with Marlin kernels
(scripts/w4a16_e2e.py:698-699). Neither package ships with the reference, so
this module states the format it implements, following the published
symmetric GPTQ rule (round-to-nearest; the GPTQ error-compensating solve is a
calibration step, out of scope for random-init weights):

* For output column n and group g (k in [128 g, 128 g + 128)):
  ``amax = max |W[k, n]|`` (an all-zero group uses amax = 1),
  ``scale = fp16(2 * amax / 15)``, zero point 8 (no zero tensor).
* ``q = clamp(round_half_even(W / scale) + 8, 0, 15)`` computed in fp32 with
  the fp16-rounded scale.
* Dequantisation: ``w = fp16((q - 8) * scale)`` (exact product, one rounding).

Packing (this library's layout, chosen for the GEMM kernel): ``qweight`` is
int32 ``[N // 128, K // 128, 4, 128, 4]`` — tile-major, so the 128 output
columns x 128 k of one GEMM step are one contiguous 8 KB block that a single
bulk copy fetches, stored chunk-plane-major inside the tile: index
``[tile_n, tile_k, c, j, w]`` is output column 128 * tile_n + j, word 4 c + w
of its row, which holds k = 8 (4 c + w) .. + 7 of that step (the 16-byte
chunks of one plane c are consecutive rows, so the GEMM's per-row reads from
shared memory are bank-conflict free). The nibbles of a word are interleaved:
k % 8 = 2i sits in nibble i and k % 8 = 2i + 1 in nibble i + 4 (i = 0..3),
so ``(word >> 4i) & 0x000F000F`` yields the consecutive pair (2i, 2i+1) as the
two halves of a 32-bit lane. ``scales`` is fp16 ``[K // 128, N]``. No
activation-order permutation (``desc_act=False``). N and K are multiples of
128.
"""
from __future__ import annotations

import torch

GROUP = 128
# bit position of k % 8 = 0..7 inside a packed word (interleaved nibble order)
NIBBLE_SHIFT = (0, 16, 4, 20, 8, 24, 12, 28)


def quantize_w4a16(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise a ``[K, N]`` weight (Y = X @ W) to
    ``(qweight [N/128, K/128, 4, 128, 4] int32, scales [K/128, N] fp16)``.

    Runs with torch ops on W's device (CPU or CUDA); the result is identical on both.
    """
    K, N = W.shape
    if K % GROUP != 0 or N % 128 != 0:
        raise ValueError(f"K ({K}) and N ({N}) must be multiples of 128")
    Wf = W.float().reshape(K // GROUP, GROUP, N)
    amax = Wf.abs().amax(dim=1)                                 # [K/128, N]
    amax = torch.where(amax == 0, torch.ones_like(amax), amax)
    scales = (2.0 * amax / 15.0).to(torch.float16)              # [K/128, N]
    q = torch.round(Wf / scales.float()[:, None, :]) + 8.0
    q = q.clamp_(0, 15).to(torch.int32).reshape(K, N)           # [K, N] in 0..15
    return pack_int4(q), scales.contiguous()


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """``[K, N]`` integer values in 0..15 -> this library's tile-major int32
    ``[N/128, K/128, 4, 128, 4]`` packing (the inverse of :func:`unpack_int4`)."""
    K, N = q.shape
    if K % GROUP != 0 or N % 128 != 0:
        raise ValueError(f"K ({K}) and N ({N}) must be multiples of 128")
    qt = q.to(torch.int64).t().contiguous().view(N, K // 8, 8)  # [N, K/8, 8], k % 8 last
    shifts = torch.tensor(NIBBLE_SHIFT, dtype=torch.int64, device=q.device)
    words = (qt << shifts).sum(dim=-1)                          # 0 .. 2^32-1
    words = torch.where(words < 2**31, words, words - 2**32).to(torch.int32)  # [N, K/8]
    return words.view(N // 128, 128, K // 128, 4, 4).permute(0, 2, 3, 1, 4).contiguous()


def _unpack_gptq_nibbles(packed: torch.Tensor, along_rows: bool) -> torch.Tensor:
    """GPTQ int32 packing, 8 values per word, value i in bits 4i..4i+3: rows
    ``[R/8, C] -> [R, C]`` (``along_rows``) or columns ``[R, C/8] -> [R, C]``."""
    w = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(0, 32, 4, dtype=torch.int64, device=packed.device)
    if along_rows:
        vals = (w[:, None, :] >> shifts[None, :, None]) & 0xF   # [R/8, 8, C]
        return vals.reshape(-1, packed.shape[1]).to(torch.int32)
    vals = (w[:, :, None] >> shifts[None, None, :]) & 0xF       # [R, C/8, 8]
    return vals.reshape(packed.shape[0], -1).to(torch.int32)


def from_gptq(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor | None = None,
              g_idx: torch.Tensor | None = None, *, group_size: int = GROUP,
              zero_offset: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """A GPTQ-format linear (the checkpoint layout GPTQModel / AutoGPTQ save and
    the reference loads: scripts/w4a16_e2e.py:749-753, quantised with
    bits=4, group_size=128, sym=True, desc_act=False at
    scripts/quantize_llama31.py:41-46) -> ``(qweight, scales)`` in this
    library's format, bit for bit the same weights.

    GPTQ layout: ``qweight`` int32 ``[K/8, N]`` holds k = 8r + i of column n in
    bits 4i..4i+3 of word ``[r, n]``; ``scales`` fp16 ``[K/group, N]``;
    ``qzeros`` int32 ``[K/group, N/8]`` packs the zero points the same way
    along N, stored minus ``zero_offset`` (1 in the classic checkpoint format,
    0 in GPTQModel's internal one); ``g_idx`` int32 ``[K]`` is the group of each
    k. Dequantisation is ``(q - zero) * scale`` in both formats, so a symmetric
    checkpoint (every zero 8) with group 128 and no activation order maps onto
    this library's ``fp16((q - 8) * scale)`` exactly. Anything else (asymmetric
    zeros, another group size, an act-order ``g_idx``, bits other than 4)
    raises ``ValueError``: the GEMM kernel implements that one format.
    """
    if qweight.dtype != torch.int32 or qweight.dim() != 2:
        raise ValueError("qweight must be a 2-D int32 tensor [K/8, N] (4-bit GPTQ packing)")
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    if group_size != GROUP:
        raise ValueError(f"group_size {group_size} is not supported (the kernel uses {GROUP})")
    if K % GROUP != 0 or N % 128 != 0:
        raise ValueError(f"K ({K}) and N ({N}) must be multiples of 128")
    if tuple(scales.shape) != (K // GROUP, N):
        raise ValueError(f"scales must be [{K // GROUP}, {N}], got {tuple(scales.shape)}")
    if g_idx is not None:
        expect = torch.arange(K, device=g_idx.device, dtype=torch.int64) // GROUP
        if g_idx.numel() != K or not torch.equal(g_idx.to(torch.int64).flatten(), expect):
            raise ValueError("g_idx is not k // group_size: act-order (desc_act) checkpoints are not supported")
    if qzeros is not None:
        if tuple(qzeros.shape) != (K // GROUP, N // 8):
            raise ValueError(f"qzeros must be [{K // GROUP}, {N // 8}], got {tuple(qzeros.shape)}")
        zeros = _unpack_gptq_nibbles(qzeros, along_rows=False) + zero_offset
        if not bool((zeros == 8).all()):
            raise ValueError("asymmetric zero points: only symmetric (sym=True, zero 8) checkpoints are supported")
    q = _unpack_gptq_nibbles(qweight, along_rows=True)          # [K, N] in 0..15
    return pack_int4(q), scales.to(torch.float16).contiguous()


def to_gptq(qweight: torch.Tensor, scales: torch.Tensor, zero_offset: int = 1):
    """This library's ``(qweight, scales)`` -> GPTQ-format ``(qweight [K/8, N],
    scales, qzeros [K/128, N/8], g_idx [K])`` (the inverse of :func:`from_gptq`)."""
    q = unpack_int4(qweight).to(torch.int64)                   # [K, N]
    K, N = q.shape
    shifts = torch.arange(0, 32, 4, dtype=torch.int64, device=q.device)
    words = (q.view(K // 8, 8, N) << shifts[None, :, None]).sum(dim=1)
    gq = torch.where(words < 2**31, words, words - 2**32).to(torch.int32)
    z = torch.full((K // GROUP, N // 8, 8), 8 - zero_offset, dtype=torch.int64, device=q.device)
    zw = (z << shifts).sum(dim=-1)
    qz = torch.where(zw < 2**31, zw, zw - 2**32).to(torch.int32)
    g_idx = (torch.arange(K, device=q.device) // GROUP).to(torch.int32)
    return gq, scales.contiguous(), qz, g_idx


def unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """Tile-major ``[N/128, K/128, 4, 128, 4]`` int32 -> ``[K, N]`` int32 values in 0..15 (host helper)."""
    NT, KT = qweight.shape[:2]
    N, K8 = NT * 128, KT * 16
    w = qweight.permute(0, 3, 1, 2, 4).reshape(N, K8).to(torch.int64) & 0xFFFFFFFF
    shifts = torch.tensor(NIBBLE_SHIFT, dtype=torch.int64, device=qweight.device)
    vals = (w[..., None] >> shifts) & 0xF                         # [N, K/8, 8]
    return vals.reshape(N, K8 * 8).t().to(torch.int32).contiguous()


_COUNTERS = {}


def _split_counters(device, n: int):
    """Zeroed split-K tile counters of a device (every GEMM leaves them zero), or None
    when they would have to be created inside a CUDA-graph capture (that call then
    adds its partials with a second kernel). Split-K GEMMs on one device share
    them: do not run two at the same time on different streams."""
    buf = _COUNTERS.get(device.index)
    if buf is None or buf.numel() < n:
        if torch.cuda.is_current_stream_capturing():
            return None
        buf = torch.zeros(max(n, 1 << 14), dtype=torch.int32, device=device)
        _COUNTERS[device.index] = buf
    return buf


def w4a16_linear(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                 splits: int = 0, out: torch.Tensor = None) -> torch.Tensor:
    """``x @ dequant(qweight, scales)`` on the B200 tensor cores (fp16 in/out, fp32 accumulate).

    x: ``[..., K]`` fp16 CUDA (unit stride along K); qweight ``[N/128, K/128, 4, 128, 4]`` int32,
    scales ``[K/128, N]`` fp16 (see :func:`quantize_w4a16`). ``splits`` = K split
    across CTAs (0 = automatic); a split-K run uses a temporary fp32 workspace.
    """
    import ctypes
    from . import _lib
    if x.dtype != torch.float16 or not x.is_cuda:
        raise RuntimeError("w4a16_linear needs fp16 CUDA activations")
    K = x.shape[-1]
    N = qweight.shape[0] * 128
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = out if out is not None else torch.empty(M, N, dtype=torch.float16, device=x.device)
    L = _lib.lib()
    s = ctypes.c_int32(splits)
    ws_bytes = ctypes.c_int64(0)
    if splits == 0 and M > 0:
        _lib.check(L.qa_w4a16_plan(M, N, K, ctypes.byref(s), ctypes.byref(ws_bytes)), "qa_w4a16_plan")
    elif splits > 1:
        ws_bytes.value = splits * M * N * 4
    ws = torch.empty(max(1, ws_bytes.value // 4), dtype=torch.float32, device=x.device) if ws_bytes.value else None
    a = _lib.W4A16Args()
    a.x, a.qweight, a.scales, a.y = x2.data_ptr(), qweight.data_ptr(), scales.data_ptr(), y.data_ptr()
    a.workspace = ws.data_ptr() if ws is not None else None
    a.x_stride, a.y_stride = x2.stride(0), y.stride(0)
    a.M, a.N, a.K, a.splits = M, N, K, s.value
    stream = torch.cuda.current_stream(x.device)
    if s.value > 1:  # split-K in one launch (the last CTA of each tile adds the partials)
        cnt = _split_counters(x.device, (N // 128) * ((M + 15) // 16))
        a.counters = cnt.data_ptr() if cnt is not None else None
    _lib.check(L.qa_w4a16_gemm(a, stream.cuda_stream), "qa_w4a16_gemm")
    return y.view(*x.shape[:-1], N)


def w4a16_dequantize(qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """GPU dequantisation to fp16 ``[K, N]`` (for checks; the GEMM never materialises it)."""
    from . import _lib
    N, K = qweight.shape[0] * 128, qweight.shape[1] * 128
    out = torch.empty(K, N, dtype=torch.float16, device=qweight.device)
    _lib.check(_lib.lib().qa_w4a16_dequant(qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), K, N,
                                            torch.cuda.current_stream(qweight.device).cuda_stream),
               "qa_w4a16_dequant")
    return out
