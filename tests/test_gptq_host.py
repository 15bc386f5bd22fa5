"""GPTQ-checkpoint loading (quant.from_gptq): GPTQ-format tensors built here with
plain loops from the published layout (qweight int32 [K/8, N], value k = 8r + i of
column n in bits 4i..4i+3 of word [r, n]; qzeros packed the same way along N,
stored as zero - 1; scales [K/128, N]; g_idx = k // 128) load bit for bit into this
library's format: the result equals the oracle's packing of the same values, and its
dequantisation is (q - 8) * scale."""
import numpy as np
import pytest
import torch

from oracle import w4a16_oracle as wo
from qattention_b200 import quant


def _gptq_tensors(K, N, seed, zero=8, zero_offset=1):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(K, N), dtype=np.int64)
    scales = (rng.random((K // 128, N)) * 0.02 + 1e-3).astype(np.float16)
    qw = np.zeros((K // 8, N), dtype=np.uint64)
    for k in range(K):
        qw[k // 8] |= (q[k].astype(np.uint64) << np.uint64(4 * (k % 8)))
    qz = np.zeros((K // 128, N // 8), dtype=np.uint64)
    for n in range(N):
        qz[:, n // 8] |= np.uint64(zero - zero_offset) << np.uint64(4 * (n % 8))
    as_i32 = lambda a: torch.from_numpy(a.astype(np.uint32).view(np.int32).copy())  # noqa: E731
    g_idx = torch.arange(K, dtype=torch.int32) // 128
    return q, torch.from_numpy(scales), as_i32(qw), as_i32(qz), g_idx


@pytest.mark.parametrize("K,N,offset", [(256, 128, 1), (384, 256, 0)])
def test_from_gptq_bit_exact(K, N, offset):
    q, scales, qw, qz, g_idx = _gptq_tensors(K, N, seed=K + N, zero_offset=offset)
    ours, s = quant.from_gptq(qw, scales, qz, g_idx, zero_offset=offset)
    assert ours.shape == (N // 128, K // 128, 4, 128, 4) and ours.dtype == torch.int32
    assert torch.equal(quant.unpack_int4(ours), torch.from_numpy(q).to(torch.int32))
    assert torch.equal(s, scales)
    # the oracle's own packing of the same values (restated independently), and its dequantisation
    assert np.array_equal(wo.pack(q.astype(np.uint32)), ours.numpy())
    deq = wo.dequantize(quant.unpack_int4(ours).numpy(), s.numpy())
    ref = ((q.astype(np.float32) - 8.0) * scales.numpy().astype(np.float32).repeat(128, axis=0)).astype(np.float16)
    assert np.array_equal(deq.view(np.uint16), ref.view(np.uint16))
    # and back: to_gptq reproduces the checkpoint tensors
    gq, gs, gz, gi = quant.to_gptq(ours, s, zero_offset=offset)
    assert torch.equal(gq, qw) and torch.equal(gz, qz) and torch.equal(gi, g_idx) and torch.equal(gs, scales)


def test_from_gptq_rejects_other_formats():
    q, scales, qw, qz, g_idx = _gptq_tensors(256, 128, seed=1)
    _, _, _, qz_asym, _ = _gptq_tensors(256, 128, seed=1, zero=7)
    with pytest.raises(ValueError, match="asymmetric"):
        quant.from_gptq(qw, scales, qz_asym, g_idx)
    with pytest.raises(ValueError, match="act-order"):
        quant.from_gptq(qw, scales, qz, g_idx.flip(0))
    with pytest.raises(ValueError, match="group_size"):
        quant.from_gptq(qw, scales, qz, g_idx, group_size=64)
    with pytest.raises(ValueError, match="scales"):
        quant.from_gptq(qw, scales[:1], qz, g_idx)
    with pytest.raises(ValueError, match="int32"):
        quant.from_gptq(qw.to(torch.int64), scales, qz, g_idx)
