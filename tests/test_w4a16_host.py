"""W4A16 format on the host: the product quantiser against the numpy oracle (bit-exact)."""
import numpy as np
import torch

from oracle import w4a16_oracle as wo
from qattention_b200 import quant


def test_quantiser_matches_oracle_bit_exact():
    g = torch.Generator().manual_seed(0)
    W = torch.randn(512, 128, generator=g) * 0.05
    W[:128, 3] = 0.0  # an all-zero group
    qw, sc = quant.quantize_w4a16(W)
    q_ref, s_ref = wo.quantize(W.numpy())
    assert qw.dtype == torch.int32 and qw.shape == (1, 4, 4, 128, 4)
    assert sc.dtype == torch.float16 and sc.shape == (4, 128)
    assert np.array_equal(sc.numpy().view(np.uint16), s_ref.view(np.uint16))
    assert np.array_equal(qw.numpy(), wo.pack(q_ref))
    assert np.array_equal(quant.unpack_int4(qw).numpy(), q_ref.astype(np.int32))


def test_dequant_error_bound():
    g = torch.Generator().manual_seed(1)
    W = torch.randn(256, 64, generator=g)
    q, s = wo.quantize(W.numpy())
    Wd = wo.dequantize(q, s).astype(np.float32)
    step = np.repeat(s.astype(np.float32), 128, axis=0)
    # round-to-nearest: |w - w'| <= scale/2 (+ fp16 rounding of the product)
    assert np.all(np.abs(W.numpy() - Wd) <= step * 0.5 + np.abs(Wd) * 2 ** -10 + 1e-7)


def test_rejects_ragged_k():
    import pytest
    with pytest.raises(ValueError):
        quant.quantize_w4a16(torch.zeros(100, 8))
