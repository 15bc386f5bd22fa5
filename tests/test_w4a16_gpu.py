"""GPU W4A16: dequantisation bit-exact vs the CPU spec, GEMM vs the fp32 oracle."""
import numpy as np
import pytest
import torch

from oracle import w4a16_oracle as wo

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qattention_b200 import _lib, quant


def _weights(K, N, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(K, N, generator=g) * 0.02
    qw, sc = quant.quantize_w4a16(W)
    return qw, sc


@pytest.mark.parametrize("K,N", [(128, 128), (512, 384), (4096, 1024)])
def test_dequant_bit_exact(K, N):
    qw, sc = _weights(K, N, K + N)
    out = quant.w4a16_dequantize(qw.cuda(), sc.cuda()).cpu()
    ref = wo.dequantize(quant.unpack_int4(qw).numpy().astype(np.uint8), sc.numpy())
    assert np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("M,N,K,splits", [
    (1, 128, 128, 1), (7, 256, 512, 0), (16, 256, 512, 1), (40, 256, 512, 2), (64, 384, 1024, 1), (65, 256, 512, 0), (128, 128, 4096, 0),
    (200, 512, 2048, 1), (200, 512, 2048, 4), (1024, 1024, 4096, 0), (33, 4096, 4096, 0),
    # token counts whose shared-memory ring or TMEM buffer count is not a multiple of the
    # kernel's chain count before rounding (ring slots must stay with one chain)
    (16, 2048, 8192, 1), (80, 512, 8192, 1), (96, 512, 8192, 1), (112, 512, 8192, 1), (160, 256, 8192, 1),
])
def test_gemm_vs_oracle(M, N, K, splits):
    qw, sc = _weights(K, N, M * 7 + N)
    g = torch.Generator().manual_seed(M)
    X = torch.randn(M, K, generator=g).half()
    Y = quant.w4a16_linear(X.cuda(), qw.cuda(), sc.cuda(), splits=splits).float().cpu()
    ref = torch.from_numpy(wo.gemm(X.numpy(), quant.unpack_int4(qw).numpy().astype(np.uint8), sc.numpy()))
    assert _lib.device_error() == 0
    scale = ref.abs().max().item() + 1e-6
    err = (Y - ref).abs().max().item()
    # fp16 output rounding (2^-11 relative) plus fp32 accumulation order
    assert err <= 2e-3 * scale + 1e-3, f"max err {err:.3e} (max |ref| {scale:.3e})"


def test_gemm_strided_activations():
    K, N, M = 1024, 256, 96
    qw, sc = _weights(K, N, 5)
    g = torch.Generator().manual_seed(9)
    big = torch.randn(M, 2 * K, generator=g).half().cuda()
    X = big[:, :K]  # row stride 2K
    Y = quant.w4a16_linear(X, qw.cuda(), sc.cuda())
    Y2 = quant.w4a16_linear(X.contiguous(), qw.cuda(), sc.cuda())
    assert torch.equal(Y, Y2)


def test_gemm_on_gptq_checkpoint_tensors():
    # a GPTQ-format linear (qweight [K/8, N], classic zero-1 qzeros, g_idx) loaded by
    # quant.from_gptq runs through the GEMM like a natively quantised one
    K, N, M = 1024, 384, 48
    qw, sc = _weights(K, N, 21)
    gq, gs, gz, gi = quant.to_gptq(qw, sc)
    qw2, sc2 = quant.from_gptq(gq, gs, gz, gi)
    g = torch.Generator().manual_seed(22)
    X = torch.randn(M, K, generator=g).half()
    Y = quant.w4a16_linear(X.cuda(), qw2.cuda(), sc2.cuda()).float().cpu()
    q = quant.unpack_int4(qw2).numpy().astype(np.uint8)
    ref = torch.from_numpy(wo.gemm(X.numpy(), q, sc2.numpy()))
    scale = ref.abs().max().item() + 1e-6
    assert (Y - ref).abs().max().item() <= 2e-3 * scale + 1e-3
    assert torch.equal(qw2, qw) and torch.equal(sc2, sc)


# The four W4A16 GEMMs of one Llama-3.1-8B decoder layer as the bench runs them
# (q/k/v and gate/up fused along N; the linears the reference's E2E script runs
# through Marlin, scripts/w4a16_e2e.py:698-699), at the token counts of the
# bench sweep. The automatic split count is what the bench uses (qkv 6, o 8,
# down 9 and gate_up 1 at small M), and M = 8184 takes the large-M tile shape.
# The fp64 oracle runs on a fixed sample of 64 rows x every column.
LLAMA_LAYER = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 28672), ("down", 14336, 4096)]
_layer_cache = {}


def _layer_weights(name, K, N):
    if name not in _layer_cache:
        qw, sc = _weights(K, N, 1000 + [n for n, _, _ in LLAMA_LAYER].index(name))
        q = quant.unpack_int4(qw).numpy().astype(np.uint8)
        _layer_cache[name] = (qw.cuda(), sc.cuda(), wo.dequantize(q, sc.numpy()))  # W' fp16 [K, N]
    return _layer_cache[name]


def _oracle_rows(Xs, W):
    """fp64 product of sampled activation rows with the dequantised weights, column chunk by chunk."""
    out = np.empty((Xs.shape[0], W.shape[1]), dtype=np.float32)
    X64 = Xs.astype(np.float64)
    for c in range(0, W.shape[1], 4096):
        out[:, c:c + 4096] = X64 @ W[:, c:c + 4096].astype(np.float64)
    return out


@pytest.mark.parametrize("name,K,N", LLAMA_LAYER)
@pytest.mark.parametrize("M", [16, 64, 1023, 8184])
def test_llama_layer_shapes_vs_oracle(name, K, N, M):
    import ctypes
    qw, sc, W = _layer_weights(name, K, N)
    g = torch.Generator().manual_seed(M + K + N)
    X = torch.randn(M, K, generator=g).half()
    Y = quant.w4a16_linear(X.cuda(), qw, sc).float().cpu()
    assert _lib.device_error() == 0
    rows = torch.unique(torch.cat([torch.tensor([0, M - 1]),
                                   torch.randint(0, M, (62,), generator=g)]))[:64] if M > 64 else torch.arange(M)
    ref = torch.from_numpy(_oracle_rows(X[rows].numpy(), W))
    scale = ref.abs().max().item() + 1e-6
    err = (Y[rows] - ref).abs().max().item()
    sp, wb = ctypes.c_int32(), ctypes.c_int64()
    _lib.check(_lib.lib().qa_w4a16_plan(M, N, K, ctypes.byref(sp), ctypes.byref(wb)), "qa_w4a16_plan")
    assert err <= 2e-3 * scale + 1e-3, f"{name} M={M} splits={sp.value}: max err {err:.3e} (max |ref| {scale:.3e})"
    assert torch.isfinite(Y).all()
