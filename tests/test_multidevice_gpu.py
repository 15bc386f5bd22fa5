"""One process, two GPUs: every kernel launches on a second device after the first.

Kernel attributes (the dynamic shared-memory limit above 48 KB) and the SM
count are per device, so the library keeps them per device. Each hot-path
kernel runs on cuda:0, then on cuda:1 with that device current, on the same
inputs, and the two results must be bit-identical. Skipped with one GPU.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qattention_b200 import _lib, quant
    from qattention_b200 import ragged_attn as ra

two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs two visible GPUs")


def _on(dev_index, fn, *host_tensors):
    dev = torch.device("cuda", dev_index)
    with torch.cuda.device(dev):
        out = fn(*(t.to(dev) for t in host_tensors))
        torch.cuda.synchronize(dev)
        assert _lib.device_error() == 0
    return [o.cpu() for o in (out if isinstance(out, (tuple, list)) else (out,))]


@two_gpus
def test_ancestor_tile_and_walk_kernels_on_second_device():
    g = torch.Generator().manual_seed(21)
    b, d, B, H, D = 4, 4, 3, 8, 128
    N = (b ** (d + 1) - 1) // (b - 1)
    Q, K, V = (torch.randn(B * N, H, D, generator=g).half() for _ in range(3))
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32)
    par = torch.tensor([0] + [(i - 1) // b for i in range(1, N)], dtype=torch.int32).repeat(B)
    tile = lambda q, k, v: ra.ragged_attention_with_lse(q, k, v, cu, b, d)
    walk = lambda q, k, v: ra.ragged_attention_with_parents(q, k, v, cu, par, d)
    for fn in (tile, walk):
        r0 = _on(0, fn, Q, K, V)
        r1 = _on(1, fn, Q, K, V)
        for a, c in zip(r0, r1):
            assert torch.equal(a, c)


@two_gpus
def test_prefix_pass_on_second_device():
    g = torch.Generator().manual_seed(22)
    B, L, N, Hq, Hkv, D = 2, 640, 85, 8, 2, 128
    Q = torch.randn(B, N, Hq, D, generator=g).half()
    K = torch.randn(B, L, Hkv, D, generator=g).half()
    V = torch.randn(B, L, Hkv, D, generator=g).half()
    r0 = _on(0, ra.prefix_attention_with_lse, Q, K, V)
    r1 = _on(1, ra.prefix_attention_with_lse, Q, K, V)
    for a, c in zip(r0, r1):
        assert torch.equal(a, c)


@two_gpus
def test_w4a16_gemm_and_noalloc_on_second_device():
    import ctypes
    g = torch.Generator().manual_seed(23)
    M, K, N = 64, 4096, 4096
    qw, sc = quant.quantize_w4a16(torch.randn(K, N, generator=g) * 0.02)
    X = torch.randn(M, K, generator=g).half()
    r0 = _on(0, quant.w4a16_linear, X, qw, sc)
    r1 = _on(1, quant.w4a16_linear, X, qw, sc)
    assert torch.equal(r0[0], r1[0])

    def noalloc(x, q, s):
        y = torch.empty(M, N, dtype=torch.float16, device=x.device)
        a = _lib.W4A16Args()
        a.x, a.qweight, a.scales, a.y = x.data_ptr(), q.data_ptr(), s.data_ptr(), y.data_ptr()
        a.workspace = None
        a.x_stride, a.y_stride = x.stride(0), y.stride(0)
        a.M, a.N, a.K, a.splits = M, N, K, 4
        assert _lib.lib().qa_w4a16_gemm_noalloc(ctypes.byref(a),
                                                torch.cuda.current_stream(x.device).cuda_stream) == 0
        return y

    n0 = _on(0, noalloc, X, qw, sc)
    n1 = _on(1, noalloc, X, qw, sc)
    assert torch.equal(n0[0], n1[0])
    scale = r0[0].float().abs().max().item()
    assert (n1[0].float() - r0[0].float()).abs().max().item() <= 2e-3 * scale + 1e-3
