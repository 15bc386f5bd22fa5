"""The allocation-free W4A16 entry point agrees with the regular one.

qa_w4a16_gemm_noalloc exists for callers that may not call cudaMalloc while
they run (their host framework only lends them buffers it owns, or an
allocation's implicit device synchronisation would stall a serving loop). It
keeps the split-K partial sums in a fixed array inside the library instead of a
caller-provided workspace. This test calls it through the C ABI, twice in a
row on different shapes (the shared array then holds the previous call's
contents) and once more on the first shape, and compares each result with
qa_w4a16_gemm given a freshly allocated workspace, within the tolerance the
other W4A16 tests use. The file is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qattention_b200 import _lib, quant


def _args(x, qw, sc, y, ws, M, N, K, splits):
    a = _lib.W4A16Args()
    a.x, a.qweight, a.scales, a.y = x.data_ptr(), qw.data_ptr(), sc.data_ptr(), y.data_ptr()
    a.workspace = ws.data_ptr() if ws is not None else None
    a.x_stride, a.y_stride = x.stride(0), y.stride(0)
    a.M, a.N, a.K, a.splits = M, N, K, splits
    return a


def _pair(M, N, K, splits, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(K, N, generator=g) * 0.02
    qw, sc = (t.cuda() for t in quant.quantize_w4a16(W))
    x = torch.randn(M, K, generator=g).half().cuda()
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    y_ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ws = torch.empty(max(splits, 32) * M * N, dtype=torch.float32, device="cuda")
    assert L.qa_w4a16_gemm(_args(x, qw, sc, y_ref, ws, M, N, K, splits), stream) == 0
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    assert L.qa_w4a16_gemm_noalloc(_args(x, qw, sc, y, None, M, N, K, splits), stream) == 0
    torch.cuda.synchronize()
    return y.float().cpu(), y_ref.float().cpu()


def _close(y, y_ref):
    scale = y_ref.abs().max().item() + 1e-6
    assert torch.isfinite(y).all()
    assert (y - y_ref).abs().max().item() <= 2e-3 * scale + 1e-3


def test_noalloc_matches_allocating_entry_point_two_calls_in_a_row():
    first = (16, 1024, 4096, 4, 1)
    second = (40, 256, 1024, 2, 2)
    for M, N, K, splits, seed in (first, second, first):
        y, y_ref = _pair(M, N, K, splits, seed)
        _close(y, y_ref)
    assert _lib.device_error() == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    # 8 splits x 64 x 14336 fp32 partials = 29 MB > the 16 MiB array
    g = torch.Generator().manual_seed(3)
    qw, sc = (t.cuda() for t in quant.quantize_w4a16(torch.randn(4096, 14336, generator=g) * 0.02))
    x = torch.randn(64, 4096, generator=g).half().cuda()
    y = torch.empty(64, 14336, dtype=torch.float16, device="cuda")
    rc = _lib.lib().qa_w4a16_gemm_noalloc(_args(x, qw, sc, y, None, 64, 14336, 4096, 8),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == -1


@pytest.mark.parametrize("M,N,K,splits", [
    (24, 512, 1024, 0),     # automatic split count, small shape
    (64, 14336, 4096, 0),   # automatic: 8 splits would not fit the array, so it steps down
    (16, 256, 512, 9),      # more splits than K steps (4): clamped before the size check
    (32, 1024, 2048, 1),    # one split: no scratch at all
])
def test_noalloc_split_resolution(M, N, K, splits):
    y, y_ref = _pair(M, N, K, splits, 11)
    _close(y, y_ref)
    assert _lib.device_error() == 0
