"""Host-buffer ancestor attention with overlapped copies: bit-identical to the device path."""
import pytest
import torch

from qattention_b200.host_pipeline import chunk_bounds

gpu = pytest.mark.gpu


def test_chunk_bounds_cover_every_tree_once():
    cu = [0, 10, 20, 30, 40]
    for chunks in (1, 2, 3, 4, 8):
        pts = chunk_bounds(cu, chunks)
        assert pts[0] == 0 and pts[-1] == 4 and pts == sorted(set(pts))
        assert len(pts) - 1 <= chunks
    assert chunk_bounds([0, 5, 100, 105], 2) == [0, 2, 3]  # cut nearest half of the tokens
    assert chunk_bounds([0, 7], 4) == [0, 1]
    assert chunk_bounds([0, 1023, 2046], 8) == [0, 1, 2]  # two trees: two chunks, not one


def _batch(lengths, H, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(lengths)
    Q, K, V = (torch.randn(T, H, D, generator=g).to(dtype) for _ in range(3))
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0).tolist()), dtype=torch.int32)
    return Q, K, V, cu


@gpu
@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_host_pipeline_matches_device_path(chunks, dtype):
    from qattention_b200 import ragged_attn as ra
    from qattention_b200.host_pipeline import ragged_attention_with_lse_host

    b, d, H, D = 2, 6, 4, 128
    lengths = [127, 100, 64, 127, 1, 127, 90]  # complete and truncated BFS trees
    Q, K, V, cu = _batch(lengths, H, D, dtype, 3)
    O_ref, L_ref = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    torch.cuda.synchronize()
    O, L = ragged_attention_with_lse_host(Q.pin_memory(), K.pin_memory(), V.pin_memory(), cu, b, d,
                                          chunks=chunks)
    assert not O.is_cuda and not L.is_cuda
    assert torch.equal(O, O_ref.cpu())
    assert torch.equal(L, L_ref.cpu())


@gpu
def test_host_pipeline_full_size_c3_against_device_path():
    from qattention_b200 import ragged_attn as ra
    from qattention_b200.host_pipeline import ragged_attention_with_lse_host

    b, d, H, D, B = 2, 9, 32, 128, 16
    Q, K, V, cu = _batch([1023] * B, H, D, torch.float16, 9)
    O_ref, L_ref = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    torch.cuda.synchronize()
    out = torch.empty_like(Q).pin_memory()
    lse = torch.empty(Q.shape[0], H, dtype=torch.float32).pin_memory()
    for _ in range(2):  # the second call reuses the streams and the caller's outputs
        O, L = ragged_attention_with_lse_host(Q.pin_memory(), K.pin_memory(), V.pin_memory(), cu, b, d,
                                              out=out, lse_out=lse)
        assert O.data_ptr() == out.data_ptr()
        assert torch.equal(O, O_ref.cpu()) and torch.equal(L, L_ref.cpu())


@gpu
def test_host_pipeline_rejects_device_tensors():
    from qattention_b200.host_pipeline import ragged_attention_with_lse_host

    Q, K, V, cu = _batch([15], 2, 64, torch.float16, 1)
    with pytest.raises(ValueError):
        ragged_attention_with_lse_host(Q.cuda(), K, V, cu, 2, 3)
