"""GPU parity of the tensor-core prefix pass and of prefix + tree verification.

Oracles: dense fp32 attention over the prefix (every key visible), and the
reference's rectangular [N, L+N] masked SDPA for hybrid/E2E layouts
(tests/test_correctness.py:402-469 of the reference), GQA expanded like
repeat_kv. Tolerance atol = rtol = 1e-2 on outputs (the reference's regime),
1e-3 on LSE.
"""
import math

import numpy as np
import pytest
import torch

from oracle import tree_attn_oracle as orc

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-2

if torch.cuda.is_available():
    from qattention_b200 import _lib
    from qattention_b200 import ragged_attn as ra
    from qattention_b200 import tree_mask as tm


def _prefix_oracle(Q, K, V):
    """Q [B,N,Hq,D], K/V [B,L,Hkv,D] -> O [B,N,Hq,D] fp32, LSE [B,N,Hq]."""
    B, N, Hq, D = Q.shape
    r = Hq // K.shape[2]
    k = K.float().repeat_interleave(r, dim=2)
    v = V.float().repeat_interleave(r, dim=2)
    s = torch.einsum("bnhd,blhd->bhnl", Q.float(), k) / math.sqrt(D)
    o = torch.einsum("bhnl,blhd->bnhd", torch.softmax(s, -1), v)
    return o, torch.logsumexp(s, -1).permute(0, 2, 1)


@pytest.mark.parametrize("B,N,L,Hq,Hkv,D", [
    (1, 16, 64, 1, 1, 128),
    (2, 31, 100, 4, 4, 128),
    (2, 50, 64, 2, 2, 64),
    (1, 85, 640, 8, 2, 128),
    (2, 33, 257, 8, 1, 128),
    (3, 7, 1, 4, 2, 64),
])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefix_vs_oracle(B, N, L, Hq, Hkv, D, dtype):
    g = torch.Generator().manual_seed(B * 1000 + N + L)
    Q = torch.randn(B, N, Hq, D, generator=g).to(dtype)
    K = torch.randn(B, L, Hkv, D, generator=g).to(dtype)
    V = torch.randn(B, L, Hkv, D, generator=g).to(dtype)
    O, LSE = ra.prefix_attention_with_lse(Q.cuda(), K.cuda(), V.cuda())
    ro, rl = _prefix_oracle(Q, K, V)
    assert _lib.device_error() == 0
    err = (O.float().cpu() - ro).abs().max().item()
    assert torch.allclose(O.float().cpu(), ro, atol=ATOL, rtol=RTOL), f"max err {err:.3e}"
    assert (LSE.cpu() - rl).abs().max().item() <= 1e-3


def test_prefix_strided_hf_layout():
    # K/V as [B, Hkv, L, D] tensors (HF cache layout) passed as permuted views
    B, N, L, Hq, Hkv, D = 2, 40, 200, 8, 2, 128
    g = torch.Generator().manual_seed(5)
    Q = torch.randn(B, Hq, N, D, generator=g).half().cuda()
    K = torch.randn(B, Hkv, L, D, generator=g).half().cuda()
    V = torch.randn(B, Hkv, L, D, generator=g).half().cuda()
    O, LSE = ra.prefix_attention_with_lse(Q.permute(0, 2, 1, 3), K.permute(0, 2, 1, 3), V.permute(0, 2, 1, 3))
    ro, rl = _prefix_oracle(Q.permute(0, 2, 1, 3).cpu(), K.permute(0, 2, 1, 3).cpu(), V.permute(0, 2, 1, 3).cpu())
    assert torch.allclose(O.float().cpu(), ro, atol=ATOL, rtol=RTOL)
    assert (LSE.cpu() - rl).abs().max().item() <= 1e-3


@pytest.mark.parametrize("B,b,d", [(1, 2, 3), (4, 2, 5), (4, 3, 5), (8, 2, 5), (8, 3, 5), (4, 4, 4), (2, 8, 3)])
def test_hybrid_parity_with_base(B, b, d):
    """Mirror of the reference's hybrid test: L=0 equals the base kernel, L=32 equals masked SDPA."""
    torch.manual_seed(B * 100 + b * 10 + d)
    N = tm.num_tree_nodes(b, d)
    H, D = 4, 64
    Q, K, V = (torch.randn(B * N, H, D).half() for _ in range(3))
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32)
    O_base = ra.ragged_attention(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    O0 = ra.ragged_attention_hybrid(Q.cuda(), K.cuda(), V.cuda(), 0, N, b, d)
    assert torch.allclose(O_base.float(), O0.float(), atol=ATOL, rtol=RTOL)
    L = 32
    Kp, Vp = torch.randn(B, L, H, D).half(), torch.randn(B, L, H, D).half()
    Kh = torch.cat([Kp, K.view(B, N, H, D)], 1).reshape(B * (L + N), H, D)
    Vh = torch.cat([Vp, V.view(B, N, H, D)], 1).reshape(B * (L + N), H, D)
    OL = ra.ragged_attention_hybrid(Q.cuda(), Kh.cuda(), Vh.cuda(), L, N, b, d).float().cpu()
    mask = tm.tree_attention_mask(b, d)
    for s in range(B):
        sl = slice(s * N, (s + 1) * N)
        ref = orc.prefix_tree_sdpa(Q[sl], Kp[s], Vp[s], K[sl], V[sl], mask)
        assert torch.allclose(OL[sl], ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("use_parents", [False, True])
def test_tree_verify_attention_e2e_layout(use_parents):
    # scripts/w4a16_e2e.py:_ragged_tree_attn layout: Q [B,Hq,N,D], K/V [B,Hkv,L+N,D]
    B, b, d, Hq, Hkv, D, L = 2, 3, 3, 8, 2, 128, 300
    if use_parents:
        tree = tm.build_pruned_tree(b, d, rng=np.random.default_rng(3))
        parents = torch.from_numpy(tm.kernel_parents(tree))
    else:
        tree, parents = tm.build_tree(b, d), None
    N = len(tree)
    g = torch.Generator().manual_seed(11)
    Q = torch.randn(B, Hq, N, D, generator=g).half()
    K = torch.randn(B, Hkv, L + N, D, generator=g).half()
    V = torch.randn(B, Hkv, L + N, D, generator=g).half()
    out = ra.tree_verify_attention(Q.cuda(), K.cuda(), V.cuda(), b, d, tree_parents=parents)
    assert out.shape == (B, Hq, N, D)
    if use_parents:  # one plan shared by the layers of a verify step: same bits
        plan = ra.plan_tree_parents(parents, B, d, device="cuda")
        out2 = ra.tree_verify_attention(Q.cuda(), K.cuda(), V.cuda(), b, d, tree_parents=parents, plan=plan)
        assert torch.equal(out2, out)
    mask = tm.tree_attention_mask_pruned(tree)
    for s in range(B):
        q = Q[s].permute(1, 0, 2)
        kk, vv = K[s].permute(1, 0, 2), V[s].permute(1, 0, 2)
        ref = orc.prefix_tree_sdpa(q, kk[:L], vv[:L], kk[L:], vv[L:], mask)
        assert torch.allclose(out[s].permute(1, 0, 2).float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_config4_full_size_first_sequence():
    """bench config C4: B=16, L=10240, 4-ary depth-4 trees (N=341), GQA 32/8, D=128."""
    B, L, b, d, Hq, Hkv, D = 16, 10240, 4, 4, 32, 8, 128
    N = tm.num_tree_nodes(b, d)
    g = torch.Generator().manual_seed(4)
    Q = torch.randn(B, Hq, N, D, generator=g).half()
    K = torch.randn(B, Hkv, L + N, D, generator=g).half()
    V = torch.randn(B, Hkv, L + N, D, generator=g).half()
    out = ra.tree_verify_attention(Q.cuda(), K.cuda(), V.cuda(), b, d).float().cpu()
    assert _lib.device_error() == 0
    assert torch.isfinite(out).all()
    mask = tm.tree_attention_mask(b, d)
    for s in (0, B - 1):
        q = Q[s].permute(1, 0, 2)
        kk, vv = K[s].permute(1, 0, 2), V[s].permute(1, 0, 2)
        ref = orc.prefix_tree_sdpa(q, kk[:L], vv[:L], kk[L:], vv[L:], mask)
        assert torch.allclose(out[s].permute(1, 0, 2), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("L", [0, 200])
@pytest.mark.parametrize("use_parents", [False, True])
def test_tree_verify_query_layouts_read_in_place(L, use_parents):
    # The queries are read in place in three layouts: a contiguous [B, Hq, N, D]
    # tensor (the kernel's batch stride), a head slice of a fused qkv projection
    # (packed rows, one token stride) and an odd offset that forces the copy.
    # All three must give bit-identical results.
    B, b, d, Hq, Hkv, D = 3, 2, 5, 8, 2, 64
    if use_parents:
        tree = tm.build_pruned_tree(b, d, rng=np.random.default_rng(5))
        parents = torch.from_numpy(tm.kernel_parents(tree))
    else:
        tree, parents = tm.build_tree(b, d), None
    N = len(tree)
    g = torch.Generator().manual_seed(17)
    K = torch.randn(B, Hkv, L + N, D, generator=g).half().cuda()
    V = torch.randn(B, Hkv, L + N, D, generator=g).half().cuda()
    Q = torch.randn(B, Hq, N, D, generator=g).half().cuda()
    qkv = torch.zeros(B, N, Hq + 2 * Hkv, D, dtype=torch.float16, device="cuda")
    qkv[:, :, :Hq] = Q.permute(0, 2, 1, 3)
    q_slice = qkv[:, :, :Hq].permute(0, 2, 1, 3)                  # [B, Hq, N, D] view, token pitch (Hq+2Hkv)D
    buf = torch.zeros(B * Hq * N * D + 4, dtype=torch.float16, device="cuda")
    q_odd = buf[4:].view(B, Hq, N, D)                              # 8-byte offset: not 16-byte aligned
    q_odd.copy_(Q)
    outs = [ra.tree_verify_attention(q, K, V, b, d, tree_parents=parents) for q in (Q, q_slice, q_odd)]
    assert _lib.device_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    mask = tm.tree_attention_mask_pruned(tree)
    for s in (0, B - 1):
        q = Q[s].permute(1, 0, 2).cpu()
        kk, vv = K[s].permute(1, 0, 2).cpu(), V[s].permute(1, 0, 2).cpu()
        ref = orc.prefix_tree_sdpa(q, kk[:L], vv[:L], kk[L:], vv[L:], mask)
        assert torch.allclose(outs[0][s].permute(1, 0, 2).float().cpu(), ref, atol=ATOL, rtol=RTOL)
