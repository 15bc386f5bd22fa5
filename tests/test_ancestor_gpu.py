"""GPU parity of the ancestor-walk kernel against the CPU oracle (reference restatement).

Mirrors the reference suite tests/test_correctness.py:254-350 (72-config sweep,
benchmark shapes, head dims, single token, linear chain) with the same
tolerance (atol = rtol = 1e-2 vs an fp32 padded masked SDPA), plus golden
fixtures produced by the reference itself, LSE, explicit parents, ragged and
truncated trees, strided views, GQA, bf16 and full-size sliced checks.
"""
import itertools
import math

import numpy as np
import pytest
import torch

from oracle import tree_attn_oracle as orc
from tests.golden.make_golden import SDPA_CASES

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2

if torch.cuda.is_available():
    from qattention_b200 import ragged_attn as ra
    from qattention_b200 import tree_mask as tm


def _gen(seed, n, H, D, B, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    mk = lambda: [torch.randn(n, H, D, generator=g).to(dtype) for _ in range(B)]  # noqa: E731
    return mk(), mk(), mk()


def _check(B, b, d, H, D, dtype=torch.float16):
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(B * 100 + b * 10 + d, N, H, D, B, dtype)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    O = ra.ragged_attention(Q.cuda(), K.cuda(), V.cuda(), cu, branching_factor=b, max_depth=d)
    ref = torch.cat(orc.padded_sdpa(qs, ks, vs, [tm.tree_attention_mask(b, d)] * B), 0)
    out = O.float().cpu()
    assert O.dtype == dtype and O.shape == Q.shape
    err = (out - ref).abs().max().item()
    assert torch.allclose(out, ref, atol=ATOL, rtol=RTOL), f"B={B} b={b} d={d} peak_abs={err:.3e}"
    return err


@pytest.mark.parametrize("B,b,d", list(itertools.product([1, 2, 4, 8], [1, 2, 3], [1, 2, 3, 4, 5, 6])))
def test_ragged_vs_sdpa(B, b, d):
    _check(B, b, d, 4, 64)


@pytest.mark.parametrize("B,b,d", [(4, 2, 5), (4, 3, 5), (8, 2, 5), (8, 3, 5), (4, 2, 6), (4, 3, 6)])
def test_benchmark_configs(B, b, d):
    _check(B, b, d, 8, 128)


@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_head_dims(D):
    _check(4, 2, 3, 4, D)


def test_single_token():
    _check(4, 1, 0, 4, 64)


def test_linear_chain():
    _check(4, 1, 8, 4, 64)


@pytest.mark.parametrize("b,d", [(4, 3), (5, 2), (8, 2), (28, 1)])
def test_wide_trees(b, d):
    # b > 4 splits siblings into register chunks of 4
    _check(2, b, d, 4, 64)


@pytest.mark.parametrize("b,d", [(2, 4), (3, 3)])
def test_bf16(b, d):
    _check(2, b, d, 4, 64, dtype=torch.bfloat16)


@pytest.mark.parametrize("case", [c[0] for c in SDPA_CASES])
def test_golden_fixtures(golden, case):
    c = golden["sdpa_cases"]
    B, b, d, H, D = (int(x) for x in c[f"{case}_meta"])
    Q, K, V = (torch.from_numpy(c[f"{case}_{x}"]).cuda() for x in "qkv")
    cu = torch.from_numpy(c[f"{case}_cu"])
    O = ra.ragged_attention(Q, K, V, cu, b, d)
    ref = torch.from_numpy(c[f"{case}_out"]).float()
    assert torch.allclose(O.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_config1_fp32_inputs(golden):
    # bench config C1 draws fp32 inputs; the kernel computes from their fp16 cast.
    c = golden["sdpa_cases"]
    q, k, v = (torch.from_numpy(c[f"c1_{x}"]) for x in "qkv")
    cu = torch.tensor([0, q.shape[0]], dtype=torch.int32)
    O = ra.ragged_attention(q.half().cuda(), k.half().cuda(), v.half().cuda(), cu, 2, 3)
    ref = torch.from_numpy(c["c1_out"]).float()
    assert (O.float().cpu() - ref).abs().max().item() <= ATOL


def test_lse_matches_oracle():
    B, b, d, H, D = 3, 3, 4, 4, 64
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(7, N, H, D, B)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    O, L = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    ro, rl = orc.sparse_ancestor_attention(Q, K, V, cu, b, d)
    assert L.dtype == torch.float32 and L.shape == (B * N, H)
    assert torch.allclose(L.cpu().double(), rl, atol=1e-4)
    assert torch.allclose(O.float().cpu(), ro.float(), atol=ATOL, rtol=RTOL)
    O2 = ra.ragged_attention(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    assert torch.equal(O2, O)


def test_ragged_lengths_and_truncated_depth():
    # sequences that are not complete trees, and max_depth below the true depth
    H, D, b, d = 4, 64, 2, 3
    lens = [15, 9, 1, 40, 2]
    g = torch.Generator().manual_seed(3)
    qs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    ks = [torch.randn(n, H, D, generator=g).half() for n in lens]
    vs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    O, L = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    masks = [orc.ancestor_mask(n, b, d) for n in lens]
    ref, rl = orc.padded_sdpa(qs, ks, vs, masks, return_lse=True)
    assert torch.allclose(O.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL)
    assert torch.allclose(L.cpu(), torch.cat(rl, 0), atol=1e-3)


@pytest.mark.parametrize("b,d,target,seed", [(2, 4, None, 11), (3, 4, 30, 12), (4, 5, 60, 13), (1, 6, None, 14)])
def test_explicit_parents_pruned_trees(b, d, target, seed):
    H, D, B = 4, 64, 3
    rng = np.random.default_rng(seed)
    trees = [tm.build_pruned_tree(b, d, target_nodes=target, rng=rng) for _ in range(B)]
    g = torch.Generator().manual_seed(seed)
    qs = [torch.randn(len(t), H, D, generator=g).half() for t in trees]
    ks = [torch.randn(len(t), H, D, generator=g).half() for t in trees]
    vs = [torch.randn(len(t), H, D, generator=g).half() for t in trees]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    parents = torch.from_numpy(np.concatenate([tm.kernel_parents(t) for t in trees]))
    O, L = ra.ragged_attention_with_parents(Q.cuda(), K.cuda(), V.cuda(), cu, parents, d)
    masks = [tm.tree_attention_mask_pruned(t) for t in trees]
    ref, rl = orc.padded_sdpa(qs, ks, vs, masks, return_lse=True)
    assert torch.allclose(O.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL)
    assert torch.allclose(L.cpu(), torch.cat(rl, 0), atol=1e-3)


@pytest.mark.parametrize("b,d,target,seed,D,dtype", [
    (8, 5, 1365, 21, 128, torch.float16),   # C2-sized pruned trees: every tile on the key lists
    (4, 6, 1365, 22, 128, torch.float16),   # tiles past the staged rows: walk warps
    (3, 7, 1365, 23, 64, torch.float16),
    (4, 5, 1365, 24, 256, torch.bfloat16),
    (2, 12, 3000, 25, 128, torch.float16),  # deep walks (13 keys per row)
])
def test_explicit_parents_large_pruned_trees(b, d, target, seed, D, dtype):
    # the reference's E2E verify path (ragged_attention_with_parents on EAGLE-style
    # pruned trees, scripts/w4a16_e2e.py:1277-1284), at C2-like sizes on the tile path
    H, B = 8, 3
    rng = np.random.default_rng(seed)
    trees = [tm.build_pruned_tree(b, d, target_nodes=target, rng=rng) for _ in range(B)]
    g = torch.Generator().manual_seed(seed)
    qs = [torch.randn(len(t), H, D, generator=g).to(dtype) for t in trees]
    ks = [torch.randn(len(t), H, D, generator=g).to(dtype) for t in trees]
    vs = [torch.randn(len(t), H, D, generator=g).to(dtype) for t in trees]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    parents = torch.from_numpy(np.concatenate([tm.kernel_parents(t) for t in trees]))
    O, L = ra.ragged_attention_with_parents(Q.cuda(), K.cuda(), V.cuda(), cu, parents, d)
    from qattention_b200 import _lib
    assert _lib.ancestor_diagnostics()[0] == 0
    ro, rl = orc.sparse_ancestor_attention(Q, K, V, cu, 0, d, parents=parents, dtype=torch.float32)
    assert torch.allclose(O.float().cpu(), ro, atol=ATOL, rtol=RTOL)
    assert torch.allclose(L.cpu(), rl, atol=1e-3)
    # plans made once and reused give the same bits
    plan = ra.plan_parents(cu, parents, d, device="cuda")
    assert plan is not None
    for _ in range(2):
        O2, L2 = ra.ragged_attention_with_parents(Q.cuda(), K.cuda(), V.cuda(), cu, parents, d, plan=plan)
        assert torch.equal(O2, O) and torch.equal(L2, L)


def test_explicit_parents_gqa_paged_and_strided():
    # GQA, a page table and strided query views on the explicit-parent tile path
    b, d, H, Hkv, D, page = 4, 5, 8, 2, 128, 16
    rng = np.random.default_rng(31)
    trees = [tm.build_pruned_tree(b, d, target_nodes=400, rng=rng) for _ in range(3)]
    lens = [len(t) for t in trees]
    g = torch.Generator().manual_seed(31)
    qs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    ks = [torch.randn(n, Hkv, D, generator=g).half() for n in lens]
    vs = [torch.randn(n, Hkv, D, generator=g).half() for n in lens]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    parents = torch.from_numpy(np.concatenate([tm.kernel_parents(t) for t in trees]))
    Qs = torch.zeros(Q.shape[0], H, 2 * D, dtype=torch.float16)
    Qs[:, :, :D] = Q
    O, L = ra.ragged_attention_with_parents(Qs.cuda()[:, :, :D], K.cuda(), V.cuda(), cu, parents, d)
    rep = H // Hkv
    ro, rl = orc.sparse_ancestor_attention(Q, K, V, cu, 0, d, parents=parents, dtype=torch.float32)
    assert torch.allclose(O.float().cpu(), ro, atol=ATOL, rtol=RTOL)
    # paged K/V through the C ABI: the same plans, rows looked up in the page table
    Kc, Vc, pt = ra.build_paged_kv(ks, vs, page_size=page)
    from qattention_b200 import _lib
    import ctypes, math
    Qd, Kd, Vd = Q.cuda(), Kc.cuda(), Vc.cuda()
    Od = torch.empty_like(Qd)
    ptd, cud, pard = pt.cuda(), cu.cuda(), parents.cuda().int()
    a = _lib.AncestorArgs()
    a.q, a.k, a.v, a.o = Qd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), Od.data_ptr()
    a.cu_seqlens_q, a.parents = cud.data_ptr(), pard.data_ptr()
    a.q_stride_t, a.q_stride_h = Qd.stride(0), Qd.stride(1)
    a.k_stride_t, a.k_stride_h, a.k_stride_page = Kd.stride(1), Kd.stride(2), Kd.stride(0)
    a.v_stride_t, a.v_stride_h, a.v_stride_page = Vd.stride(1), Vd.stride(2), Vd.stride(0)
    a.o_stride_t, a.o_stride_h = Od.stride(0), Od.stride(1)
    a.page_table, a.page_table_stride, a.page_size = ptd.data_ptr(), ptd.stride(0), page
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = 3, H, Hkv, D
    a.max_depth, a.max_seqlen, a.scale, a.dtype = d, max(lens), 1.0 / math.sqrt(D), _lib.QA_DTYPE_F16
    need = ctypes.c_int64(0)
    assert _lib.lib().qa_ancestor_workspace_bytes(a, ctypes.byref(need)) == 0 and need.value > 0
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
    assert _lib.lib().qa_ancestor_attn(a, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.allclose(Od.float().cpu(), ro, atol=ATOL, rtol=RTOL)
    # without a workspace the per-query walk serves the call: same results within tolerance
    a.workspace, a.workspace_bytes = None, 0
    Od2 = torch.empty_like(Qd)
    a.o = Od2.data_ptr()
    assert _lib.lib().qa_ancestor_attn(a, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert (Od2.float() - Od.float()).abs().max().item() <= 2e-3
    assert _lib.ancestor_diagnostics()[0] == 0


def test_parents_path_equals_formula_on_complete_tree():
    B, b, d, H, D = 2, 3, 4, 4, 64
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(9, N, H, D, B)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    par = torch.from_numpy(np.tile(tm.kernel_parents(tm.build_tree(b, d)), B))
    Of, Lf = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    Op, Lp = ra.ragged_attention_with_parents(Q.cuda(), K.cuda(), V.cuda(), cu, par, d)
    assert (Of.float() - Op.float()).abs().max().item() <= 2e-3
    assert (Lf - Lp).abs().max().item() <= 1e-5


def test_strided_views_b1_layout():
    # the E2E caller passes [N, H, D] transposed views of [H, N, D] (scripts/w4a16_e2e.py:1262-1265)
    b, d, H, D = 2, 4, 8, 128
    N = tm.num_tree_nodes(b, d)
    g = torch.Generator().manual_seed(4)
    base = [torch.randn(H, N, D, generator=g).half().cuda() for _ in range(3)]
    Qv, Kv, Vv = (t.transpose(0, 1) for t in base)
    cu = torch.tensor([0, N], dtype=torch.int32)
    O = ra.ragged_attention(Qv, Kv, Vv, cu, b, d)
    O_ref = ra.ragged_attention(Qv.contiguous(), Kv.contiguous(), Vv.contiguous(), cu, b, d)
    assert torch.equal(O, O_ref)


def test_gqa_heads():
    b, d, Hq, Hkv, D, B = 4, 3, 8, 2, 128, 2
    N = tm.num_tree_nodes(b, d)
    g = torch.Generator().manual_seed(8)
    Q = torch.randn(B * N, Hq, D, generator=g).half()
    K = torch.randn(B * N, Hkv, D, generator=g).half()
    V = torch.randn(B * N, Hkv, D, generator=g).half()
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32)
    O, L = ra._ancestor(Q.cuda(), K.cuda(), V.cuda(), cu.cuda(), N, branching=b, max_depth=d, want_lse=True)
    ro, rl = orc.sparse_ancestor_attention(Q, K, V, cu, b, d)
    assert torch.allclose(O.float().cpu(), ro.float(), atol=ATOL, rtol=RTOL)
    assert torch.allclose(L.cpu().double(), rl, atol=1e-4)


def test_fused_lse_merge_permuted_views():
    B, H, N, D = 2, 4, 37, 64
    g = torch.Generator().manual_seed(10)
    lp, lt = torch.randn(B, H, N, generator=g) * 3, torch.randn(B, H, N, generator=g) * 3
    op = torch.randn(B, N, H, D, generator=g).half()
    ot = torch.randn(B, H, N, D, generator=g).half()
    res = ra.fused_lse_merge(lp.cuda(), lt.cuda(), op.cuda().permute(0, 2, 1, 3), ot.cuda())
    ref = orc.lse_merge(lp, lt, op.permute(0, 2, 1, 3).float(), ot.float())
    assert res.shape == (B, H, N, D) and res.is_contiguous()
    assert (res.float().cpu() - ref).abs().max().item() <= 2e-3


def test_prefix_merge_fused_in_ancestor_kernel():
    # ancestor pass seeded with a prefix result == separate passes + LSE merge
    b, d, H, D, B = 3, 3, 4, 64, 2
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(12, N, H, D, B)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    g = torch.Generator().manual_seed(13)
    po = torch.randn(B * N, H, D, generator=g).half()
    pl = torch.randn(B * N, H, generator=g) * 2
    O, L = ra._ancestor(Q.cuda(), K.cuda(), V.cuda(), cu.cuda(), N, branching=b, max_depth=d,
                        want_lse=True, prefix_o=po.cuda(), prefix_lse=pl.cuda())
    to, tl = orc.sparse_ancestor_attention(Q, K, V, cu, b, d)
    ref = orc.lse_merge(pl, tl.float(), po.float(), to.float())
    assert (O.float().cpu() - ref).abs().max().item() <= ATOL
    assert torch.allclose(L.cpu().double(), torch.logaddexp(pl.double(), tl), atol=1e-4)


def test_batch_permutation_is_bit_exact():
    # trees are independent: permuting sequences permutes outputs exactly
    b, d, H, D, B = 2, 5, 8, 128, 4
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(21, N, H, D, B)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    O = ra.ragged_attention(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    perm = [2, 0, 3, 1]
    Q2, K2, V2, _ = ra.pack_inputs([qs[i] for i in perm], [ks[i] for i in perm], [vs[i] for i in perm])
    O2 = ra.ragged_attention(Q2.cuda(), K2.cuda(), V2.cuda(), cu, b, d)
    for j, i in enumerate(perm):
        assert torch.equal(O2[j * N:(j + 1) * N], O[i * N:(i + 1) * N])


@pytest.mark.parametrize("cfg,dtype", [("C2", torch.float16), ("C3", torch.float16),
                                       ("C2", torch.bfloat16), ("C3", torch.bfloat16)])
def test_full_size_sliced_against_oracle(cfg, dtype):
    # bench configs C2 and C3 at full size, fp16 and bf16; the oracle checks the first and last tree
    B, b, d = (8, 4, 5) if cfg == "C2" else (16, 2, 9)
    H, D = 32, 128
    N = tm.num_tree_nodes(b, d)
    g = torch.Generator().manual_seed(2)
    Q, K, V = (torch.randn(B * N, H, D, generator=g).to(dtype) for _ in range(3))
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32)
    O, L = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    O, L = O.cpu(), L.cpu()
    assert torch.isfinite(O.float()).all()
    for s in (0, B - 1):
        sl = slice(s * N, (s + 1) * N)
        ro, rl = orc.sparse_ancestor_attention(Q[sl], K[sl], V[sl], [0, N], b, d, dtype=torch.float32)
        assert O.dtype == dtype
        assert torch.allclose(O[sl].float(), ro, atol=ATOL, rtol=RTOL)
        assert torch.allclose(L[sl], rl, atol=1e-3)


def test_cuda_graph_capture():
    b, d, H, D, B = 2, 4, 4, 64, 2
    N = tm.num_tree_nodes(b, d)
    qs, ks, vs = _gen(31, N, H, D, B)
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    Q, K, V, cud = Q.cuda(), K.cuda(), V.cuda(), cu.cuda()
    ref = ra.ragged_attention(Q, K, V, cu, b, d)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ra.ragged_attention(Q, K, V, cud, b, d, max_seqlen=N)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = ra.ragged_attention(Q, K, V, cud, b, d, max_seqlen=N)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_tile_plan_tables_reassigned_under_a_captured_graph():
    # Tile plans of a full-length tree shape live in a small set of tables inside
    # the library; a graph captured while one shape's table was valid must stay
    # correct after other shapes take the tables over (its launches then plan on
    # the device), and shorter sequences (planned on the device) must agree too.
    H, D = 4, 64
    shapes = [(2, 7), (3, 4), (4, 3), (2, 8), (5, 3), (2, 6)]
    runs = []
    for i, (b, d) in enumerate(shapes):
        N = tm.num_tree_nodes(b, d)
        lens = [N, N - 5, N]  # the middle sequence is shorter than max_seqlen
        qs, ks, vs = ([torch.randn(n, H, D, generator=torch.Generator().manual_seed(1000 * k + 10 * i + j)).half()
                       for j, n in enumerate(lens)] for k in range(3))
        Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
        runs.append((b, d, N, lens, qs, ks, vs, Q.cuda(), K.cuda(), V.cuda(), cu))
    b, d, N, lens, qs, ks, vs, Q, K, V, cu = runs[0]
    first = ra.ragged_attention(Q, K, V, cu, b, d)
    cud = cu.cuda()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = ra.ragged_attention(Q, K, V, cud, b, d, max_seqlen=N)
    for b2, d2, N2, lens2, qs2, ks2, vs2, Q2, K2, V2, cu2 in runs[1:]:  # the tables change hands
        O2 = ra.ragged_attention(Q2, K2, V2, cu2, b2, d2)
        ref2 = torch.cat(orc.padded_sdpa(qs2, ks2, vs2, [orc.ancestor_mask(n, b2, d2) for n in lens2]), 0)
        assert torch.allclose(O2.float().cpu(), ref2, atol=ATOL, rtol=RTOL)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    ref = torch.cat(orc.padded_sdpa(qs, ks, vs, [orc.ancestor_mask(n, b, d) for n in lens]), 0)
    assert torch.allclose(first.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    assert torch.equal(ra.ragged_attention(Q, K, V, cu, b, d), first)
    from qattention_b200 import _lib
    assert _lib.ancestor_diagnostics()[0] == 0  # every plan the kernel used passed its checks


@pytest.mark.parametrize("lens,d,H", [([511, 300, 130, 511, 64, 1], 8, 32), ([511, 511, 255, 400], 5, 32),
                                      ([1023, 700, 129], 9, 4)])
def test_deep_trees_ragged_subtree_tiles(lens, d, H):
    # deep binary trees take the subtree tiling (tiles of sibling subtrees plus
    # their root path); ragged lengths cut the last levels, and max_depth below
    # the tree's depth truncates the walks (second case); with 32 heads the
    # launch hands out (tile, head-chunk) units
    b, D = 2, 64
    g = torch.Generator().manual_seed(sum(lens) + d)
    qs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    ks = [torch.randn(n, H, D, generator=g).half() for n in lens]
    vs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    O, L = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    masks = [orc.ancestor_mask(n, b, d) for n in lens]
    ref, rl = orc.padded_sdpa(qs, ks, vs, masks, return_lse=True)
    err = (O.float().cpu() - torch.cat(ref, 0)).abs().max().item()
    assert torch.allclose(O.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL), f"peak_abs={err:.3e}"
    assert torch.allclose(L.cpu(), torch.cat(rl, 0), atol=1e-3)


@pytest.mark.parametrize("lens,b,d,H,Hkv,D,page", [
    ([15, 9, 40, 15], 2, 3, 4, 4, 64, 16),          # contiguous tiles, ragged, truncated walks
    ([1365, 1000, 1365], 4, 5, 8, 8, 128, 16),      # C2-shaped trees
    ([511, 300, 130, 511], 2, 8, 8, 2, 64, 32),     # deep trees: subtree tiles, GQA
    ([6, 4, 6, 1], 1, 5, 4, 4, 64, 4),              # chains (b = 1): the per-query walk
    ([40, 33, 40], 1, 39, 8, 2, 128, 16),           # long chains, GQA, walks past the staged levels
])
def test_paged_kv_matches_packed_and_oracle(lens, b, d, H, Hkv, D, page):
    # src/ragged_attn.py:827-1047: K/V in pages through a page table; the physical
    # pages are shuffled so the table matters. Same kernel as the packed path, so
    # the outputs are bit-identical to ragged_attention on packed K/V.
    g = torch.Generator().manual_seed(sum(lens) + page)
    qs = [torch.randn(n, H, D, generator=g).half() for n in lens]
    ks = [torch.randn(n, Hkv, D, generator=g).half() for n in lens]
    vs = [torch.randn(n, Hkv, D, generator=g).half() for n in lens]
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    Kc, Vc, pt = ra.build_paged_kv(ks, vs, page_size=page)
    perm = torch.randperm(Kc.shape[0], generator=g)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    Kc, Vc = Kc[perm], Vc[perm]                      # physical page j now holds old page perm[j]
    pt = inv[pt.long()].to(torch.int32)
    O = ra.ragged_attention_paged(Q.cuda(), Kc.cuda(), Vc.cuda(), pt, cu, b, d)
    O_packed = ra.ragged_attention(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    assert torch.equal(O, O_packed)
    rep = H // Hkv
    masks = [orc.ancestor_mask(n, b, d) for n in lens]
    ref = orc.padded_sdpa(qs, [k.repeat_interleave(rep, 1) for k in ks],
                          [v.repeat_interleave(rep, 1) for v in vs], masks)
    assert torch.allclose(O.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL)


def test_paged_kv_rejects_unsupported():
    Q = torch.randn(15, 2, 64, device="cuda").half()
    Kc = torch.zeros(1, 16, 2, 64, device="cuda").half()
    pt = torch.zeros(1, 1, dtype=torch.int32)
    cu = torch.tensor([0, 15], dtype=torch.int32)
    with pytest.raises(ValueError):
        ra.ragged_attention_paged(Q, Kc, Kc, pt, cu, 0, 3)       # branching factor 0
    with pytest.raises(AssertionError):
        ra.ragged_attention_paged(Q, Kc, Kc[:, :8], pt, cu, 2, 3)


def test_empty_sequences_and_empty_batch():
    # zero-length sequences anywhere in the batch (the reference's grid returns early for
    # rows past a sequence's length, src/ragged_attn.py:294-296) and a batch of no tokens
    H, D, b, d = 4, 128, 2, 4
    lens = [0, 31, 0, 0, 17, 31, 0]
    g = torch.Generator().manual_seed(21)
    qs, ks, vs = ([torch.randn(n, H, D, generator=g).half() for n in lens] for _ in range(3))
    Q, K, V, cu = ra.pack_inputs(qs, ks, vs)
    assert cu.tolist() == [0, 0, 31, 31, 31, 48, 79, 79]
    O, L = ra.ragged_attention_with_lse(Q.cuda(), K.cuda(), V.cuda(), cu, b, d)
    nz = [i for i, n in enumerate(lens) if n]
    ref, rl = orc.padded_sdpa([qs[i] for i in nz], [ks[i] for i in nz], [vs[i] for i in nz],
                              [orc.ancestor_mask(lens[i], b, d) for i in nz], return_lse=True)
    assert torch.allclose(O.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL)
    assert torch.allclose(L.cpu(), torch.cat(rl, 0), atol=1e-3)
    # the explicit-parent path on the same batch: BFS parents of the complete tree, per sequence
    par = torch.cat([torch.tensor([max(0, (j - 1) // b) for j in range(n)], dtype=torch.int32) for n in lens])
    Op, Lp = ra.ragged_attention_with_parents(Q.cuda(), K.cuda(), V.cuda(), cu, par.cuda(), d)
    assert torch.allclose(Op.float().cpu(), torch.cat(ref, 0), atol=ATOL, rtol=RTOL)
    assert torch.allclose(Lp.cpu(), torch.cat(rl, 0), atol=1e-3)
    from qattention_b200 import _lib
    assert _lib.ancestor_diagnostics()[0] == 0
    # no tokens at all
    E = torch.empty(0, H, D, dtype=torch.float16, device="cuda")
    Oe, Le = ra.ragged_attention_with_lse(E, E, E, torch.tensor([0, 0], dtype=torch.int32), b, d)
    assert Oe.shape == (0, H, D) and Le.shape == (0, H)
