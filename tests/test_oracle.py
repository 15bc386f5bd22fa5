"""Pin the CPU oracle against golden vectors produced by the reference itself."""
import numpy as np
import pytest
import torch

from oracle import tree_attn_oracle as orc
from tests.golden.make_golden import SDPA_CASES, TOPO_CASES, PRUNED_CASES


def test_ancestor_walk_matches_reference_masks(golden):
    topo = golden["tree_topology"]
    for b, d in TOPO_CASES:
        ref = topo[f"mask_b{b}_d{d}"]
        n = ref.shape[0]
        # complete trees: the walk with max_depth=d visits exactly the ancestor set
        assert np.array_equal(orc.ancestor_mask(n, b, d), ref), (b, d)


def test_ancestor_walk_explicit_parents(golden):
    topo = golden["tree_topology"]
    for b, d, _, seed in PRUNED_CASES:
        par = topo[f"pruned_b{b}_d{d}_s{seed}"]
        ref = topo[f"pruned_mask_b{b}_d{d}_s{seed}"]
        kpar = par.copy()
        kpar[kpar < 0] = np.nonzero(kpar < 0)[0]
        assert np.array_equal(orc.ancestor_mask(len(par), 0, d, kpar), ref)


def test_truncated_walk():
    # depth-5 tree walked with max_depth=2 sees only self + 2 ancestors
    walk = orc.ancestor_walk(62, 63, 2, 2)
    assert walk == [62, 30, 14]
    assert orc.ancestor_walk(0, 63, 2, 5) == [0]


def test_config1_against_reference_sdpa(golden):
    c = golden["sdpa_cases"]
    q, k, v = (torch.from_numpy(c[f"c1_{x}"]) for x in "qkv")
    mask = golden["tree_topology"]["mask_b2_d3"]
    out = orc.padded_sdpa([q], [k], [v], [mask])[0]
    ref = torch.from_numpy(c["c1_out"]).float()  # the reference casts its output to fp16
    assert (out - ref).abs().max().item() <= 1e-3


@pytest.mark.parametrize("case", [c[0] for c in SDPA_CASES])
def test_oracles_against_reference_sdpa(golden, case):
    c = golden["sdpa_cases"]
    B, b, d, H, D = (int(x) for x in c[f"{case}_meta"])
    Q, K, V = (torch.from_numpy(c[f"{case}_{x}"]) for x in "qkv")
    cu = c[f"{case}_cu"]
    ref = torch.from_numpy(c[f"{case}_out"]).float()
    N = int(cu[1])
    mask = orc.ancestor_mask(N, b, d)
    qs = [Q[cu[i]:cu[i + 1]] for i in range(B)]
    ks = [K[cu[i]:cu[i + 1]] for i in range(B)]
    vs = [V[cu[i]:cu[i + 1]] for i in range(B)]
    dense = torch.cat(orc.padded_sdpa(qs, ks, vs, [mask] * B), 0)
    sparse, lse = orc.sparse_ancestor_attention(Q, K, V, cu, b, d)
    assert (dense - ref).abs().max().item() <= 1e-3
    assert (sparse.float() - ref).abs().max().item() <= 1e-3
    _, lse_dense = orc.padded_sdpa(qs, ks, vs, [mask] * B, dtype=torch.float64, return_lse=True)
    assert torch.allclose(lse, torch.cat(lse_dense, 0), atol=1e-9)


def test_prefix_tree_sdpa_consistent_with_full_sequence_mask(golden):
    # prefix + tree over a full-sequence mask == rectangular rows of the padded oracle
    g = torch.Generator().manual_seed(5)
    L, b, d, H, D = 6, 2, 2, 4, 32
    N = 7
    full = golden["tree_topology"]["full_seq_c5_b2_d2"]
    assert full.shape == (5 + N, 5 + N)
    kp, vp = torch.randn(L, H, D, generator=g), torch.randn(L, H, D, generator=g)
    q, k, v = (torch.randn(N, H, D, generator=g) for _ in range(3))
    tm = orc.ancestor_mask(N, b, d)
    o, lse = orc.prefix_tree_sdpa(q, kp, vp, k, v, tm, dtype=torch.float64, return_lse=True)
    # independent restatement: split into prefix and tree parts and merge by LSE
    o_t, lse_t = orc.sparse_ancestor_attention(q, k, v, [0, N], b, d)
    zeros = np.ones((N, L), dtype=bool)
    s = torch.einsum("nhd,lhd->hnl", q.double(), kp.double()) / D ** 0.5
    lse_p = torch.logsumexp(s, -1).T
    o_p = torch.einsum("hnl,lhd->nhd", torch.softmax(s, -1), vp.double())
    merged = orc.lse_merge(lse_p, lse_t, o_p, o_t)
    assert zeros.all()
    assert torch.allclose(merged.double(), o, atol=1e-6)
    assert torch.allclose(torch.logaddexp(lse_p, lse_t), lse, atol=1e-9)
