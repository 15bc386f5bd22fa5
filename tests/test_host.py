"""Host-side logic (no GPU): tree topology mirror, pack_inputs, C-ABI library exports."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from qattention_b200 import tree_mask as tm
from qattention_b200 import _lib
from qattention_b200.ragged_attn import pack_inputs
from tests.golden.make_golden import BALANCED_CASES, PRUNED_CASES, TOPO_CASES

ROOT = Path(__file__).resolve().parents[1]


def test_tree_topology_matches_reference(golden):
    topo = golden["tree_topology"]
    for b, d in TOPO_CASES:
        assert tm.num_tree_nodes(b, d) == len(topo[f"parent_b{b}_d{d}"])
        assert np.array_equal(np.asarray(tm.build_tree(b, d)), topo[f"parent_b{b}_d{d}"])
        assert np.array_equal(tm.tree_attention_mask(b, d), topo[f"mask_b{b}_d{d}"])
        assert tm.verify_tree_mask(b, d, verbose=False) == bool(topo[f"verify_b{b}_d{d}"])
    for b, n in [(2, 10), (3, 17), (4, 21), (28, 60)]:
        assert np.array_equal(tm.tree_attention_mask_n(b, n), topo[f"mask_n_b{b}_n{n}"])
    assert np.array_equal(tm.full_sequence_mask(5, 2, 2), topo["full_seq_c5_b2_d2"])


def test_random_trees_match_reference(golden):
    topo = golden["tree_topology"]
    for b, d, tgt, seed in PRUNED_CASES:
        p = tm.build_pruned_tree(b, d, target_nodes=tgt, rng=np.random.default_rng(seed))
        assert np.array_equal(np.asarray(p), topo[f"pruned_b{b}_d{d}_s{seed}"])
        assert np.array_equal(tm.tree_attention_mask_pruned(p), topo[f"pruned_mask_b{b}_d{d}_s{seed}"])
    for b, d, n, seed in BALANCED_CASES:
        p = tm.sample_balanced_tree_nodes(b, d, n, rng=np.random.default_rng(seed))
        assert np.array_equal(np.asarray(p), topo[f"balanced_b{b}_d{d}_n{n}_s{seed}"])


def test_kernel_parents_self_loop():
    p = tm.kernel_parents([-1, 0, 0, 1, -1, 4])
    assert p.dtype == np.int32 and p.tolist() == [0, 0, 0, 1, 4, 4]


def test_build_tree_rejects_bad_args():
    with pytest.raises(ValueError):
        tm.build_tree(0, 2)
    with pytest.raises(ValueError):
        tm.build_tree(2, -1)


def test_pack_inputs_cu_seqlens_bit_exact(golden):
    packs = golden["pack_inputs"]
    for name in ("ragged", "single", "zeros"):
        lens = packs[f"lens_{name}"].tolist()
        qs = [torch.randn(n, 2, 8) for n in lens]
        Q, K, V, cu = pack_inputs(qs, qs, qs)
        assert cu.dtype == torch.int32 and cu.device.type == "cpu"
        assert np.array_equal(cu.numpy(), packs[f"cu_{name}"])
        assert Q.shape[0] == sum(lens) and torch.equal(Q, torch.cat(qs, 0))


def test_ragged_attention_rejects_cpu_and_bad_dtype():
    from qattention_b200.ragged_attn import ragged_attention
    x = torch.zeros(3, 2, 64, dtype=torch.float32)
    with pytest.raises(AssertionError):
        ragged_attention(x, x, x, torch.tensor([0, 3], dtype=torch.int32), 2, 1)
    h = x.half()
    with pytest.raises(RuntimeError):
        ragged_attention(h, h, h, torch.tensor([0, 3], dtype=torch.int32), 2, 1)


def _header_symbols():
    text = (ROOT / "include" / "qattn_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*QA_API\s+(?:int|const char\*)\s+(qa_\w+)\s*\(", text, re.M)))


def test_library_exports_every_header_symbol():
    syms = _header_symbols()
    assert syms and set(syms) == set(_lib.EXPORTED)
    L = _lib.lib()  # loads libqattn_b200.so (built by __graft_entry__.build / qattention_b200.build)
    for s in syms:
        assert hasattr(L, s), s
    assert L.qa_version().decode().startswith("qattn-b200")
    assert L.qa_status_string(-3).decode().startswith("pointer or stride")


def test_argument_errors_need_no_gpu():
    # invalid arguments are rejected on the host before any CUDA call
    L = _lib.lib()
    a = _lib.AncestorArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = 1, 4, 3, 64  # 4 % 3 != 0
    a.max_seqlen, a.branching, a.dtype = 8, 2, 0
    assert L.qa_ancestor_attn(a, None) == -1
    a.num_kv_heads, a.head_dim = 4, 48
    assert L.qa_ancestor_attn(a, None) == -2
    a.head_dim, a.branching = 64, 0
    assert L.qa_ancestor_attn(a, None) == -1
    a.branching, a.batch = 2, 0  # empty batch is a no-op
    assert L.qa_ancestor_attn(a, None) == 0
    assert L.qa_ancestor_attn(None, None) == -1


def test_struct_layout_matches_header():
    # field names of qa_ancestor_args in the header, in order, equal the ctypes mirror
    text = (ROOT / "include" / "qattn_b200.h").read_text()
    body = text[text.index("typedef struct qa_ancestor_args"):text.index("} qa_ancestor_args;")]
    names = []
    for line in body.splitlines()[1:]:
        line = line.split("/*")[0].strip().rstrip(";")
        if not line:
            continue
        types = {"const", "void", "float", "int32_t", "int64_t"}
        names += [t for t in re.split(r"[\s,*]+", line) if t and t not in types]
    assert names == [f[0] for f in _lib.AncestorArgs._fields_]
    # 12 pointers and 19 int64 (8 bytes), 10 int32 and a float (4 bytes); the float and the
    # int32 dtype pack into one 8-byte slot before the page-table pointer, page_size is
    # padded to 8 before q_stride_b
    # (workspace_planned, an int32, is padded to 8 at the end)
    assert ctypes.sizeof(_lib.AncestorArgs) == (12 + 19) * 8 + (10 + 1) * 4 + 4 + 8


def test_build_paged_kv_layout():
    # src/ragged_attn.py:1007-1047: consecutive physical pages per sequence, zero padding
    from qattention_b200 import ragged_attn as ra
    ks = [torch.arange(n * 2 * 8, dtype=torch.float32).view(n, 2, 8).half() for n in (5, 17, 16)]
    vs = [k + 1 for k in ks]
    Kc, Vc, pt = ra.build_paged_kv(ks, vs, page_size=8)
    assert Kc.shape == (1 + 3 + 2, 8, 2, 8) and pt.dtype == torch.int32
    assert pt.tolist() == [[0, 0, 0], [1, 2, 3], [4, 5, 0]]
    for b, k in enumerate(ks):
        for n in range(k.shape[0]):
            assert torch.equal(Kc[pt[b, n // 8], n % 8], k[n])
            assert torch.equal(Vc[pt[b, n // 8], n % 8], vs[b][n])
    assert Kc[0, 5:].abs().sum() == 0
