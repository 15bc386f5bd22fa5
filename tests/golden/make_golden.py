"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run where QAttention's source tree is available (it is not on GPU boxes):

    python tests/golden/make_golden.py /path/to/QAttention

It imports the reference's own ``src.tree_mask``, ``src.ragged_attn.pack_inputs``
and ``tests.test_correctness.padded_sdpa_reference`` (all CPU-runnable) and
stores their outputs with the inputs that produced them:

* ``tree_topology.npz``  — build_tree / tree_attention_mask(_n/_pruned) /
  full_sequence_mask / build_pruned_tree / sample_balanced_tree_nodes /
  verify_tree_mask results for a set of (b, d) and seeds.
* ``pack_inputs.npz``    — cu_seqlens of pack_inputs for ragged lengths.
* ``sdpa_cases.npz``     — padded masked SDPA outputs (the reference oracle,
  fp16 output as the reference casts it) for bench config C1 (fp32 inputs,
  seed 0) and a sample of the reference test sweep's shapes (fp16 inputs).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

TOPO_CASES = [(1, 0), (1, 4), (1, 8), (2, 1), (2, 3), (2, 5), (3, 2), (3, 4), (4, 2), (4, 3), (5, 2), (8, 2)]
PRUNED_CASES = [(2, 4, None, 11), (3, 4, 30, 12), (4, 5, 60, 13), (1, 6, None, 14), (5, 3, 40, 15)]
BALANCED_CASES = [(2, 5, 20, 21), (3, 4, 50, 22), (4, 4, 100, 23), (4, 2, 21, 24)]
SDPA_CASES = [  # (name, B, b, d, H, D, seed)
    ("b1_d0", 4, 1, 0, 4, 64, 400),
    ("chain_d8", 4, 1, 8, 4, 64, 418),
    ("b2_d3", 1, 2, 3, 4, 64, 123),
    ("b3_d2", 2, 3, 2, 4, 64, 232),
    ("b2_d5", 2, 2, 5, 4, 64, 225),
    ("b3_d4_D32", 2, 3, 4, 4, 32, 234),
    ("b2_d4_D128", 2, 2, 4, 8, 128, 224),
    ("b4_d3_H8", 1, 4, 3, 8, 64, 143),
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from src import tree_mask as tm  # noqa: E402  (the reference)
    from src.ragged_attn import pack_inputs  # noqa: E402
    from tests.test_correctness import padded_sdpa_reference  # noqa: E402

    topo = {}
    for b, d in TOPO_CASES:
        topo[f"parent_b{b}_d{d}"] = np.asarray(tm.build_tree(b, d), dtype=np.int64)
        topo[f"mask_b{b}_d{d}"] = tm.tree_attention_mask(b, d)
        topo[f"verify_b{b}_d{d}"] = np.asarray(tm.verify_tree_mask(b, d, verbose=False))
    for b, n in [(2, 10), (3, 17), (4, 21), (28, 60)]:
        topo[f"mask_n_b{b}_n{n}"] = tm.tree_attention_mask_n(b, n)
    topo["full_seq_c5_b2_d2"] = tm.full_sequence_mask(5, 2, 2)
    for b, d, tgt, seed in PRUNED_CASES:
        p = tm.build_pruned_tree(b, d, target_nodes=tgt, rng=np.random.default_rng(seed))
        topo[f"pruned_b{b}_d{d}_s{seed}"] = np.asarray(p, dtype=np.int64)
        topo[f"pruned_mask_b{b}_d{d}_s{seed}"] = tm.tree_attention_mask_pruned(p)
    for b, d, n, seed in BALANCED_CASES:
        p = tm.sample_balanced_tree_nodes(b, d, n, rng=np.random.default_rng(seed))
        topo[f"balanced_b{b}_d{d}_n{n}_s{seed}"] = np.asarray(p, dtype=np.int64)
    np.savez_compressed(HERE / "tree_topology.npz", **topo)

    packs = {}
    for name, lens in {"ragged": [3, 1, 7, 15, 2], "single": [5], "zeros": [0, 4, 0]}.items():
        qs = [torch.zeros(n, 2, 8) for n in lens]
        _, _, _, cu = pack_inputs(qs, qs, qs)
        packs[f"lens_{name}"] = np.asarray(lens, dtype=np.int64)
        packs[f"cu_{name}"] = cu.numpy()
    np.savez_compressed(HERE / "pack_inputs.npz", **packs)

    cases = {}
    # bench config C1: one binary tree b=2 d=3 (N=15), H=4, D=64, fp32 N(0,1) from seed 0,
    # drawn in the order q, k, v.
    g = torch.Generator().manual_seed(0)
    N = tm.num_tree_nodes(2, 3)
    q = torch.randn(N, 4, 64, generator=g, dtype=torch.float32)
    k = torch.randn(N, 4, 64, generator=g, dtype=torch.float32)
    v = torch.randn(N, 4, 64, generator=g, dtype=torch.float32)
    out = padded_sdpa_reference([q], [k], [v], [tm.tree_attention_mask(2, 3)], torch.device("cpu"))
    cases.update({"c1_q": q.numpy(), "c1_k": k.numpy(), "c1_v": v.numpy(),
                  "c1_out": out[0].numpy(), "c1_meta": np.asarray([1, 2, 3, 4, 64])})
    for name, B, b, d, H, D, seed in SDPA_CASES:
        torch.manual_seed(seed)
        N = tm.num_tree_nodes(b, d)
        qs = [torch.randn(N, H, D, dtype=torch.float16) for _ in range(B)]
        ks = [torch.randn(N, H, D, dtype=torch.float16) for _ in range(B)]
        vs = [torch.randn(N, H, D, dtype=torch.float16) for _ in range(B)]
        Q, K, V, cu = pack_inputs(qs, ks, vs)
        ref = padded_sdpa_reference(qs, ks, vs, [tm.tree_attention_mask(b, d)] * B,
                                    torch.device("cpu"))
        cases[f"{name}_q"] = Q.numpy()
        cases[f"{name}_k"] = K.numpy()
        cases[f"{name}_v"] = V.numpy()
        cases[f"{name}_cu"] = cu.numpy()
        cases[f"{name}_out"] = torch.cat(ref, 0).numpy()
        cases[f"{name}_meta"] = np.asarray([B, b, d, H, D])
    np.savez_compressed(HERE / "sdpa_cases.npz", **cases)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
