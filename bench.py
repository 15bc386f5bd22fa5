"""Benchmark of the tree-verification hot path (one JSON line on rank 0).

Headline workload: bench config C3 — B=16 complete binary trees of depth 9
(N=1023 tokens each, 16368 packed), H=32, D=128, fp16, no prefix, sharded by
tree across the ranks (strong scaling: the global batch is fixed, rank r owns
16/N trees through ``qattention_b200.sharding``). One step = one ancestor-walk
attention pass (``ragged_attention_with_lse`` semantics, O and LSE written)
over the rank's trees.

value  = algorithmic HBM bytes of the whole batch / device time of the slowest
         rank (GB/s), where algorithmic bytes = Q, K, V read once + O written
         once + LSE (4 B/row).
e2e    = the same metric through the public API (sharding helper ->
         ``ragged_attention_with_lse``) with pinned host buffers: each rank's
         H2D of its Q/K/V, the call, D2H of its O and LSE inside the timed region.
After timing, O and LSE are gathered to rank 0 with one NCCL gather per tensor
(timed under ``gather``) and checked against the CPU oracle on two trees.

Secondary results in the same line (``secondary``): config C2 (B=8 4-ary trees
of depth 5) sharded the same way; at N=1 also the reference's Triton kernel on
C2 and C3 (``triton_reference``, imported unmodified from ``baseline/_ref`` where
it is installed), config C4 whole verify attention and its prefix pass beside
the reference's prefix phase (``repeat_kv`` + aten flash SDPA), the W4A16
layer sweep at M = 16, 64, 1023, 8184; at every N config C5's W4A16 verify step
(8 sequences split over the ranks).

``--impl reference`` times the reference's CPU path for this operator (padded
masked SDPA, restated in oracle/, all host threads) on a bounded sample.

Stand-alone arms (one JSON line each, N=1): ``--kernel prefix | hybrid |
w4a16 | verify`` print the same secondary measurements as their own lines.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "tree-verify attention µs + achieved HBM GB/s; W4A16 verify-step tokens/s"
CONFIGS = {
    # name: (B, b, d, H, D)
    "C2": (8, 4, 5, 32, 128),
    "C3": (16, 2, 9, 32, 128),
}
HEADLINE = "C3"
L2_BYTES = 126 * 1024 * 1024
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _num_nodes(b: int, d: int) -> int:
    return d + 1 if b == 1 else (b ** (d + 1) - 1) // (b - 1)


def algorithmic_bytes(T: int, H: int, D: int, elt: int = 2, lse: bool = True) -> int:
    """Q, K, V read once + O written once (+ fp32 LSE per row)."""
    return 4 * T * H * D * elt + (4 * T * H if lse else 0)


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons every 100 ms in the background."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        inside = [r for t, r in self.rows if self.t0 is not None and self.t0 - 0.1 <= t <= self.t1 + 0.1]
        use = inside or [r for _, r in self.rows[-3:]]
        mhz = [float(r[1]) for r in use if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": float(use[0][2]) if use and use[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(inside)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return ws, rank, local


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_trees(cfg: str, lo: int, hi: int, seed: int = 0):
    """Seeded synthetic fp16 N(0,1) inputs of trees lo..hi-1 of a config, on the host.

    Each tree has its own generator (seed, tree index), so a tree's values do not
    depend on how the batch is sharded. Returns packed Q, K, V and cu_seqlens.
    """
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    qs, ks, vs = [], [], []
    for t in range(lo, hi):
        g = torch.Generator().manual_seed(seed * 100003 + t)
        qs.append(torch.randn(N, H, D, generator=g).half())
        ks.append(torch.randn(N, H, D, generator=g).half())
        vs.append(torch.randn(N, H, D, generator=g).half())
    n = hi - lo
    if n == 0:
        e = torch.empty(0, H, D, dtype=torch.float16)
        return e, e.clone(), e.clone(), torch.zeros(1, dtype=torch.int32)
    cu = torch.arange(0, (n + 1) * N, N, dtype=torch.int32)
    return torch.cat(qs), torch.cat(ks), torch.cat(vs), cu


def global_cu(cfg: str) -> torch.Tensor:
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    return torch.arange(0, (B + 1) * N, N, dtype=torch.int32)


def _traffic_from_profile(cfg: str):
    """DRAM bytes per full-batch launch of the ancestor kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "ancestor_attn_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        j = json.load(f)
    return j.get(cfg, {}).get("dram_bytes_per_launch")


def graph_steps(fn, copies: int, dev, per_graph: int = 8):
    """CUDA graphs of back-to-back steps over rotating input copies.

    One graph of G steps (G a multiple of `copies`; consecutive launches overlap
    through programmatic dependent launch, as in a serving loop) plus one
    single-step graph per copy for a remainder; returns run(n), which replays
    exactly n steps.
    """
    G = copies * max(1, per_graph // copies)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(copies):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(stream)
    graph_g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_g):
        for j in range(G):
            fn(j)
    singles = []
    for i in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(i)
        singles.append(g)

    def run(n):
        for _ in range(n // G):
            graph_g.replay()
        for i in range(n % G):
            singles[i % copies].replay()

    run.graphs = (graph_g, singles)
    run.per_graph = G
    return run


def time_run(run, steps: int, warmup: int, dev, before=None, after=None) -> float:
    """ms per step of run(n) with CUDA events on the current stream.

    `before` runs after the warm-up and a synchronize, right before the first
    event (a barrier, a clock mark); `after` right after the closing synchronize.
    """
    run(warmup)
    torch.cuda.synchronize(dev)
    if before is not None:
        before()
        torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    run(steps)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    if after is not None:
        after()
    return e0.elapsed_time(e1) / steps


def _rotating(Qh, Kh, Vh, dev, nbytes):
    copies = max(2, -(-3 * L2_BYTES // max(nbytes, 1)))
    return copies, [(Qh.to(dev), Kh.to(dev), Vh.to(dev)) for _ in range(copies)]


def time_ancestor_ours(cfg, Qh, Kh, Vh, cu, dev, steps, warmup, before=None, after=None):
    """Device ms per step of this library's ancestor pass (graph replay, rotating copies)."""
    from qattention_b200 import ragged_attn as ra
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    T = Qh.shape[0]
    copies, ins = _rotating(Qh, Kh, Vh, dev, algorithmic_bytes(T, H, D))
    cud = cu.to(dev)
    O = torch.empty(T, H, D, dtype=torch.float16, device=dev)
    L = torch.empty(T, H, dtype=torch.float32, device=dev)

    def step(i):
        Q, K, V = ins[i % copies]
        ra._ancestor(Q, K, V, cud, N, branching=b, max_depth=d, want_lse=True, out=O, lse_out=L)

    run = graph_steps(step, copies, dev)
    ms = time_run(run, steps, warmup, dev, before, after)
    step(0)
    torch.cuda.synchronize(dev)
    del run
    return ms, O, L, copies


def _import_reference():
    """The unmodified reference module from baseline/_ref (None, reason when absent)."""
    if not os.path.isdir(os.path.join(REF_DIR, "src")):
        return None, "baseline/_ref is not installed (the reference package was not found next to bench.py)"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import src.ragged_attn as ref  # noqa: WPS433 (the reference's own module name)
        return ref, None
    except Exception as e:  # the reason goes into the JSON line
        return None, f"import failed: {type(e).__name__}: {str(e).splitlines()[0][:200]}"


def time_triton_reference(cfg, dev, steps, warmup, ours_out=None, seed=0):
    """The reference's Triton kernel (``ragged_attention_with_lse``) on the same inputs and timing.

    Its first calls run its autotuner; the timed steps replay CUDA graphs over the
    same rotating input copies as this library's arm. Returns a dict for the
    JSON line (``unavailable`` with the reason when it cannot run).
    """
    ref, why = _import_reference()
    if ref is None:
        return {"unavailable": why}
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    Qh, Kh, Vh, cu = make_trees(cfg, 0, B, seed)
    T = Qh.shape[0]
    nbytes = algorithmic_bytes(T, H, D)
    try:
        copies, ins = _rotating(Qh, Kh, Vh, dev, nbytes)
        cud = cu.to(dev)
        for i in range(copies):  # autotune outside the graphs
            ref.ragged_attention_with_lse(*ins[i], cud, b, d, max_seqlen=N)
        torch.cuda.synchronize(dev)
        outs = {}

        def step(i):
            outs["o"] = ref.ragged_attention_with_lse(*ins[i % copies], cud, b, d, max_seqlen=N)

        run = graph_steps(step, copies, dev)
        ms = time_run(run, steps, warmup, dev)
        O, L = ref.ragged_attention_with_lse(*ins[0], cud, b, d, max_seqlen=N)
        torch.cuda.synchronize(dev)
        res = {"us_per_step": ms * 1e3, "gbs": nbytes / (ms * 1e-3) / 1e9,
               "kernel": "_ragged_attn_sparse_kernel_lse (Triton, reference src/ragged_attn.py:401-572)",
               "timing": "CUDA-graph replay of back-to-back steps over the same rotating copies"}
        if ours_out is not None:
            res["max_abs_diff_vs_ours"] = float((O.float() - ours_out[0].float()).abs().max())
            res["lse_max_abs_diff_vs_ours"] = float((L - ours_out[1]).abs().max())
        del run, ins
        return res
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200] if str(e) else ''}"}


def _capture(fn, n, dev):
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(n):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(stream)
    graphs = []
    for i in range(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(i)
        graphs.append(g)
    return graphs


def _timed_graphs(graphs, steps, warmup, dev):
    """Replays the captured graphs round-robin; returns ms per replay (CUDA events)."""
    def run(n):
        for i in range(n):
            graphs[i % len(graphs)].replay()
    return time_run(run, steps, warmup, dev)


C4 = dict(B=16, L=10240, b=4, d=4, Hq=32, Hkv=8, D=128)


def measure_prefix(dev, steps, warmup):
    """Config 4's shared-prefix pass: this library's tcgen05 kernel, and the reference's
    prefix phase on the same inputs (``repeat_kv`` then aten flash SDPA,
    scripts/w4a16_e2e.py:1236-1249), both timed by graph replay."""
    from qattention_b200 import ragged_attn as ra
    B, L, Hq, Hkv, D = C4["B"], C4["L"], C4["Hq"], C4["Hkv"], C4["D"]
    N = _num_nodes(C4["b"], C4["d"])
    g = torch.Generator().manual_seed(4)
    Q = torch.randn(B, N, Hq, D, generator=g).half().to(dev)
    K = torch.randn(B, L, Hkv, D, generator=g).half().to(dev)
    V = torch.randn(B, L, Hkv, D, generator=g).half().to(dev)
    flops = 4.0 * B * Hq * N * L * D
    graphs = _capture(lambda i: ra.prefix_attention_with_lse(Q, K, V), 1, dev)
    ms = _timed_graphs(graphs, steps, warmup, dev)
    O, LSE = ra.prefix_attention_with_lse(Q, K, V)
    del graphs
    peak, kind = _tensor_peak()
    res = {"us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12, "peak": peak, "peak_kind": kind,
           "frac": flops / (ms * 1e-3) / 1e12 / peak, "flops_per_launch": flops,
           "kernel": "prefix_attn_kernel (qa_prefix_attn)"}
    # the reference's prefix phase: K/V in the model's [B, H, L, D] layout after repeat_kv
    Qr = Q.transpose(1, 2).contiguous()
    Kc, Vc = K.transpose(1, 2).contiguous(), V.transpose(1, 2).contiguous()  # [B, Hkv, L, D] cache

    def repeat_kv(x):
        return x[:, :, None].expand(B, Hkv, Hq // Hkv, L, D).reshape(B, Hq, L, D)

    def ref_phase(_):
        Kr, Vr = repeat_kv(Kc).contiguous(), repeat_kv(Vc).contiguous()
        return torch.ops.aten._scaled_dot_product_flash_attention(
            Qr, Kr, Vr, dropout_p=0.0, is_causal=False, scale=1.0 / math.sqrt(D), return_debug_mask=False)

    try:
        out = ref_phase(0)
        ref_o = out[0].transpose(1, 2).float()
        diff = float((ref_o - O.float()).abs().max())
        graphs = _capture(ref_phase, 1, dev)
        ms_ref = _timed_graphs(graphs, steps, warmup, dev)
        del graphs
        Kr, Vr = repeat_kv(Kc).contiguous(), repeat_kv(Vc).contiguous()
        lib_graphs = _capture(lambda i: torch.ops.aten._scaled_dot_product_flash_attention(
            Qr, Kr, Vr, dropout_p=0.0, is_causal=False, scale=1.0 / math.sqrt(D), return_debug_mask=False), 1, dev)
        ms_flash = _timed_graphs(lib_graphs, steps, warmup, dev)
        del lib_graphs, Kr, Vr
        res["reference_prefix_phase"] = {
            "us": ms_ref * 1e3, "tflops": flops / (ms_ref * 1e-3) / 1e12,
            "flash_alone_us": ms_flash * 1e3, "flash_alone_tflops": flops / (ms_flash * 1e-3) / 1e12,
            "what": "repeat_kv of the [B, Hkv, L, D] cache + aten _scaled_dot_product_flash_attention "
                    "(scripts/w4a16_e2e.py:1236-1249); flash_alone = the SDPA call on pre-expanded K/V",
            "max_abs_diff_vs_ours": diff}
    except Exception as e:
        res["reference_prefix_phase"] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    return res


def measure_parents(dev, steps, warmup):
    """Explicit-parent trees (``ragged_attention_with_parents``, the reference's E2E verify call):
    the C2 batch given as parent arrays, and a C2-sized batch of EAGLE-style pruned trees
    (8 trees of ~1365 nodes, b=8, d=5); algorithmic GB/s as for the headline."""
    import numpy as np
    from qattention_b200 import ragged_attn as ra
    from qattention_b200 import tree_mask as tm
    H, D, B = 32, 128, 8
    out = {}
    for name, b, d, pruned in (("C2_as_parents", 4, 5, False), ("C2_sized_pruned_b8_d5", 8, 5, True)):
        rng = np.random.default_rng(77)
        trees = [tm.build_pruned_tree(b, d, target_nodes=1365, rng=rng) if pruned else tm.build_tree(b, d)
                 for _ in range(B)]
        lens = [len(t) for t in trees]
        T = sum(lens)
        g = torch.Generator().manual_seed(78)
        Qh, Kh, Vh = (torch.randn(T, H, D, generator=g).half() for _ in range(3))
        cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
        par = torch.from_numpy(np.concatenate([tm.kernel_parents(t) for t in trees])).to(dev)
        nbytes = algorithmic_bytes(T, H, D)
        copies, ins = _rotating(Qh, Kh, Vh, dev, nbytes)
        cud = cu.to(dev)
        ms_len = max(lens)

        def step(i):
            ra.ragged_attention_with_parents(*ins[i % copies], cud, par, d, max_seqlen=ms_len)

        run = graph_steps(step, copies, dev)
        ms = time_run(run, steps, warmup, dev)
        del run
        # the same trees planned once (as every layer of a verify step can share)
        plan = ra.plan_parents(cud, par, d, max_seqlen=ms_len)

        def step_planned(i):
            ra.ragged_attention_with_parents(*ins[i % copies], cud, par, d, max_seqlen=ms_len, plan=plan)

        run = graph_steps(step_planned, copies, dev)
        ms_planned = time_run(run, steps, warmup, dev)
        O, L = ra.ragged_attention_with_parents(*ins[0], cud, par, d, max_seqlen=ms_len)
        from oracle import tree_attn_oracle as orc
        sl = slice(0, lens[0])
        ro, rl = orc.sparse_ancestor_attention(Qh[sl, :4], Kh[sl, :4], Vh[sl, :4], [0, lens[0]], 0, d,
                                               parents=par[sl].cpu(), dtype=torch.float32)
        err = float((O[sl, :4].float().cpu() - ro).abs().max())
        peak, kind = _peaks()
        out[name] = {"us_per_step": ms * 1e3, "gbs": nbytes / (ms * 1e-3) / 1e9,
                     "frac": nbytes / (ms * 1e-3) / 1e9 / peak, "tokens": T, "algorithmic_bytes": nbytes,
                     "plan_reused": {"us_per_step": ms_planned * 1e3, "gbs": nbytes / (ms_planned * 1e-3) / 1e9,
                                     "frac": nbytes / (ms_planned * 1e-3) / 1e9 / peak},
                     "check_tree0_4heads_max_abs_err": err,
                     "launches_per_step": 2, "kernels": "ancestor_parents_plan_kernel + ancestor_tc_kernel"}
        del run, ins
    return out


def measure_hybrid(dev, steps, warmup):
    """Config 4 whole verify attention: tcgen05 prefix pass + ancestor pass with the LSE merge fused."""
    from qattention_b200 import ragged_attn as ra
    B, L, b, d, Hq, Hkv, D = (C4[k] for k in ("B", "L", "b", "d", "Hq", "Hkv", "D"))
    N = _num_nodes(b, d)
    g = torch.Generator().manual_seed(6)
    Q = torch.randn(B, Hq, N, D, generator=g).half().to(dev)
    K = torch.randn(B, Hkv, L + N, D, generator=g).half().to(dev)
    V = torch.randn(B, Hkv, L + N, D, generator=g).half().to(dev)
    graphs = _capture(lambda i: ra.tree_verify_attention(Q, K, V, b, d), 1, dev)
    ms = _timed_graphs(graphs, steps, warmup, dev)
    del graphs
    prefix_flops = 4.0 * B * Hq * N * L * D
    return {"us": ms * 1e3, "prefix_tflops_of_whole": prefix_flops / (ms * 1e-3) / 1e12,
            "what": "tree_verify_attention on the [B, Hkv, L+N, D] KV cache (no repeat_kv)"}


# (name, K, N) of one Llama-3.1-8B decoder layer, Y = X W with W [K, N]; q/k/v
# and gate/up are fused along N as serving stacks load them (same weights, 4 GEMMs)
LLAMA_LINEARS = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 28672), ("down", 14336, 4096)]


def measure_w4a16(dev, steps, warmup, ms_list):
    """One decoder layer's W4A16 linears (random-init int4 weights) at several M."""
    import ctypes
    from qattention_b200 import _lib, quant
    g = torch.Generator().manual_seed(5)
    layer = []
    for _, K, N in LLAMA_LINEARS:
        qw, sc = quant.quantize_w4a16(torch.randn(K, N, generator=g) * 0.02)
        layer.append((qw.to(dev), sc.to(dev), K, N))
    wbytes = sum(qw.numel() * 4 + sc.numel() * 2 for qw, sc, _, _ in layer)
    copies = max(2, -(-3 * L2_BYTES // wbytes))
    layers = [layer] + [[(qw.clone(), sc.clone(), K, N) for qw, sc, K, N in layer] for _ in range(copies - 1)]
    sweep = {}
    for M in ms_list:
        xs = {K: torch.randn(M, K, device=dev).half() for K in (4096, 14336)}
        ys = [torch.empty(M, N, dtype=torch.float16, device=dev) for _, _, _, N in layer]

        def step(i, xs=xs, ys=ys):
            for j, (qw, sc, K, N) in enumerate(layers[i % copies]):
                quant.w4a16_linear(xs[K], qw, sc, out=ys[j])

        graphs = _capture(step, copies, dev)
        n = max(copies, min(steps, 200 if M <= 1023 else 40))
        ms = _timed_graphs(graphs, n, warmup, dev)
        flops = sum(2.0 * M * K * N for _, _, K, N in layer)
        splits = []
        for _, _, K, N in layer:  # one launch per GEMM: split-K partials are summed by the last CTA of a tile
            sp, wb = ctypes.c_int32(), ctypes.c_int64()
            _lib.check(_lib.lib().qa_w4a16_plan(M, N, K, ctypes.byref(sp), ctypes.byref(wb)), "qa_w4a16_plan")
            splits.append(sp.value)
        launches = len(layer)
        sweep[str(M)] = {"us_per_layer": ms * 1e3, "weight_gbs": wbytes / (ms * 1e-3) / 1e9,
                         "tflops": flops / (ms * 1e-3) / 1e12, "launches_per_layer": launches,
                         "splits": splits}
        del graphs
    hb, hkind = _peaks()
    tp, tkind = _tensor_peak()
    for v in sweep.values():
        v["hbm_frac"] = v["weight_gbs"] / hb
        v["tensor_frac"] = v["tflops"] / tp
    return {"sweep": sweep, "bytes_per_layer": wbytes, "copies": copies, "hbm_peak": hb, "hbm_peak_kind": hkind,
            "tensor_peak": tp, "tensor_peak_kind": tkind,
            "workload": "Llama-3.1-8B decoder layer W4A16 linears, qkv and gate_up fused (4 GEMMs, 218.1 M "
                        "weights, group 128), rotating weight copies > 3x L2"}


def measure_verify(ws, rank, dev, steps, warmup, layers=0):
    """Config 5: the W4A16 tree-verify step, 8 sequences split over the ranks; tokens/s (strong scaling)."""
    from qattention_b200 import verify as vf
    B_all, L, b, d = 8, 2048, 2, 9
    if B_all % ws:
        return {"unavailable": "config 5 shards 8 sequences: use 1, 2, 4 or 8 GPUs"}
    B = B_all // ws
    N = _num_nodes(b, d)
    cfg = vf.LlamaConfig()
    if layers:
        cfg.layers = layers
    model = vf.VerifyModel(cfg, dev, seed=7)
    cache = model.new_cache(B, L, N, seed=8 + rank)
    g = torch.Generator().manual_seed(9 + rank)
    tok_host = torch.randint(0, cfg.vocab, (B, N), generator=g).pin_memory()
    tokens = tok_host.to(dev)
    steps = max(1, min(steps, 10))
    for _ in range(max(warmup, 2)):
        model.step(tokens, cache, L, b, d)
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(steps):
        model.step(tokens, cache, L, b, d)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    eager_ms = _max_over_ranks(e0.elapsed_time(e1) / steps, ws)
    graph, logits = model.capture(tokens, cache, L, b, d)
    for _ in range(max(warmup, 2)):
        graph.replay()
    torch.cuda.synchronize(dev)
    _barrier(ws)
    torch.cuda.synchronize(dev)
    e0.record(cur)
    for _ in range(steps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, ws)
    out_host = torch.empty(B * N, dtype=torch.int64).pin_memory()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(ws)
    f0.record(cur)
    for _ in range(steps):
        tokens.copy_(tok_host, non_blocking=True)
        graph.replay()
        out_host.copy_(logits.argmax(-1), non_blocking=True)
    f1.record(cur)
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1) / steps, ws)
    del graph, logits, model, cache
    torch.cuda.empty_cache()
    tokens_total = B_all * N
    return {"tokens_per_s": tokens_total / (ms * 1e-3), "ms_per_step": ms, "eager_ms_per_step": eager_ms,
            "e2e": {"tokens_per_s": tokens_total / (e2e_ms * 1e-3), "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": B * N * 8, "d2h_bytes_per_step": B * N * 8},
            "layers": cfg.layers, "sequences_per_gpu": B, "steps": steps,
            "workload": f"C5: random-init Llama-3.1-8B architecture ({cfg.layers} layers), W4A16 linears "
                        "(qkv and gate_up fused), fp16 LM head; B=8 sequences x (2048-token cached prefix + "
                        "binary depth-9 tree, 1023 tokens) = 8184 verify tokens per step, sharded by sequence",
            "timing": "one CUDA graph per step (VerifyModel.capture), max over ranks"}


def cpu_reference_step(Q, K, V, cfg, heads: int, trees: int = 1):
    """The reference's CPU path on a sample: padded masked SDPA over `trees` trees x `heads` heads."""
    from oracle import tree_attn_oracle as orc
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    mask = orc.ancestor_mask(N, b, d)
    qs = [Q[i * N:(i + 1) * N, :heads] for i in range(trees)]
    ks = [K[i * N:(i + 1) * N, :heads] for i in range(trees)]
    vs = [V[i * N:(i + 1) * N, :heads] for i in range(trees)]
    return orc.padded_sdpa(qs, ks, vs, [mask] * trees)


def cpu_sample_plan(Q, K, V, cfg, per_step_budget_s: float):
    """How many heads of one tree a CPU step covers so that it fits the budget."""
    H = CONFIGS[cfg][3]
    t0 = time.perf_counter()
    cpu_reference_step(Q, K, V, cfg, 1)
    t1 = time.perf_counter() - t0
    return int(max(1, min(H, per_step_budget_s // max(t1, 1e-6))))


def _config_dict(cfg, ws):
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    return {"workload": f"{cfg}: B={B} complete {b}-ary trees depth {d} (N={N}/tree, T={B * N}), "
                        f"H={H}, D={D}, fp16 I/O, no prefix",
            "batch": B, "branching": b, "depth": d, "heads": H, "head_dim": D, "tokens": B * N,
            "parallelism": f"trees sharded by qattention_b200.sharding over {ws} rank(s) (strong scaling: "
                           f"{B // ws if B % ws == 0 else 'about ' + str(B / ws)} trees per GPU), no collective "
                           "in the timed region, one NCCL gather of O and LSE afterwards",
            "l2": "rotating input copies, total > 3x the 126 MB L2"}


def run_reference(args):
    """--impl reference: the reference's CPU implementation of the path (oracle restatement), rank 0 only."""
    ws, rank, _ = _dist()
    if rank != 0:
        return
    cfg = args.config
    torch.set_num_threads(os.cpu_count() or 1)
    Q, K, V, cu = make_trees(cfg, 0, 1, 0)
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    heads = cpu_sample_plan(Q, K, V, cfg, 150.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference_step(Q, K, V, cfg, heads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(Q, K, V, cfg, heads)
    dt = (time.perf_counter() - t0) / args.steps
    gbs = algorithmic_bytes(N, heads, D) / dt / 1e9
    sample = (f"1 of {B} trees x {heads} of {H} heads per step (padded masked SDPA, fp32, torch CPU); "
              "GB/s from that sample's own algorithmic bytes")
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": _config_dict(cfg, args.gpus),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _oracle_check(O, L, cfg, trees, heads=8, seed=0):
    """Max |O - oracle| and |LSE - oracle| over the given trees (first `heads` heads)."""
    from oracle import tree_attn_oracle as orc
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    eo = el = 0.0
    for t in trees:
        Q, K, V, cu = make_trees(cfg, t, t + 1, seed)
        ref, rl = orc.sparse_ancestor_attention(Q[:, :heads], K[:, :heads], V[:, :heads], cu, b, d)
        s = slice(t * N, (t + 1) * N)
        eo = max(eo, float((O[s, :heads].float() - ref.float()).abs().max()))
        el = max(el, float((L[s, :heads].double() - rl).abs().max()))
    return eo, el


def ancestor_sharded(cfg, ws, rank, dev, steps, warmup, clocks=None, with_e2e=True, with_gather=True):
    """Config `cfg` sharded by tree over the ranks: device time, e2e, gather, oracle check."""
    from qattention_b200 import sharding
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    sh = sharding.shard_trees(global_cu(cfg), ws, rank)
    Qh, Kh, Vh, cu = make_trees(cfg, sh.tree_lo, sh.tree_hi, 0)
    local_bytes = algorithmic_bytes(sh.num_tokens, H, D)
    total_bytes = algorithmic_bytes(B * N, H, D)

    def before():
        _barrier(ws)
        if clocks is not None:
            clocks.mark("t0")

    def after():
        if clocks is not None:
            clocks.mark("t1")
        _barrier(ws)

    ms, O, L, copies = time_ancestor_ours(cfg, Qh, Kh, Vh, cu, dev, steps, warmup, before, after)
    ms_max = _max_over_ranks(ms, ws)
    res = {"ms_per_step": ms_max, "us_per_step": ms_max * 1e3, "local_us": ms * 1e3,
           "gbs": total_bytes / (ms_max * 1e-3) / 1e9, "per_gpu_gbs": local_bytes / (ms * 1e-3) / 1e9,
           "local_bytes": local_bytes, "total_bytes": total_bytes, "trees_per_rank": sh.num_trees,
           "copies": copies}
    if with_e2e:
        from qattention_b200.host_pipeline import ragged_attention_with_lse_host
        Qp, Kp, Vp = Qh.pin_memory(), Kh.pin_memory(), Vh.pin_memory()
        Op = torch.empty(sh.num_tokens, H, D, dtype=torch.float16).pin_memory()
        Lp = torch.empty(sh.num_tokens, H, dtype=torch.float32).pin_memory()
        e2e_steps = max(3, min(steps, 20))

        def e2e_step():
            if sh.num_trees:
                ragged_attention_with_lse_host(Qp, Kp, Vp, sh.cu_local, b, d, device=dev, out=Op, lse_out=Lp)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        _barrier(ws)
        cur = torch.cuda.current_stream(dev)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(cur)
        for _ in range(e2e_steps):
            e2e_step()
        f1.record(cur)
        torch.cuda.synchronize(dev)
        e2e_ms = _max_over_ranks(f0.elapsed_time(f1) / e2e_steps, ws)
        res["e2e"] = {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                      "h2d_bytes_per_step": 3 * B * N * H * D * 2, "d2h_bytes_per_step": B * N * H * (2 * D + 4),
                      "what": "each rank: host_pipeline.ragged_attention_with_lse_host on its trees' pinned "
                              "Q/K/V (H2D, ancestor pass and D2H of O and LSE overlapped over chunks of "
                              "whole trees on three streams); bytes summed over ranks"}
    if with_gather:
        if ws > 1:  # the first gather sets up NCCL's peer connections: warm them up untimed
            sharding.gather_outputs(O[:1], L[:1], sharding.shard_trees(
                torch.arange(ws + 1, dtype=torch.int32), ws, rank), dst=0)
        _barrier(ws)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        Og, Lg = sharding.gather_outputs(O, L, sh, dst=0)
        torch.cuda.synchronize(dev)
        g_ms = _max_over_ranks((time.perf_counter() - t0) * 1e3, ws)
        res["gather"] = {"ms": g_ms, "bytes": B * N * H * (2 * D + 4),
                         "what": "one torch.distributed.gather of O and one of LSE to rank 0 (NCCL), "
                                 "wall clock max over ranks, after the timed region"}
        if rank == 0:
            eo, el = _oracle_check(Og.cpu(), Lg.cpu(), cfg, sorted({0, B - 1}))
            res["check"] = {"trees": sorted({0, B - 1}), "heads": 8, "max_abs_err_o": eo,
                            "max_abs_err_lse": el, "tolerance": "1e-2 (O), 1e-3 (LSE)",
                            "ok": bool(eo <= 1e-2 and el <= 1e-3)}
            res["checksum"] = [float(Og.float().sum()), float(Lg.double().sum())]
    return res, (O, L)


def run_ours(args):
    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    cfg = args.config
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    head, (O, L) = ancestor_sharded(cfg, ws, rank, dev, args.steps, args.warmup, clocks)
    if rank == 0:
        clocks.stop()
    peak, peak_kind = _peaks()
    traffic = _traffic_from_profile(cfg)
    if traffic is not None:  # the profile holds one full-batch launch; this rank's launch covers its share
        traffic = traffic * head["local_bytes"] / head["total_bytes"]

    secondary = {}
    if args.secondary:
        other = "C2" if cfg == "C3" else "C3"
        sec, ours_other = ancestor_sharded(other, ws, rank, dev, args.steps, args.warmup, None,
                                           with_e2e=False, with_gather=True)
        secondary[other] = sec
        if ws == 1:
            secondary["triton_reference"] = {
                cfg: time_triton_reference(cfg, dev, args.steps, args.warmup, (O, L)),
                other: time_triton_reference(other, dev, args.steps, args.warmup, ours_other)}
            torch.cuda.empty_cache()
            secondary["explicit_parents"] = measure_parents(dev, args.steps, args.warmup)
            secondary["C4_prefix"] = measure_prefix(dev, max(args.steps, 10), args.warmup)
            secondary["C4_verify_attention"] = measure_hybrid(dev, max(args.steps, 10), args.warmup)
            torch.cuda.empty_cache()
            secondary["w4a16_layer"] = measure_w4a16(dev, max(args.steps, 20), args.warmup,
                                                     [int(m) for m in args.w4_m.split(",")])
            torch.cuda.empty_cache()
        secondary["C5_verify_step"] = measure_verify(ws, rank, dev, args.steps, args.warmup, args.verify_layers)

    if rank != 0:
        return
    cpu_base = None
    if ws == 1 and not args.skip_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        Qh, Kh, Vh, _ = make_trees(cfg, 0, 1, 0)
        heads = cpu_sample_plan(Qh, Kh, Vh, cfg, 2.0)
        t0 = time.perf_counter()
        n = 0
        while True:
            cpu_reference_step(Qh, Kh, Vh, cfg, heads)
            n += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        cdt = (time.perf_counter() - t0) / n
        cpu_base = {"value": algorithmic_bytes(N, heads, D) / cdt / 1e9, "unit": "GB/s",
                    "cores": torch.get_num_threads(), "kind": "port",
                    "sample": f"{n} runs x 1 of {B} trees x {heads} of {H} heads (padded masked SDPA, fp32, "
                              "torch CPU); GB/s from that sample's own algorithmic bytes"}
    ms = head["ms_per_step"]
    line = {
        "metric": METRIC, "value": head["gbs"], "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "us_per_step": ms * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": {**_config_dict(cfg, ws),
                                        "graphs": "8 back-to-back steps per CUDA graph over the rotating copies "
                                                  "(programmatic dependent launch between steps)"},
        "roofline": {"bound": "hbm", "achieved": head["per_gpu_gbs"], "peak": peak, "unit": "GB/s",
                     "frac": head["per_gpu_gbs"] / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes": head["local_bytes"],
                     "per": "rank 0's launch (its share of the batch)",
                     "kernel": "ancestor_tc_kernel (qa_ancestor_attn)"},
        "cpu_baseline": cpu_base,
        "e2e": head["e2e"],
        "gather": head.get("gather"), "check": head.get("check"),
        "gpu_launches": args.steps, "gpu_launches_per": "rank (one ancestor_tc_kernel per step)",
        "clocks": clocks.summary(),
        "checksum": head.get("checksum"),
        "secondary": secondary,
    }
    print(json.dumps(line), flush=True)


def run_kernel_arm(args):
    """Stand-alone secondary arms, one JSON line each."""
    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    clocks.mark("t0")
    if args.kernel == "prefix":
        r = measure_prefix(dev, args.steps, args.warmup)
        line = {"metric": "prefix pass TFLOP/s", "value": r["tflops"], "unit": "TFLOP/s", "higher_is_better": True,
                "ms_per_step": r["us"] * 1e-3, "roofline": {"bound": "tensor", "achieved": r["tflops"],
                                                            "peak": r["peak"], "unit": "TFLOP/s", "frac": r["frac"],
                                                            "peak_kind": r["peak_kind"]}, "detail": r}
    elif args.kernel == "hybrid":
        r = measure_hybrid(dev, args.steps, args.warmup)
        line = {"metric": "tree-verify attention us (prefix + tree, merged)", "value": r["us"], "unit": "us",
                "higher_is_better": False, "ms_per_step": r["us"] * 1e-3, "detail": r}
    elif args.kernel == "w4a16":
        r = measure_w4a16(dev, args.steps, args.warmup, [int(m) for m in args.w4_m.split(",")])
        m = "64" if "64" in r["sweep"] else min(r["sweep"], key=int)
        v = r["sweep"][m]
        line = {"metric": f"W4A16 weight-stream GB/s (M={m})", "value": v["weight_gbs"], "unit": "GB/s",
                "higher_is_better": True, "ms_per_step": v["us_per_layer"] * 1e-3,
                "roofline": {"bound": "hbm", "achieved": v["weight_gbs"], "peak": r["hbm_peak"], "unit": "GB/s",
                             "frac": v["hbm_frac"], "peak_kind": r["hbm_peak_kind"]}, "detail": r}
    elif args.kernel == "parents":
        r = measure_parents(dev, args.steps, args.warmup)
        line = {"metric": "explicit-parent ancestor attention GB/s (C2-sized pruned batch)",
                "value": r["C2_sized_pruned_b8_d5"]["gbs"], "unit": "GB/s", "higher_is_better": True, "detail": r}
    elif args.kernel == "verify":
        r = measure_verify(ws, rank, dev, args.steps, args.warmup, args.verify_layers)
        line = {"metric": "W4A16 verify-step tokens/s", "value": r.get("tokens_per_s"), "unit": "tokens/s",
                "higher_is_better": True, "scaling": "strong", "ms_per_step": r.get("ms_per_step"), "detail": r}
    else:  # "triton": the reference's Triton kernel alone on the selected config
        r = time_triton_reference(args.config, dev, args.steps, args.warmup)
        line = {"metric": "reference Triton ancestor kernel GB/s", "value": r.get("gbs"), "unit": "GB/s",
                "higher_is_better": True, "detail": r}
    clocks.mark("t1")
    if rank == 0:
        clocks.stop()
        line.update({"n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "dtype": "f16",
                     "data": "synthetic", "clocks": clocks.summary()})
        print(json.dumps(line), flush=True)


def _finish():
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=HEADLINE, choices=sorted(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--no-secondary", dest="secondary", action="store_false",
                    help="headline only (no C2/C4/C5/W4A16/Triton measurements)")
    ap.add_argument("--kernel", default="ancestor",
                    choices=["ancestor", "prefix", "hybrid", "w4a16", "verify", "triton", "parents"])
    ap.add_argument("--verify-layers", type=int, default=0, help="override the layer count (tests only)")
    ap.add_argument("--w4-m", default="16,64,1023,8184", help="token counts of the w4a16 measurement")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.kernel != "ancestor":
        run_kernel_arm(args)
    else:
        run_ours(args)
    _finish()


if __name__ == "__main__":
    main()
