"""Benchmark of the tree-verification hot path (one JSON line on rank 0).

Workload (N=1 headline): bench config C2 — B=8 complete 4-ary trees of depth
5 (N=1365 tokens each, 10920 packed), H=32, D=128, fp16, no prefix. One step =
one ancestor-walk attention pass over the batch (``ragged_attention_with_lse``
semantics, O and LSE written). ``--config C3`` selects config 3 (B=16 binary
trees of depth 9).

value  = algorithmic HBM bytes of all ranks' steps / device time (GB/s), where
         algorithmic bytes = Q, K, V read once + O written once + LSE (4 B/row).
e2e    = the same metric through the public API with pinned host buffers:
         H2D of Q/K/V, the call, D2H of O and LSE inside the timed region.
Multi-GPU (torchrun): each rank runs its own batch of the workload (trees are
independent; weak scaling); no collective inside the timed region; one NCCL
all-gather of per-rank checksums afterwards.

``--impl reference`` times the reference's CPU path for this operator (padded
masked SDPA, restated in oracle/, all host threads) on a bounded sample.

Secondary arms (one JSON line each, N=1; used for the profiles of the other
hot-path kernels, not the headline):
``--kernel prefix``  bench config C4's shared-prefix pass (B=16, L=10240 prefix
                     keys, 341 tree queries, GQA 32/8, D=128): TFLOP/s against
                     the measured bf16 tensor peak.
``--kernel verify``  config 5: the W4A16 tree-verify step of random-init
                     Llama-3.1-8B (32 layers) on B=8 sequences (2048-token prefix
                     + binary depth-9 tree), tokens/s; under torchrun the 8
                     sequences are split over the ranks (strong scaling).
``--kernel hybrid``  config 4 whole: prefix pass + ancestor pass with the LSE
                     merge fused (``tree_verify_attention``), µs per call.
``--kernel w4a16``   the W4A16 linears of one Llama-3.1-8B decoder layer (q/k/v
                     and gate/up fused along N: 4 GEMMs)
                     (config 5's architecture, random-init int4 weights) at
                     M = 16, 64, 1023 and 8184 tokens; value = weight-stream
                     GB/s at M = 64 (HBM-bound regime), the sweep in ``sweep``.
"""
from __future__ import annotations

import argparse
import json
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
L2_BYTES = 126 * 1024 * 1024


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


def make_inputs(cfg: str, seed: int):
    """Seeded synthetic fp16 N(0,1) inputs on the host: packed Q, K, V and cu_seqlens."""
    B, b, d, H, D = CONFIGS[cfg]
    N = _num_nodes(b, d)
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn(B * N, H, D, generator=g, dtype=torch.float32).half() for _ in range(3))
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32)
    return Q, K, V, cu, (B, b, d, H, D, N)


def _traffic_from_profile(cfg: str):
    """DRAM bytes per launch of the ancestor kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "ancestor_attn_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        j = json.load(f)
    return j.get(cfg, {}).get("dram_bytes_per_launch")


def cpu_reference_step(Q, K, V, shape, heads: int, trees: int = 1):
    """The reference's CPU path on a sample: padded masked SDPA over `trees` trees × `heads` heads."""
    from oracle import tree_attn_oracle as orc
    B, b, d, H, D, N = shape
    mask = orc.ancestor_mask(N, b, d)
    qs = [Q[i * N:(i + 1) * N, :heads] for i in range(trees)]
    ks = [K[i * N:(i + 1) * N, :heads] for i in range(trees)]
    vs = [V[i * N:(i + 1) * N, :heads] for i in range(trees)]
    return orc.padded_sdpa(qs, ks, vs, [mask] * trees)


def cpu_sample_plan(Q, K, V, shape, per_step_budget_s: float):
    """Pick how many heads of one tree a CPU step covers so it fits the budget."""
    B, b, d, H, D, N = shape
    t0 = time.perf_counter()
    cpu_reference_step(Q, K, V, shape, 1)
    t1 = time.perf_counter() - t0
    heads = int(max(1, min(H, per_step_budget_s // max(t1, 1e-6))))
    return heads


def run_reference(args):
    """--impl reference: the reference's CPU implementation of the path (oracle restatement)."""
    ws, rank, _ = _dist()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    Q, K, V, cu, shape = make_inputs(args.config, 0)
    B, b, d, H, D, N = shape
    heads = cpu_sample_plan(Q, K, V, shape, 150.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference_step(Q, K, V, shape, heads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(Q, K, V, shape, heads)
    dt = (time.perf_counter() - t0) / args.steps
    nbytes = algorithmic_bytes(N, heads, D)
    gbs = nbytes / dt / 1e9
    sample = f"1 of {B} trees x {heads} of {H} heads per step (padded masked SDPA, fp32, torch CPU)"
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": _config_dict(args.config, shape),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config_dict(cfg, shape):
    B, b, d, H, D, N = shape
    return {"workload": f"{cfg}: B={B} complete {b}-ary trees depth {d} (N={N}/tree, T={B * N}), "
                        f"H={H}, D={D}, fp16 I/O, no prefix",
            "batch": B, "branching": b, "depth": d, "heads": H, "head_dim": D, "tokens": B * N,
            "parallelism": "trees sharded per rank (weak scaling)",
            "l2": "rotating input copies, total > 3x the 126 MB L2"}


def run_ours(args):
    from qattention_b200 import ragged_attn as ra

    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    Qh, Kh, Vh, cu, shape = make_inputs(args.config, 1000 * rank)
    B, b, d, H, D, N = shape
    T = B * N
    nbytes = algorithmic_bytes(T, H, D)
    in_bytes = 3 * T * H * D * 2
    copies = max(2, -(-3 * L2_BYTES // nbytes))
    ins = [(Qh.to(dev), Kh.to(dev), Vh.to(dev)) for _ in range(copies)]
    cud = cu.to(dev)
    O = torch.empty(T, H, D, dtype=torch.float16, device=dev)
    L = torch.empty(T, H, dtype=torch.float32, device=dev)

    def step(i):
        Q, K, V = ins[i % copies]
        ra._ancestor(Q, K, V, cud, N, branching=b, max_depth=d, want_lse=True, out=O, lse_out=L)

    # CUDA graphs of back-to-back steps over the rotating input copies: one of G steps
    # (the kernel is launched with programmatic dependent launch, so a step plans its
    # first tile while the previous step finishes, as consecutive launches of a serving
    # loop do; each step still waits for the previous one before touching memory) and
    # one single-step graph per copy for a remainder, so that exactly K steps run
    G = copies * max(1, 8 // copies)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(copies):
            step(i)
    torch.cuda.current_stream(dev).wait_stream(stream)
    graph_g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_g):
        for j in range(G):
            step(j)
    graphs = []
    for i in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(i)
        graphs.append(g)

    def run(n):  # exactly n steps
        for _ in range(n // G):
            graph_g.replay()
        for i in range(n % G):
            graphs[i % copies].replay()

    run(args.warmup)
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(ws)
    torch.cuda.synchronize(dev)
    clocks.mark("t0")
    e0.record(cur)
    run(args.steps)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    clocks.mark("t1")
    _barrier(ws)
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = _max_over_ranks(ms, ws)
    if rank == 0:
        clocks.stop()

    # end to end through the public API: pinned host inputs, H2D + call + D2H in the timed region
    Qp, Kp, Vp = Qh.pin_memory(), Kh.pin_memory(), Vh.pin_memory()
    Op = torch.empty(T, H, D, dtype=torch.float16).pin_memory()
    Lp = torch.empty(T, H, dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        Qd, Kd, Vd = (x.to(dev, non_blocking=True) for x in (Qp, Kp, Vp))
        Od, Ld = ra.ragged_attention_with_lse(Qd, Kd, Vd, cu, b, d)
        Op.copy_(Od, non_blocking=True)
        Lp.copy_(Ld, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    _barrier(ws)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(cur)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(cur)
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1) / e2e_steps, ws)

    # the only collective: gather per-rank output checksums to every rank (after timing)
    csum = torch.stack([O.float().sum(), L.sum()]).double()
    if ws > 1:
        import torch.distributed as dist
        gathered = [torch.zeros_like(csum) for _ in range(ws)]
        dist.all_gather(gathered, csum)
    if rank != 0:
        return

    peak, peak_kind = _peaks()
    gbs = nbytes * ws / (ms_max * 1e-3) / 1e9
    per_gpu_gbs = nbytes / (ms * 1e-3) / 1e9
    cpu_base = None
    if ws == 1 and not args.skip_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        heads = cpu_sample_plan(Qh, Kh, Vh, shape, 2.0)
        t0 = time.perf_counter()
        n = 0
        while True:
            cpu_reference_step(Qh, Kh, Vh, shape, heads)
            n += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        cdt = (time.perf_counter() - t0) / n
        cpu_base = {"value": algorithmic_bytes(N, heads, D) / cdt / 1e9, "unit": "GB/s",
                    "cores": torch.get_num_threads(), "kind": "port",
                    "sample": f"{n} runs x 1 of {B} trees x {heads} of {H} heads "
                              "(padded masked SDPA, fp32, torch CPU)"}
    traffic = _traffic_from_profile(args.config)
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "us_per_step": ms_max * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": {**_config_dict(args.config, shape),
                                        "graphs": f"{G} back-to-back steps per CUDA graph over the rotating copies "
                                                  "(programmatic dependent launch between steps)"},
        "roofline": {"bound": "hbm", "achieved": per_gpu_gbs, "peak": peak, "unit": "GB/s",
                     "frac": per_gpu_gbs / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes": nbytes,
                     "kernel": "ancestor_tc_kernel (qa_ancestor_attn)"},
        "cpu_baseline": cpu_base,
        "e2e": {"value": nbytes * ws / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": T * H * D * 2 + T * H * 4},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "checksum": [float(x) for x in csum.tolist()],
    }
    print(json.dumps(line), flush=True)


def _timed_graphs(graphs, steps, warmup, dev):
    """Replays the captured graphs round-robin; returns ms per replay (CUDA events)."""
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for i in range(steps):
        graphs[i % len(graphs)].replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / steps


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


def _tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def run_prefix(args):
    """Shared-prefix pass of config 4 (tcgen05 kernel), TFLOP/s."""
    from qattention_b200 import ragged_attn as ra
    dev = torch.device("cuda", 0)
    B, L, N, Hq, Hkv, D = 16, 10240, 341, 32, 8, 128
    g = torch.Generator().manual_seed(4)
    Q = torch.randn(B, N, Hq, D, generator=g).half().to(dev)
    K = torch.randn(B, L, Hkv, D, generator=g).half().to(dev)
    V = torch.randn(B, L, Hkv, D, generator=g).half().to(dev)
    graphs = _capture(lambda i: ra.prefix_attention_with_lse(Q, K, V), 1, dev)
    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark("t0")
    ms = _timed_graphs(graphs, args.steps, args.warmup, dev)
    clocks.mark("t1")
    clocks.stop()
    flops = 4.0 * B * Hq * N * L * D
    tf = flops / (ms * 1e-3) / 1e12
    peak, kind = _tensor_peak()
    print(json.dumps({
        "metric": "prefix pass TFLOP/s", "value": tf, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "f16",
        "data": "synthetic", "config": {"workload": "C4 prefix pass: B=16, L=10240 prefix keys, N=341 tree "
                                        "queries, GQA 32/8, D=128, fp16", "l2": "K/V 671 MB > L2"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                     "peak_kind": kind, "flops_per_launch": flops, "kernel": "prefix_attn_kernel (qa_prefix_attn)"},
        "gpu_launches": args.steps, "clocks": clocks.summary()}), flush=True)


# (name, K, N) of one Llama-3.1-8B decoder layer, Y = X W with W [K, N]; q/k/v
# and gate/up are fused along N as serving stacks load them (same weights, 4 GEMMs)
def run_hybrid(args):
    """Config 4 whole verify attention: tcgen05 prefix pass + ancestor pass with the LSE merge fused."""
    from qattention_b200 import ragged_attn as ra
    dev = torch.device("cuda", 0)
    B, L, b, d, Hq, Hkv, D = 16, 10240, 4, 4, 32, 8, 128
    N = _num_nodes(b, d)
    g = torch.Generator().manual_seed(6)
    Q = torch.randn(B, Hq, N, D, generator=g).half().to(dev)
    K = torch.randn(B, Hkv, L + N, D, generator=g).half().to(dev)
    V = torch.randn(B, Hkv, L + N, D, generator=g).half().to(dev)
    graphs = _capture(lambda i: ra.tree_verify_attention(Q, K, V, b, d), 1, dev)
    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark("t0")
    ms = _timed_graphs(graphs, args.steps, args.warmup, dev)
    clocks.mark("t1")
    clocks.stop()
    prefix_flops = 4.0 * B * Hq * N * L * D
    print(json.dumps({
        "metric": "tree-verify attention us (prefix + tree, merged)", "value": ms * 1e3, "unit": "us",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
        "dtype": "f16", "data": "synthetic",
        "config": {"workload": "C4: B=16, L=10240 cached prefix + complete 4-ary depth-4 tree (N=341), "
                               "GQA 32/8, D=128; ragged_attention tree_verify_attention (KV cache layout "
                               "[B, Hkv, L+N, D], no repeat_kv)", "l2": "K/V 2.1 GB > L2"},
        "prefix_tflops": prefix_flops / (ms * 1e-3) / 1e12,
        "gpu_launches": args.steps * 2, "clocks": clocks.summary()}), flush=True)


LLAMA_LINEARS = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 28672), ("down", 14336, 4096)]


def run_w4a16(args):
    """One decoder layer's W4A16 linears (random-init int4 weights) at several M."""
    import ctypes
    from qattention_b200 import _lib, quant
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    layer = []
    for _, K, N in LLAMA_LINEARS:
        qw, sc = quant.quantize_w4a16(torch.randn(K, N, generator=g) * 0.02)
        layer.append((qw.to(dev), sc.to(dev), K, N))
    wbytes = sum(qw.numel() * 4 + sc.numel() * 2 for qw, sc, _, _ in layer)
    copies = max(2, -(-3 * L2_BYTES // wbytes))
    layers = [layer] + [[(qw.clone(), sc.clone(), K, N) for qw, sc, K, N in layer] for _ in range(copies - 1)]
    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark("t0")
    sweep = {}
    for M in [int(m) for m in args.w4_m.split(",")]:
        xs = {K: torch.randn(M, K, device=dev).half() for K in (4096, 14336)}
        ys = [torch.empty(M, N, dtype=torch.float16, device=dev) for _, _, _, N in layer]

        def step(i, M=M, xs=xs, ys=ys):
            for j, (qw, sc, K, N) in enumerate(layers[i % copies]):
                quant.w4a16_linear(xs[K], qw, sc, out=ys[j])

        graphs = _capture(step, copies, dev)
        steps = max(copies, min(args.steps, 200 if M <= 1023 else 40))
        ms = _timed_graphs(graphs, steps, args.warmup, dev)
        flops = sum(2.0 * M * K * N for _, _, K, N in layer)
        launches = 0
        for _, _, K, N in layer:  # one GEMM, plus the split-K reduce when the plan splits K
            sp, wb = ctypes.c_int32(), ctypes.c_int64()
            _lib.check(_lib.lib().qa_w4a16_plan(M, N, K, ctypes.byref(sp), ctypes.byref(wb)), "qa_w4a16_plan")
            launches += 1 + (sp.value > 1)
        sweep[str(M)] = {"us_per_layer": ms * 1e3, "weight_gbs": wbytes / (ms * 1e-3) / 1e9,
                         "tflops": flops / (ms * 1e-3) / 1e12, "launches_per_layer": launches}
        del graphs
    clocks.mark("t1")
    clocks.stop()
    hb, hkind = _peaks()
    tp, tkind = _tensor_peak()
    m_small = "64" if "64" in sweep else min(sweep, key=int)
    m_large = max(sweep, key=int)
    v = sweep[m_small]["weight_gbs"]
    print(json.dumps({
        "metric": f"W4A16 weight-stream GB/s (M={m_small})", "value": v, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sweep[m_small]["us_per_layer"] * 1e-3,
        "higher_is_better": True, "dtype": "int4 x f16 -> f32 acc", "data": "synthetic (random-init weights)",
        "config": {"workload": "Llama-3.1-8B decoder layer W4A16 linears, qkv and gate_up fused "
                                "(4 GEMMs, 218.1 M weights, group 128)",
                   "l2": f"{copies} rotating weight copies (> 3x L2)"},
        "roofline": {"bound": "hbm", "achieved": v, "peak": hb, "unit": "GB/s", "frac": v / hb, "peak_kind": hkind,
                     "bytes_per_layer": wbytes, "kernel": "w4a16_gemm_kernel (qa_w4a16_gemm)"},
        "large_m_roofline": {"bound": "tensor", "M": int(m_large), "achieved": sweep[m_large]["tflops"], "peak": tp,
                             "unit": "TFLOP/s", "frac": sweep[m_large]["tflops"] / tp, "peak_kind": tkind},
        "sweep": sweep, "clocks": clocks.summary()}), flush=True)


def run_verify(args):
    """Config 5: W4A16 tree-verify step of random-init Llama-3.1-8B, tokens/s (strong scaling over ranks)."""
    from qattention_b200 import verify as vf
    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    B_all, L, b, d = 8, 2048, 2, 9
    if B_all % ws:
        raise SystemExit("config 5 shards 8 sequences: use 1, 2, 4 or 8 GPUs")
    B = B_all // ws
    N = _num_nodes(b, d)
    cfg = vf.LlamaConfig()
    if args.verify_layers:
        cfg.layers = args.verify_layers
    model = vf.VerifyModel(cfg, dev, seed=7)
    cache = model.new_cache(B, L, N, seed=8 + rank)
    g = torch.Generator().manual_seed(9 + rank)
    tok_host = torch.randint(0, cfg.vocab, (B, N), generator=g).pin_memory()
    tokens = tok_host.to(dev)
    steps = max(1, min(args.steps, 10))
    for _ in range(max(args.warmup, 2)):
        model.step(tokens, cache, L, b, d)
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    # eager launches (for reference), then the step as one CUDA graph (VerifyModel.capture)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(steps):
        model.step(tokens, cache, L, b, d)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    eager_ms = _max_over_ranks(e0.elapsed_time(e1) / steps, ws)
    graph, logits = model.capture(tokens, cache, L, b, d)
    for _ in range(max(args.warmup, 2)):
        graph.replay()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    _barrier(ws)
    torch.cuda.synchronize(dev)
    clocks.mark("t0")
    e0.record(cur)
    for _ in range(steps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    clocks.mark("t1")
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, ws)
    if rank == 0:
        clocks.stop()
    # end to end: tokens H2D from pinned memory into the graph's input, the step, argmax tokens D2H
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
    if rank != 0:
        return
    tokens_total = B_all * N
    print(json.dumps({
        "metric": "W4A16 verify-step tokens/s", "value": tokens_total / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": ws, "steps": steps, "warmup": max(args.warmup, 2), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights x f16 activations, f32 accumulate", "data": "synthetic (random-init weights, random tokens)",
        "config": {"workload": f"C5: random-init Llama-3.1-8B architecture ({cfg.layers} layers), W4A16 linears "
                               "(qkv and gate_up fused), fp16 LM head; B=8 sequences x (2048-token cached prefix "
                               "+ binary depth-9 tree, 1023 tokens) = 8184 verify tokens per step",
                   "sequences_per_gpu": B, "parallelism": f"sequences sharded over {ws} GPU(s), no collective"},
        "e2e": {"value": tokens_total / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": B * N * 8, "d2h_bytes_per_step": B * N * 8},
        "eager_ms_per_step": eager_ms, "timing": "one CUDA graph per step (VerifyModel.capture); eager launches beside",
        "clocks": clocks.summary()}), flush=True)


def _finish():
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="C2", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--kernel", default="ancestor", choices=["ancestor", "prefix", "hybrid", "w4a16", "verify"])
    ap.add_argument("--verify-layers", type=int, default=0, help="override the layer count (tests only)")
    ap.add_argument("--w4-m", default="16,64,1023,8184", help="token counts of the w4a16 arm")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.kernel == "prefix":
        run_prefix(args)
    elif args.kernel == "hybrid":
        run_hybrid(args)
    elif args.kernel == "w4a16":
        run_w4a16(args)
    elif args.kernel == "verify":
        run_verify(args)
    else:
        run_ours(args)
    _finish()


if __name__ == "__main__":
    main()
