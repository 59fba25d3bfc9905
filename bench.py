"""Cascade-decode benchmark (BASELINE metric: cascade decode attention HBM GB/s
and us/step on the Llama-3-8B-shaped cascade, plus the SwiGLU gate_up line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one cascade decode step of one layer on synthetic inputs with the
config's shapes (B=64 requests sharing a 4096-token prefix, suffix lengths
U[128,1024], 32 q heads / 8 kv heads, head dim 128, block size 128, bf16,
random-permutation block tables): stage-1 prefix attention over the shared
pages, per-request suffix decode, LSE merge to the bf16 output.

Multi-GPU (torchrun, one rank per GPU): attention is partitioned by kv head
with no hot-path collective, so every rank owns 8 kv heads / 32 q heads of a
model with 8N kv heads (weak scaling); NCCL is used only for the barrier, the
max-over-ranks timing and, after timing, the all_gather of the sharded
outputs that rank 0 checks against single-GPU runs.

``value`` = algorithmic bytes of all ranks / max-over-ranks device time of
exactly K steps.  The K timed steps are captured back to back in one CUDA
graph, as a decode forward runs attention layer after layer; step i reads
layer (i mod 8)'s own q and K/V pools (8 x 185 MB, far more than the 126 MB
L2), so consecutive steps never find their K/V in L2.  The same step timed
alone (L2 flushed by a 256 MiB write and a 256 MiB read before it, one event
pair around a one-step graph) is reported beside it.  ``e2e`` repeats the K
steps through the public API with host buffers: every step's q and tables
are copied from pinned host memory and its output copied back inside the
timed graph.
``--impl reference`` times the reference's CPU golden path (its numpy fp64
restatement in oracle/) on the host cores, on rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vllm-hust-cascade-kernel_b200"))

METRIC = "cascade decode attention HBM GB/s (Llama-3-8B cascade step, B=64, prefix 4096)"
FLUSH_BYTES = 256 * 1024 * 1024
LAYERS = 8          # distinct per-layer q/K/V sets the timed steps rotate through
STEP_KERNELS = 3    # suffix decode + stage-1 + combine
DECODE_TRAFFIC_BYTES = 162_836_224 + 4_373_760   # ncu dram__bytes_read.sum + dram__bytes_write.sum


class L2Flush:
    """Evict L2 between timed steps: write a buffer larger than L2, then read
    another one, leaving L2 full of clean lines (no write-back is pending when
    the timed region starts)."""

    def __init__(self, torch):
        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
        self.r = torch.zeros(FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.r.sum()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except Exception:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def setup_dist():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- ours

def run_ours(args, rank, world, local):
    import torch
    import cascade_kernel  # noqa: F401  (registers the ops; fails loudly if unbuilt)
    from cascade_kernel import capi, workloads
    from cascade_kernel.cascade import CascadeLayersGraph, CascadeStepGraph, cascade_decode

    peaks = _peaks()
    w = workloads.c2_llama8b(seed=args.seed + 1000 * rank)
    t = w.tables
    stream = torch.cuda.current_stream()
    ab = w.algorithmic_bytes()

    # Per-layer inputs, as a decode forward walks the layers: layer 0 is the
    # workload's own q/K/V, layers 1.. are seeded N(0,1) tensors of the same
    # shapes; all layers share the tables. The timed steps rotate through the
    # layers, so consecutive steps read different K/V (LAYERS x 185 MB, far
    # more than the 126 MB L2): no L2 flush is needed between them.
    layers = [(w.q, w.k_pool, w.v_pool)]
    for l in range(1, LAYERS):
        gen = torch.Generator(device="cuda").manual_seed(7919 * (args.seed + 1) + 1000 * rank + l)
        layers.append(tuple(torch.randn(x.shape, device="cuda", generator=gen).to(x.dtype)
                            for x in (w.q, w.k_pool, w.v_pool)))
    K = args.steps
    lay = [i % LAYERS for i in range(K)]

    # the K timed steps are captured in ONE CUDA graph (3 kernels per step, no
    # host work), as a serving loop replays a decode forward
    graph = CascadeLayersGraph([layers[l] + (t,) for l in lay])
    outs = graph.replay()
    torch.cuda.synchronize()
    for i in range(min(K, LAYERS)):
        assert torch.equal(outs[i], cascade_decode(*layers[lay[i]], t)), "graph step differs from the eager step"

    # the dominant kernel alone: the suffix decode kernel writing its split
    # partials (C ABI, CASCADE_FLAG_PARTIALS_ONLY: one launch, no combine),
    # K launches rotating through the layers' pools
    dom_desc = [capi.paged_desc(q, k, v, t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1,
                                flags=capi.FLAG_PARTIALS_ONLY) for q, k, v in layers]
    dom_ws = torch.empty(capi.suffix_workspace_size(dom_desc[0]), dtype=torch.uint8, device="cuda")

    def suffix_ops():
        for l in lay:
            capi.suffix_decode(dom_desc[l], None, None, dom_ws)

    suffix_ops()
    torch.cuda.synchronize()
    dom_graph = torch.cuda.CUDAGraph()       # the K launches back to back, no host gaps
    with torch.cuda.graph(dom_graph):
        suffix_ops()

    def burn(seconds):
        # back-to-back replays outside the timed regions, so that the clock
        # samples are taken under the step's own load
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end:
            for _ in range(8):
                graph.replay()
            torch.cuda.synchronize()

    for i in range(args.warmup):
        cascade_decode(*layers[i % LAYERS], t)
        capi.suffix_decode(dom_desc[i % LAYERS], None, None, dom_ws)
    graph.replay()
    torch.cuda.synchronize()

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier(world)
    with ClockSampler(local) as clk:
        burn(0.4)
        barrier(world)
        torch.cuda.synchronize()
        ev[0].record(stream)
        graph.replay()                      # exactly K steps
        ev[1].record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ev[2].record(stream)
        dom_graph.replay()                  # K launches of the dominant kernel
        ev[3].record(stream)
        torch.cuda.synchronize()
        burn(0.2)
    barrier(world)
    step_ms = max_over_ranks(ev[0].elapsed_time(ev[1]) / K, world)
    dom_ms = max_over_ranks(ev[2].elapsed_time(ev[3]) / K, world)

    # the same step timed alone: L2 flushed before each step, one event pair
    # around a one-step graph (reported beside the rotating-layer number)
    flush = L2Flush(torch)
    one = CascadeStepGraph(w.q, w.k_pool, w.v_pool, t)
    fev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    torch.cuda.synchronize()
    for a, b in fev:
        flush()
        a.record(stream)
        one.replay()
        b.record(stream)
    torch.cuda.synchronize()
    flushed_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in fev) / K, world)
    del one

    # e2e through the public API with host buffers: every step copies its
    # layer's inputs (q and the six index tensors, packed into one pinned
    # host buffer -> one H2D copy) and reads its merged output back (one D2H
    # copy), all inside the K-step graph (CascadeLayersGraph with host_io)
    tabs = [t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens, t.suffix_block_table,
            t.suffix_q_seqlens, t.suffix_kv_seqlens]
    from cascade_kernel.cascade import CascadeTables
    io, e2e_in = [], []
    for q, k, v in layers:
        parts = [q] + tabs
        offs, cur = [], 0
        for x in parts:
            offs.append(cur)
            cur += (x.numel() * x.element_size() + 255) // 256 * 256
        host_in = torch.empty(cur, dtype=torch.uint8).pin_memory()
        for x, o in zip(parts, offs):
            nb = x.numel() * x.element_size()
            host_in[o:o + nb].copy_(x.contiguous().view(-1).view(torch.uint8).cpu())
        dev_in = torch.empty(cur, dtype=torch.uint8, device="cuda")
        dev_in.copy_(host_in)
        views = [dev_in[o:o + x.numel() * x.element_size()].view(x.dtype).view(x.shape)
                 for x, o in zip(parts, offs)]
        out_h = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
        io.append((host_in, dev_in, out_h))
        e2e_in.append((views[0], k, v, CascadeTables(*views[1:], uniform_group=t.uniform_group)))
    # the copies run on copy streams inside the graph: step i's inputs load
    # while earlier steps compute, its output drains while later ones do
    e2e_graph = CascadeLayersGraph([e2e_in[l] for l in lay], host_io=[io[l] for l in lay], overlap_io=True)
    e2e_graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(io[lay[-1]][2], outs[K - 1].cpu()), "e2e output differs from the device-resident step"
    e2e_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    barrier(world)
    torch.cuda.synchronize()
    e2e_ev[0].record(stream)
    e2e_graph.replay()                      # exactly K steps, host copies included
    e2e_ev[1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e2e_ev[0].elapsed_time(e2e_ev[1]) / K, world)
    h2d = io[0][0].numel()
    d2h = io[0][2].numel() * io[0][2].element_size()
    del e2e_graph, io, e2e_in, dom_graph

    total_bytes = ab["total"] * world
    value = total_bytes / (step_ms * 1e-3) / 1e9
    dom_bytes = ab["suffix"]
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9

    gateup = gateup_sweep(flush, peaks) if not args.no_gateup else None
    # the Llama-3-70B MLP shard of the multi-GPU config: gate_up with K=8192 and
    # the 28672 intermediate columns split across the ranks, M=256 (per rank)
    mlp70 = (gateup_sweep(flush, peaks, Ms=(256,), K=8192, I=28672 // world, seed=11 + rank)
             if not args.no_gateup and 28672 % (128 * world) == 0 else None)

    norm = norm_sweep(flush, peaks) if not args.no_gateup else None

    verify = verify_sharded(args, rank, world, outs[0]) if world > 1 else None
    del graph

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.cpu_threads)

    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 5),
        "us_per_step": round(step_ms * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, random-permutation block tables)",
        "config": {
            "workload": "c2_llama3_8b_cascade: B=64, shared prefix 4096, suffix U[128,1024], "
                        "H=32/KVH=8 per rank, D=128, block_size=128",
            "suffix_tokens": int(w.suffix_lens.sum()),
            "algorithmic_bytes_per_step_per_rank": ab,
            "parallelism": f"kv-head partition x{world} (weak: 8 kv heads per rank)",
            "l2": (f"inputs larger than L2: the K timed steps rotate through {LAYERS} layers' q/K/V "
                   f"({LAYERS} x {ab['total'] / 1e6:.0f} MB vs 126 MB L2), so no step re-reads cached K/V"),
            "launch": "the K timed steps captured back to back in one CUDA graph (CascadeLayersGraph), "
                      "one replay, as a decode forward runs its layers",
            "layers": LAYERS,
        },
        # the same step timed alone: L2 flushed (256 MiB write + 256 MiB read)
        # before each step and one event pair around a one-step graph replay
        "us_per_step_flushed_alone": round(flushed_ms * 1e3, 2),
        "roofline": {
            "kernel": "paged_decode_kernel (suffix decode, split partials; K launches rotating through "
                      "the layers' pools, average launch duration)",
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4),
            # DRAM bytes (read + write) of one launch of this kernel from the ncu
            # capture summarised in profiles/paged_decode_kernel_c2.txt
            "traffic": DECODE_TRAFFIC_BYTES,
            "traffic_src": "ncu capture (profiles/paged_decode_kernel_c2.txt)",
            "peak_src": peaks["src"],
        },
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "us_per_step": round(e2e_ms * 1e3, 2), "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "how": "K steps in one graph, each copying its q + tables in from pinned host memory and its "
                       "output out; copies on copy streams overlap neighbouring steps' kernels"},
        # timed regions: the K-step graph, K dominant-kernel launches, the
        # flushed one-step replays and the K-step e2e graph
        "gpu_launches": 3 * STEP_KERNELS * K + K,
        "clocks": clk.summary(),
    }
    line["frac_of_hbm_roofline_step"] = round(value / world / peaks["hbm_gbs"], 4)
    if gateup is not None:
        line["gateup_swiglu"] = gateup
        line["gpu_launches"] += gateup.pop("_launches")
    if mlp70 is not None:
        mlp70["shape"] = (f"Llama-3-70B MLP shard: X[256,8192] x W[2*{28672 // world},8192]^T -> "
                          f"silu(gate)*up bf16 [256,{28672 // world}] per rank ({world} rank(s))")
        line["gateup_swiglu_70b_shard"] = mlp70
        line["gpu_launches"] += mlp70.pop("_launches")
    if norm is not None:
        line["add_rms_norm_stats"] = norm
        line["gpu_launches"] += norm.pop("_launches")
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if verify is not None:
        line["verify"] = verify
    return line


def verify_sharded(args, rank, world, out_local):
    """After timing: reassemble the sharded outputs with NCCL all_gather (the
    only collective on the data) and check them on rank 0 against a single-GPU
    run of every rank's shard -- the attention step output [T, H, D] of each
    rank's kv-head shard, and the gate_up + SwiGLU output [M, I/N] of each
    rank's column shard of the 70B MLP (X replicated, W rows split)."""
    import torch
    import torch.distributed as dist
    from cascade_kernel import workloads
    from cascade_kernel.cascade import cascade_decode
    res = {"collective": "torch.distributed.all_gather_into_tensor (NCCL)", "ranks": world}
    g_att = torch.empty((world,) + tuple(out_local.shape), dtype=out_local.dtype, device="cuda")
    dist.all_gather_into_tensor(g_att, out_local.contiguous())
    # gate_up column shard: X[256, 8192] shared, W shard [2 * 28672/N, 8192] per rank
    I_r = 28672 // world
    def mlp_inputs(r):
        gx = torch.Generator(device="cuda").manual_seed(99)
        x = torch.randn(256, 8192, device="cuda", generator=gx).to(torch.bfloat16)
        gw = torch.Generator(device="cuda").manual_seed(500 + r)
        w = (torch.randn(2 * I_r, 8192, device="cuda", generator=gw) * 0.02).to(torch.bfloat16)
        return x, w
    x, w = mlp_inputs(rank)
    mlp_local = torch.ops.npu.cascade_gateup_swiglu(x, w)
    del x, w
    g_mlp = torch.empty((world,) + tuple(mlp_local.shape), dtype=mlp_local.dtype, device="cuda")
    dist.all_gather_into_tensor(g_mlp, mlp_local.contiguous())
    torch.cuda.synchronize()
    if rank == 0:
        att_ok, mlp_ok = True, True
        for r in range(world):
            wr = workloads.c2_llama8b(seed=args.seed + 1000 * r)
            att_ok &= bool(torch.equal(g_att[r], cascade_decode(wr.q, wr.k_pool, wr.v_pool, wr.tables)))
            del wr
            x, w = mlp_inputs(r)
            mlp_ok &= bool(torch.equal(g_mlp[r], torch.ops.npu.cascade_gateup_swiglu(x, w)))
            del x, w
        res["attention_equal_to_single_gpu"] = att_ok
        res["gateup_equal_to_single_gpu"] = mlp_ok
    dist.barrier()
    return res


def norm_sweep(flush, peaks, reps=5, seed=5):
    """add_rms_norm_stats (npu.add_rms_norm_stats, one kernel per call) on the
    reference's two production shapes (add_rms_norm_stats_cases.py:21-22:
    prefill 2048 x 5120, decode 32 x 5120, bf16), every mode; L2 flushed
    before each timed call. Bytes = inputs read + outputs written."""
    import torch
    npu = torch.ops.npu
    g = torch.Generator(device="cuda").manual_seed(seed)
    res, launches = {}, 0
    for name, (M, K) in (("prefill", (2048, 5120)), ("decode", (32, 5120))):
        x1 = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        x2 = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        gamma = (1.0 + torch.randn(K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        beta = (torch.randn(K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        for mode in (0, 1, 2):
            fn = lambda: npu.add_rms_norm_stats(x1, x2, gamma, beta, 1e-6, mode)
            for _ in range(3):
                fn()
            ts = []
            for _ in range(reps):
                flush()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b) * 1e3)
                launches += 1
            ts.sort()
            us = ts[len(ts) // 2]
            byts = {0: 3 * M * K * 2, 1: 2 * M * K * 2 + 2 * K * 2, 2: 2 * M * K * 2}[mode] + 4 * ((M + 7) // 8 * 8)
            res[f"{name}_mode{mode}"] = {"us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
                                         "frac_hbm": round(byts / us / 1e3 / peaks["hbm_gbs"], 4)}
    return {"shape": "bf16 rows x 5120: prefill M=2048, decode M=32; mode 0 residual+stats, 1 stats+apply "
                     "(gamma, beta), 2 stats only", "per_case": res, "_launches": launches}


def gateup_sweep(flush, peaks, Ms=(1, 16, 64, 256, 4096), K=4096, I=14336, reps=5, seed=7):
    """gate_up + SwiGLU (default: Llama-3-8B, X[M,4096] x W[2*14336,4096]^T -> bf16 [M,14336])
    through torch.ops.npu.cascade_gateup_swiglu (one tcgen05 kernel per call).
    Per M: TFLOP/s (tensor bound at M=4096) and GB/s (HBM bound for M<=256)."""
    import torch
    npu = torch.ops.npu
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    res, launches = {}, 0
    for M in Ms:
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        for _ in range(3):
            npu.cascade_gateup_swiglu(x, w)
        ts = []
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            npu.cascade_gateup_swiglu(x, w)
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
            launches += 1
        ts.sort()
        us = ts[len(ts) // 2]
        flops = 2.0 * M * K * 2 * I
        byts = 2.0 * M * K + 2.0 * 2 * I * K + 2.0 * M * I
        res[str(M)] = {"us": round(us, 2), "tflops": round(flops / us / 1e6, 1), "gbs": round(byts / us / 1e3, 1),
                       "frac_tensor": round(flops / us / 1e6 / peaks["bf16_tflops"], 4),
                       "frac_hbm": round(byts / us / 1e3 / peaks["hbm_gbs"], 4)}
    return {"shape": "X[M,4096] x W[28672,4096]^T -> silu(gate)*up bf16 [M,14336]", "per_M": res,
            "peak_tflops": peaks["bf16_tflops"], "peak_src": peaks["src"], "_launches": launches}


# ----------------------------------------------------------------- CPU baseline

def _cpu_task(payload):
    from oracle import cascade_oracle as O
    (qh, kh, vh, bt_p, gs, pl, bt_s, sl, heads) = payload
    t0 = time.perf_counter()
    O.cascade_step_ref(qh, kh, vh, bt_p, gs, pl, bt_s, sl, kv_heads_subset=heads)
    return time.perf_counter() - t0


def cpu_baseline(w, threads=None, kv_heads=None):
    """The reference's CPU golden path (numpy fp64, oracle/cascade_oracle.py)
    on the same workload: the full cascade step (all 8 kv heads) split over a
    process pool by kv head.  Returns the cpu_baseline object."""
    import multiprocessing as mp
    import numpy as np
    import torch
    threads = threads or os.cpu_count() or 1
    kvh = w.k_pool.shape[2]
    heads = list(range(kvh)) if kv_heads is None else list(kv_heads)
    f64 = lambda x: x.float().cpu().numpy().astype(np.float64)
    qh = f64(w.q)
    # only the pages the step touches travel to the workers
    bt_p = w.tables.prefix_block_table.cpu().numpy()
    bt_s = w.tables.suffix_block_table.cpu().numpy()
    kf, vf = w.k_pool.float().cpu().numpy(), w.v_pool.float().cpu().numpy()
    payloads = []
    for g in heads:
        group = qh.shape[1] // kvh
        payloads.append((qh[:, g * group:(g + 1) * group], kf[:, :, g:g + 1].astype(np.float64),
                         vf[:, :, g:g + 1].astype(np.float64), bt_p, w.group_sizes, w.prefix_lens, bt_s,
                         w.suffix_lens, [0]))
    workers = min(threads, len(payloads))
    t0 = time.perf_counter()
    if workers > 1:
        ctx = mp.get_context("spawn")
        with ctx.Pool(workers) as pool:
            pool.map(_cpu_task, payloads)
    else:
        for pl in payloads:
            _cpu_task(pl)
    wall = time.perf_counter() - t0
    ab = w.algorithmic_bytes()["total"] * len(heads) / kvh
    return {"value": round(ab / wall / 1e9, 4), "unit": "GB/s", "cores": workers, "kind": "port",
            "sample": f"full C2 cascade step, {len(heads)} of {kvh} kv heads, numpy fp64 oracle "
                      f"(spawned pool over kv heads), wall {wall:.2f} s",
            "seconds": round(wall, 3)}


def run_reference(args, rank, world):
    import torch
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "vllm-hust-cascade-kernel_b200"))
    from cascade_kernel import workloads
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = workloads.c2_llama8b(seed=args.seed, device=dev)
    threads = args.cpu_threads or os.cpu_count() or 1
    vals, secs = [], []
    for i in range(args.warmup + args.steps):
        c = cpu_baseline(w, threads)
        if i >= args.warmup:
            vals.append(c["value"])
            secs.append(c["seconds"])
    v = sum(vals) / len(vals)
    return {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(secs) / len(secs), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded)", "config": {"workload": "c2_llama3_8b_cascade (same as ours)"},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": c["cores"], "kind": "port",
                             "sample": c["sample"]},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gateup", action="store_true",
                    help="skip the gate_up SwiGLU and add_rms_norm_stats sweeps")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, world, local = setup_dist()
    line = run_ours(args, rank, world, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
