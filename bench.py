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
# config.workload, byte-identical in both arms
WORKLOAD = ("c2_llama3_8b_cascade: B=64, shared prefix 4096, suffix U[128,1024], H=32/KVH=8 per rank, D=128, "
            "block_size=128")
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


def bind_to_gpu_numa(device):
    """Restrict this process to the CPUs NVML reports as local to `device`
    (read-only NVML query; nothing on the GPU changes), so the pinned host
    buffers of the e2e copies, allocated afterwards, are placed on the GPU's
    own NUMA node (first touch) instead of wherever the launcher started the
    rank. Returns the CPU count bound to, or None when NVML is unavailable."""
    try:
        import pynvml
        import torch
        props = torch.cuda.get_device_properties(device)
        pynvml.nvmlInit()
        try:
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, m in enumerate(words) for b in range(64) if (int(m) >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:  # no NVML, an older driver, or a platform without affinity
        return None
    return None


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
        bind_to_gpu_numa(local)
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

    # on one GPU, the same shard at the widths 2, 4 and 8 ranks own (the
    # narrow ones take the split-K cluster-of-pairs form)
    mlp70_widths = None
    if not args.no_gateup and world == 1:
        mlp70_widths = {"per_ranks": {}, "_launches": 0}
        for r in (2, 4, 8):
            blk = gateup_sweep(flush, peaks, Ms=(256,), K=8192, I=28672 // r, seed=11)
            mlp70_widths["_launches"] += blk.pop("_launches")
            mlp70_widths["per_ranks"][str(r)] = dict(blk["per_M"]["256"], I=28672 // r)

    norm = norm_sweep(flush, peaks) if not args.no_gateup else None

    verify = verify_sharded(args, rank, world, outs[0]) if world > 1 else None
    del graph
    torch.cuda.empty_cache()

    c4 = c4_sharded_block(args, peaks, rank, world, K) if not args.no_extra else None
    c5 = c5_block(peaks, K) if (world == 1 and not args.no_extra) else None
    roof = read_roof_block(peaks, achieved) if (world == 1 and not args.no_extra) else None
    hostwall = host_wall_block() if (world == 1 and not args.no_extra) else None

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
            "workload": WORKLOAD,
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
    if mlp70_widths is not None:
        line["gpu_launches"] += mlp70_widths.pop("_launches")
        mlp70_widths["shape"] = ("Llama-3-70B MLP shard on one GPU at the per-rank width of 2/4/8 ranks: "
                                 "X[256,8192] x W[2*28672/r,8192]^T -> silu(gate)*up bf16 [256,28672/r]")
        line["gateup_swiglu_70b_shard_widths"] = mlp70_widths
    if norm is not None:
        line["add_rms_norm_stats"] = norm
        line["gpu_launches"] += norm.pop("_launches")
    for key, blk in (("c4_sharded", c4), ("c5_ragged", c5), ("hbm_read_roof", roof), ("eager_host_wall", hostwall)):
        if blk is not None:
            line["gpu_launches"] += blk.pop("_launches")
            line[key] = blk
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


def _time_graph(graph, K, stream):
    """Average device time (ms) of K back-to-back replays of a step graph."""
    import torch
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(K):
        graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / K


def kernel_times(w, K):
    """Stage-1 alone and the suffix decode alone on workload w (split
    partials, no combine: CASCADE_FLAG_PARTIALS_ONLY through the C ABI), each
    the average of K back-to-back launches in one graph. Returns (stage-1 us,
    decode us)."""
    import torch
    from cascade_kernel import capi
    t = w.tables
    res = []
    for bt, qs, kvs, qv, stage1 in ((t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens, t.uniform_group,
                                     True),
                                    (t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1, False)):
        d = capi.paged_desc(w.q, w.k_pool, w.v_pool, bt, qs, kvs, qv, flags=capi.FLAG_PARTIALS_ONLY)
        n = capi.stage1_workspace_size(d) if stage1 else capi.suffix_workspace_size(d)
        ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
        fn = (lambda: capi.fa_fp32_stage1(d, None, None, ws)) if stage1 else (lambda: capi.suffix_decode(d, None, None, ws))
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(K):
                fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        res.append(a.elapsed_time(b) / K * 1e3)
        del g, ws
    return res


def c5_block(peaks, K, seed=0):
    """BASELINE config 5, the ragged stress case (N=1): 32 prefix groups of 16
    requests, prefixes lognormal(median 1024, sigma 1) in [16, 32768], suffixes
    lognormal(median 200, sigma 1) with 5% forced to 0, H=40/KVH=8, bs=16, fp16.
    One step (suffix decode, stage-1, combine) captured in a graph and replayed
    K times back to back (the pools are ~0.8 GB, far above the L2)."""
    import numpy as np
    import torch
    from cascade_kernel import workloads
    from cascade_kernel.cascade import CascadeStepGraph
    w = workloads.c5_ragged(seed=seed)
    g = CascadeStepGraph(w.q, w.k_pool, w.v_pool, w.tables)
    for _ in range(3):
        g.replay()
    ms = _time_graph(g, K, torch.cuda.current_stream())
    ab = w.algorithmic_bytes()
    gbs = ab["total"] / (ms * 1e-3) / 1e9
    suf = np.asarray(w.suffix_lens)
    del g
    s1_us, dec_us = kernel_times(w, K)
    return {"shape": "c5_ragged: 32 groups x 16 requests, prefix lognormal(ln 1024, 1.0) clipped [16, 32768], "
                     "suffix lognormal(ln 200, 1.0) with 5% zeros, H=40/KVH=8, D=128, block_size=16, fp16",
            "sigma_prefix": 1.0, "sigma_suffix": 1.0, "group_split": "16 requests per group", "zero_fraction":
            round(float((suf == 0).mean()), 4), "prefix_tokens": int(sum(w.prefix_lens)),
            "suffix_tokens": int(suf.sum()), "algorithmic_bytes_per_step": ab, "us_per_step": round(ms * 1e3, 2),
            "gbs": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "stage1_alone_us": round(s1_us, 2), "suffix_decode_alone_us": round(dec_us, 2),
            "_launches": 5 * K}


def c4_sharded_block(args, peaks, rank, world, K, seed=0):
    """BASELINE config 4's attention, ONE Llama-3-70B-shaped model (4 prefix
    groups x 64 requests, 16384-token prefixes, suffix U[256,2048], 64 q / 8 kv
    heads, bf16) partitioned by kv head over the N ranks: rank r runs its
    8/N kv heads and their q heads (sharding.shard_attention), tables
    replicated, no collective in the step. The step is captured in a graph and
    replayed K times; the time is the max over ranks. Strong scaling: the
    same model at every N. After timing, NCCL all_gather of the rank outputs,
    checked bit for bit on rank 0 against the unsharded step, which rank 0
    also times (T1) in the same run."""
    import torch
    from cascade_kernel import sharding, workloads
    from cascade_kernel.cascade import CascadeStepGraph, cascade_decode
    stream = torch.cuda.current_stream()
    w = workloads.c4_llama70b(seed=seed)
    ab, fl = w.algorithmic_bytes(), w.flops()
    q, k, v = sharding.shard_attention(w.q, w.k_pool, w.v_pool, rank, world)
    full = shard_ref = None
    if rank == 0:
        full = cascade_decode(w.q, w.k_pool, w.v_pool, w.tables)
        # every rank's shard run on this one GPU: the same shapes (hence the
        # same splits and quantisation structure) as on its rank
        shard_ref = torch.cat([cascade_decode(*sharding.shard_attention(w.q, w.k_pool, w.v_pool, r, world),
                                              w.tables) for r in range(world)], dim=1)
        t1_graph = CascadeStepGraph(w.q, w.k_pool, w.v_pool, w.tables)
        for _ in range(3):
            t1_graph.replay()
        t1_ms = _time_graph(t1_graph, K, stream)
        del t1_graph
        s1_us, dec_us = kernel_times(w, K)
    if world > 1 or rank != 0:
        w.q = w.k_pool = w.v_pool = None
    torch.cuda.empty_cache()
    g = CascadeStepGraph(q, k, v, w.tables)
    for _ in range(3):
        g.replay()
    barrier(world)
    ms = max_over_ranks(_time_graph(g, K, stream), world)
    out = g.replay()
    torch.cuda.synchronize()
    res = {"shape": "c4_llama3_70b attention: 4 groups x 64 requests, prefix 16384, suffix U[256,2048], "
                    f"H=64/KVH=8 split by kv head over {world} rank(s) ({8 // world} kv heads each), bf16",
           "scaling": "strong (one model, kv heads split across ranks)", "ranks": world,
           "us_per_step": round(ms * 1e3, 2), "algorithmic_bytes_per_step_all_ranks": ab,
           "flops_per_step_all_ranks": fl,
           "gbs_aggregate": round(ab["total"] / (ms * 1e-3) / 1e9, 1),
           "tflops_aggregate": round(fl["total"] / (ms * 1e-3) / 1e12, 1),
           "frac_hbm_per_gpu": round(ab["total"] / world / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
           "_launches": 3 * K * (2 if rank == 0 else 1) + (2 * K if rank == 0 else 0)}
    if world > 1:
        import torch.distributed as dist
        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device="cuda")
        dist.all_gather_into_tensor(gathered, out.contiguous())
        torch.cuda.synchronize()
        if rank == 0:
            B, Hr, D = out.shape
            assembled = gathered.permute(1, 0, 2, 3).reshape(B, world * Hr, D)
            # bit for bit: the gathered outputs against the same shards run on
            # one GPU; against the unsharded model (whose stage-1 splits differ
            # with the kv-head count) within the output dtype's rounding
            res["nccl_all_gather_equal_to_shards_on_1gpu"] = bool(torch.equal(assembled, shard_ref))
            res["max_abs_diff_vs_unsharded"] = float((assembled.float() - full.float()).abs().max())
        dist.barrier()
    elif rank == 0:
        res["equal_to_unsharded"] = bool(torch.equal(out, full))
    if rank == 0:
        res["us_per_step_unsharded_1gpu"] = round(t1_ms * 1e3, 2)
        # the two attention kernels of the unsharded step alone (stage-1: 137.4
        # GFLOP, tensor-bound; the suffix decode: HBM-bound)
        res["stage1_alone_us_1gpu"] = round(s1_us, 2)
        res["stage1_tflops_1gpu"] = round(fl["stage1"] / (s1_us * 1e-6) / 1e12, 1)
        res["stage1_frac_tensor_1gpu"] = round(fl["stage1"] / (s1_us * 1e-6) / 1e12 / peaks["bf16_tflops"], 4)
        res["suffix_decode_alone_us_1gpu"] = round(dec_us, 2)
        res["strong_scaling_efficiency"] = round(t1_ms / (world * ms), 4)
    del g, q, k, v, full, shard_ref
    torch.cuda.empty_cache()
    return res


def read_roof_block(peaks, dom_gbs, reps=10, gib=2):
    """The HBM read roof on this GPU: cascade_probe_hbm_read over a 2 GiB
    buffer (far above the L2) in its four modes -- plain 16-byte loads, the
    bulk-copy engine, and the decode kernel's paged 2-D TMA pattern without
    its math (rows of 8 kv heads x 256 bytes, one head's slice per CTA item),
    items in row-major and in kv-head-major order -- each timed over `reps`
    back-to-back launches."""
    import torch
    from cascade_kernel import capi
    buf = torch.empty(gib << 30, dtype=torch.uint8, device="cuda")
    buf.random_(0, 255)
    sink = torch.zeros(2048, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    res = {}
    for mode, name in ((0, "plain_loads"), (1, "bulk_copy"), (2, "paged_tma_no_math"),
                       (3, "paged_tma_no_math_head_major")):
        for _ in range(2):
            capi.probe_hbm_read(buf, mode, 2048, sink)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(reps):
            capi.probe_hbm_read(buf, mode, 2048, sink)
        b.record(stream)
        torch.cuda.synchronize()
        gbs = buf.numel() / (a.elapsed_time(b) / reps * 1e-3) / 1e9
        res[name] = {"gbs": round(gbs, 1), "frac_of_copy_peak": round(gbs / peaks["hbm_gbs"], 4)}
    best = max(v["gbs"] for v in res.values())
    del buf
    torch.cuda.empty_cache()
    out = {"what": "read-only streaming of a 2 GiB buffer (cascade_probe_hbm_read), 10 back-to-back launches "
                   "per mode", "per_mode": res, "best_read_gbs": best, "_launches": 4 * (reps + 2)}
    if dom_gbs is not None:
        out["decode_kernel_frac_of_best_read"] = round(dom_gbs / best, 4)
        out["decode_kernel_frac_of_paged_pattern"] = round(dom_gbs / res["paged_tma_no_math"]["gbs"], 4)
    return out


def host_wall_block(reps=300, seed=3):
    """Eager host wall of the reference's ops at the shapes its README quotes
    host walls for (ascend-kernel/README.md:315-317; method of
    fa_fp32_stage1/test/run_perf_driver.py:49-60: 10 warm-up calls, then
    `reps` calls back to back, one synchronize, wall / reps): fa_fp32_stage1
    fast path at T=64 query tokens of one prefix group, kv=4356, H=40/KVH=8,
    bf16; lse_merge at B=64 x H=40 x 128 (o1 fp32 padded-LSE, o2 bf16,
    out_code=1). Device time per call (CUDA events around the same loop) is
    reported beside it."""
    import numpy as np
    import torch
    npu = torch.ops.npu
    g = torch.Generator(device="cuda").manual_seed(seed)
    T, H, KVH, kv = 64, 40, 8, 4356
    pages = (kv + 127) // 128
    perm = np.random.default_rng(seed).permutation(pages + 5).astype(np.int32)
    bt = torch.from_numpy(perm[:pages].reshape(1, pages).copy()).cuda()
    q = torch.randn(T, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(pages + 5, 128, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(pages + 5, 128, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    qs = torch.tensor([T], dtype=torch.int64, device="cuda")
    kvs = torch.tensor([kv], dtype=torch.int64, device="cuda")
    o1, l1 = npu.fa_fp32_stage1(q, k, v, bt, qs, kvs, T)
    B = 64
    o1m = torch.randn(B, H, 128, device="cuda", generator=g)
    o2m = torch.randn(B, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    l1m = torch.randn(B * H, 1, device="cuda", generator=g).repeat(1, 8).reshape(-1)
    l2m = torch.randn(B * H, device="cuda", generator=g)
    calls = {"fa_fp32_stage1_fast_T64_kv4356_h40_kvh8": lambda: npu.fa_fp32_stage1(q, k, v, bt, qs, kvs, T),
             "lse_merge_b64_h40_d128_out_code1": lambda: npu.lse_merge(o1m, o2m, l1m, l2m, 1)}
    published = {"fa_fp32_stage1_fast_T64_kv4356_h40_kvh8": "133.9-135.6 us (910B2, README.md:315)",
                 "lse_merge_b64_h40_d128_out_code1": "25.4-33.6 us (910B, README.md:317)"}
    res = {}
    for name, fn in calls.items():
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / reps
        res[name] = {"host_wall_us": round(wall * 1e6, 2), "device_us": round(a.elapsed_time(b) / reps * 1e3, 2),
                     "reference_published_host_wall": published[name]}
    return {"method": "run_perf_driver.py:49-60: 10 warm-up calls, then %d eager calls back to back, one "
                      "synchronize, wall / calls" % reps, "per_op": res, "_launches": 2 * (reps + 10)}


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


def reference_c2_inputs(seed=0, device="cpu"):
    """The C2 workload for the reference arm, built without the repo's package
    (no native library of ours is loaded on that arm): the same recipe as
    cascade_kernel.workloads.c2_llama8b -- numpy default_rng(seed) draws the
    64 suffix lengths U[128,1024] and, from a fresh default_rng(seed), the
    random permutation that places the 32 prefix pages then each request's
    suffix pages in the pool; a torch generator seeded with `seed` on `device`
    draws K, V ([pages, 128, 8, 128]) then q ([64, 32, 128]) from N(0,1) in
    fp32, cast to bf16. Returns an object with the fields cpu_baseline reads."""
    import types
    import numpy as np
    import torch
    B, H, KVH, D, bs, prefix = 64, 32, 8, 128, 128, 4096
    suf = np.random.default_rng(seed).integers(128, 1025, size=B).astype(np.int64)
    rng = np.random.default_rng(seed)
    pre_pages = prefix // bs
    suf_pages = [(int(x) + bs - 1) // bs for x in suf]
    n_pages = pre_pages + sum(suf_pages)
    perm = rng.permutation(n_pages).astype(np.int32)
    bt_p = perm[:pre_pages].reshape(1, pre_pages).copy()
    bt_s = np.zeros((B, max(suf_pages)), np.int32)
    c = pre_pages
    for b in range(B):
        bt_s[b, :suf_pages[b]] = perm[c:c + suf_pages[b]]
        c += suf_pages[b]
    gen = torch.Generator(device=device).manual_seed(seed)
    k = torch.randn((n_pages, bs, KVH, D), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((n_pages, bs, KVH, D), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((B, H, D), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    kvb = 2 * KVH * D * 2
    total = (2 * B * H * D + prefix * kvb + B * H * D * 4 + B * H * 8 * 4) + \
        (2 * B * H * D + int(suf.sum()) * kvb + 2 * B * H * D + B * H * 4) + \
        (B * H * D * 4 + 2 * B * H * D + B * H * 8 * 4 + B * H * 4 + 2 * B * H * D)
    w = types.SimpleNamespace(q=q, k_pool=k, v_pool=v, group_sizes=[B], prefix_lens=[prefix], suffix_lens=suf,
                              tables=types.SimpleNamespace(prefix_block_table=torch.from_numpy(bt_p),
                                                           suffix_block_table=torch.from_numpy(bt_s)))
    w.algorithmic_bytes = lambda: {"total": total}
    return w


def run_reference(args, rank, world):
    import torch
    if rank != 0:
        return None
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = reference_c2_inputs(seed=args.seed, device=dev)
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
            "data": "synthetic (seeded N(0,1) q/k/v, random-permutation block tables)",
            "config": {"workload": WORKLOAD},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": c["cores"], "kind": "port",
                             "sample": c["sample"]},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def _jsonable(x):
    """numpy scalars (workload sizes) in the JSON line."""
    if hasattr(x, "item"):
        return x.item()
    raise TypeError(f"not JSON serializable: {type(x).__name__}")


def run_only(args):
    """One block alone: the HBM read-roof probe; stage-1 and the suffix
    decode of C4 / C2 each timed alone (args.steps launches in one graph); the
    whole C4 step (args.steps steps in one graph); or the Llama-3-70B MLP
    gate_up shard at the per-rank width of args.shard_ranks ranks (args.steps
    event-timed calls)."""
    import torch
    from cascade_kernel import workloads
    torch.cuda.set_device(0)
    if args.only == "read_roof":
        return read_roof_block(_peaks(), None)
    if args.only == "gateup_70b_shard":
        I = 28672 // args.shard_ranks
        blk = gateup_sweep(lambda: None, _peaks(), Ms=(256,), K=8192, I=I, reps=args.steps, seed=11)
        return {"block": args.only, "ranks": args.shard_ranks, "I": I, **blk["per_M"]["256"]}
    if args.only == "c4_step":
        from cascade_kernel.cascade import CascadeStepGraph
        w = workloads.c4_llama70b(seed=args.seed)
        g = CascadeStepGraph(w.q, w.k_pool, w.v_pool, w.tables)
        for _ in range(3):
            g.replay()
        return {"block": args.only, "us_per_step": round(_time_graph(g, args.steps, torch.cuda.current_stream()) * 1e3, 2)}
    w = (workloads.c4_llama70b if args.only == "c4_kernels" else workloads.c2_llama8b)(seed=args.seed)
    s1, dec = kernel_times(w, args.steps)
    return {"block": args.only, "stage1_alone_us": round(s1, 2), "suffix_decode_alone_us": round(dec, 2),
            "stage1_tflops": round(w.flops()["stage1"] / (s1 * 1e-6) / 1e12, 1)}


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
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the C4 sharded, C5 ragged, read-roof and host-wall blocks")
    ap.add_argument("--only", choices=["read_roof", "c4_kernels", "c2_kernels", "c4_step", "gateup_70b_shard"],
                    help="run one block alone on cuda:0 and print its JSON (entry points for profiling)")
    ap.add_argument("--shard-ranks", type=int, default=8, choices=[1, 2, 4, 8],
                    help="--only gateup_70b_shard: the per-rank column width of this many ranks")
    args = ap.parse_args()
    if args.only:
        print(json.dumps(run_only(args), default=_jsonable), flush=True)
        return
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line, default=_jsonable), flush=True)
        return
    rank, world, local = setup_dist()
    line = run_ours(args, rank, world, local)
    if rank == 0:
        print(json.dumps(line, default=_jsonable), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
