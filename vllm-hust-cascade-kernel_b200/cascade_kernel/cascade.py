"""The two-stage cascade decode step, composed from the registered ops.

Mirrors how the reference's consumer drives the ops (ascend-kernel/README.md:
158-201): stage-1 reads each shared prefix ONCE for all requests of its prefix
group (the group's requests are flattened into one "request" whose q_len is
the group size), stage-2 reads each request's own suffix pages, and the LSE
merge combines the two partials.

Queries must be ordered by prefix group: group g owns query rows
``[sum(group_sizes[:g]), sum(group_sizes[:g+1]))``.
"""
from dataclasses import dataclass

import torch


@dataclass
class CascadeTables:
    """Per-step index tensors (all on the device).

    prefix_block_table  int32 [G, cols_p]   pages of each group's shared prefix
    prefix_q_seqlens    int64 [G]           requests per group
    prefix_kv_seqlens   int64 [G]           prefix length of each group
    suffix_block_table  int32 [B, cols_s]   pages of each request's own suffix
    suffix_q_seqlens    int64 [B]           ones
    suffix_kv_seqlens   int64 [B]           suffix length of each request (may be 0)
    uniform_group       int                 group size if all groups are equal, else 0
    """
    prefix_block_table: torch.Tensor
    prefix_q_seqlens: torch.Tensor
    prefix_kv_seqlens: torch.Tensor
    suffix_block_table: torch.Tensor
    suffix_q_seqlens: torch.Tensor
    suffix_kv_seqlens: torch.Tensor
    uniform_group: int = 0


def cascade_decode(q, k_pool, v_pool, tables: CascadeTables, out_dtype=None, fused=True):
    """One cascade decode step for one layer.

    q [B, H, 128] (bf16 or fp16), k_pool/v_pool [numBlocks, bs, KVH, 128].
    Returns the merged attention output [B, H, 128] in ``out_dtype``
    (default: the query dtype).

    fused=True (default): ``npu.cascade_decode_step`` -- stage-1 and suffix
    kernels write split partials and one combine kernel writes the output.
    fused=False: the reference consumer's chain of three ops; bf16 + block
    size 128 uses exactly the reference ops (fa_fp32_stage1 / lse_merge
    out_code=1), other inputs the extended-domain siblings."""
    out_dtype = q.dtype if out_dtype is None else out_dtype
    code = {torch.bfloat16: 1, torch.float32: 2, torch.float16: 3}[out_dtype]
    if fused:
        return torch.ops.npu.cascade_decode_step(
            q, k_pool, v_pool, tables.prefix_block_table, tables.prefix_q_seqlens, tables.prefix_kv_seqlens,
            tables.suffix_block_table, tables.suffix_q_seqlens, tables.suffix_kv_seqlens, tables.uniform_group,
            code)
    reference_domain = (q.dtype == torch.bfloat16 and k_pool.shape[1] == 128
                        and out_dtype == torch.bfloat16)
    npu = torch.ops.npu
    prefix = npu.fa_fp32_stage1 if reference_domain else npu.cascade_prefix_attention
    o1, l1 = prefix(q, k_pool, v_pool, tables.prefix_block_table, tables.prefix_q_seqlens,
                    tables.prefix_kv_seqlens, tables.uniform_group)
    o2, l2 = npu.cascade_suffix_decode(q, k_pool, v_pool, tables.suffix_block_table,
                                       tables.suffix_q_seqlens, tables.suffix_kv_seqlens, 1)
    if reference_domain:
        return npu.lse_merge(o1, o2, l1, l2, code)
    return npu.cascade_lse_merge(o1, o2, l1, l2, code)


def copy_groups(buffers, io_group):
    """Groups of consecutive steps whose host copies share one event in
    ``CascadeLayersGraph(overlap_io=True)``; ``buffers[i]`` identifies step
    i's device input buffer. Groups hold distinct buffers, are sized 1, 2,
    then up to ``io_group`` steps -- but at most half the distinct buffers,
    so a group's copies can run while the previous group computes -- and the
    last step is a group of its own: the first kernel waits for one step's
    inputs and one step's output drains after the last kernel, as with
    per-step copies."""
    limit = max(1, min(io_group, len(set(buffers)) // 2))
    groups, cur, seen = [], [], set()
    for i, key in enumerate(buffers):
        if len(cur) >= min(limit, 1 << len(groups)) or key in seen:
            groups.append(cur)
            cur, seen = [], set()
        cur.append(i)
        seen.add(key)
    if cur:
        groups.append(cur)
    if groups and len(groups[-1]) > 1:
        groups.append([groups[-1].pop()])
    return groups


class CascadeLayersGraph:
    """Several cascade decode steps captured back to back in ONE CUDA graph,
    as a decode forward runs attention layer after layer: step i reads its
    own query and K/V pools ``steps[i] = (q, k_pool, v_pool, tables)``.

    ``replay()`` re-issues every step's suffix, stage-1 and combine kernels
    with no host work and returns the list of step outputs (fixed device
    tensors, overwritten by every replay). A serving loop writes the next
    step's queries and index tensors into the captured buffers in place.
    Requires the uniform-q path (``tables.uniform_group > 0``): the
    per-request path reads seqlens back to the host and cannot be captured.

    ``host_io`` (optional, one ``(host_in, dev_in, host_out)`` triple per
    step) puts each step's host traffic in the graph: before step i the
    pinned host buffer ``host_in`` is copied into the device buffer
    ``dev_in`` (which must back that step's q and tables), and after it the
    step's output is copied into the pinned host tensor ``host_out``.

    ``overlap_io=True`` issues those copies on two copy streams inside the
    graph instead of in line with the kernels, in groups of consecutive
    steps whose ``dev_in`` buffers differ (1, 2, then up to ``io_group``
    steps but at most half the number of distinct ``dev_in`` buffers, the
    last step alone, so filling and draining the copy pipeline costs one
    step's copies as without grouping): a group's host->device
    copies wait only for the last earlier steps that
    read the same ``dev_in`` buffers (so they run while earlier steps
    compute) and complete behind one event that the group's first kernel
    waits for; the group's device->host copies wait for its last step. Every
    step still moves its own inputs in and its own output out. Grouping
    matters because each wait of the kernel stream on a copy-engine event is
    an edge into the graph's critical path (measured: ~3 us per step with
    ``io_group=1`` on the C2 step).
    """

    def __init__(self, steps, out_dtype=None, warmup=2, host_io=None, overlap_io=False, io_group=4):
        steps = list(steps)
        if not steps:
            raise ValueError("CascadeLayersGraph needs at least one step")
        for st in steps:
            if st[3].uniform_group <= 0:
                raise ValueError("CascadeLayersGraph needs uniform prefix groups (tables.uniform_group > 0)")
        if host_io is not None and len(host_io) != len(steps):
            raise ValueError("host_io needs one (host_in, dev_in, host_out) triple per step")
        if io_group < 1:
            raise ValueError("io_group must be >= 1")
        self.steps, self.out_dtype, self.host_io = steps, out_dtype, host_io
        io_streams = (torch.cuda.Stream(), torch.cuda.Stream()) if host_io is not None and overlap_io else None

        def run_overlapped():
            main = torch.cuda.current_stream()
            s_in, s_out = io_streams
            s_in.wait_stream(main)
            s_out.wait_stream(main)
            groups = copy_groups([io[1].data_ptr() for io in host_io], io_group)
            outs, fin_of, last_use = [None] * len(steps), {}, {}
            for grp in groups:
                with torch.cuda.stream(s_in):
                    waited = set()
                    for i in grp:
                        host_in, dev_in, _ = host_io[i]
                        j = last_use.get(dev_in.data_ptr())
                        if j is not None and id(fin_of[j]) not in waited:
                            s_in.wait_event(fin_of[j])
                            waited.add(id(fin_of[j]))
                        dev_in.copy_(host_in, non_blocking=True)
                    loaded = torch.cuda.Event()
                    loaded.record(s_in)
                main.wait_event(loaded)
                for i in grp:
                    q, k_pool, v_pool, tables = steps[i]
                    outs[i] = cascade_decode(q, k_pool, v_pool, tables, out_dtype)
                fin = torch.cuda.Event()
                fin.record(main)
                for i in grp:
                    fin_of[i] = fin
                    last_use[host_io[i][1].data_ptr()] = i
                with torch.cuda.stream(s_out):
                    s_out.wait_event(fin)
                    for i in grp:
                        host_io[i][2].copy_(outs[i], non_blocking=True)
            main.wait_stream(s_in)
            main.wait_stream(s_out)
            return outs

        def run():
            if io_streams is not None:
                return run_overlapped()
            outs = []
            for i, (q, k_pool, v_pool, tables) in enumerate(steps):
                io = None if host_io is None else host_io[i]
                if io is not None:
                    io[1].copy_(io[0], non_blocking=True)
                out = cascade_decode(q, k_pool, v_pool, tables, out_dtype)
                if io is not None:
                    io[2].copy_(out, non_blocking=True)
                outs.append(out)
            return outs

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                run()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outs = run()

    def replay(self):
        self.graph.replay()
        return self.outs


class CascadeStepGraph(CascadeLayersGraph):
    """One cascade decode step captured in a CUDA graph and replayed (a
    one-step ``CascadeLayersGraph``).

    The step's inputs live in fixed device buffers (``q``, the pools and the
    ``tables`` given at construction); ``replay()`` returns the output.
    ``host_io=(host_in, dev_in, host_out)`` puts the step's host traffic in
    the same graph: every replay first copies the pinned host buffer
    ``host_in`` into the device buffer ``dev_in`` (which must back ``q`` and
    the tables), and after the step copies the output into the pinned host
    tensor ``host_out``.
    """

    def __init__(self, q, k_pool, v_pool, tables: CascadeTables, out_dtype=None, warmup=2, host_io=None):
        if tables.uniform_group <= 0:
            raise ValueError("CascadeStepGraph needs uniform prefix groups (tables.uniform_group > 0)")
        self.q, self.k_pool, self.v_pool, self.tables = q, k_pool, v_pool, tables
        super().__init__([(q, k_pool, v_pool, tables)], out_dtype, warmup,
                         None if host_io is None else [host_io])
        self.out = self.outs[0]

    def replay(self):
        self.graph.replay()
        return self.out
