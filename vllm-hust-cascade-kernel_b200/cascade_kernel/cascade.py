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


class CascadeStepGraph:
    """A cascade decode step captured once in a CUDA graph and replayed.

    The step's inputs live in fixed device buffers (``q``, the pools and the
    ``tables`` given at construction); a serving loop writes the next step's
    queries and index tensors into them in place and calls ``replay()``,
    which re-issues the suffix, stage-1 and combine kernels without any host
    work. Requires the uniform-q path (``tables.uniform_group > 0``): the
    per-request path reads seqlens back to the host and cannot be captured.

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
        self.out_dtype = out_dtype
        self.host_io = host_io

        def step():
            if host_io is not None:
                host_io[1].copy_(host_io[0], non_blocking=True)
            out = cascade_decode(q, k_pool, v_pool, tables, out_dtype)
            if host_io is not None:
                host_io[2].copy_(out, non_blocking=True)
            return out

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                step()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step()

    def replay(self):
        self.graph.replay()
        return self.out
