"""Multi-GPU partitioning of the cascade path (one process per GPU).

Attention is partitioned by kv head: rank r of G owns kv heads
[r*KVH/G, (r+1)*KVH/G) and the q heads of those GQA groups, so stage-1, the
suffix and the merge are all rank-local (no collective on the hot path).
gate_up is partitioned by output column: rank r owns gate rows
[r*I/G, (r+1)*I/G) and the SAME up rows [I + r*I/G, ...), so SwiGLU stays
local.  The collectives here (all_gather) only reassemble full outputs for
verification against the single-device / CPU oracle.
"""
import torch


def kv_head_range(kv_heads, rank, world):
    if kv_heads % world:
        raise ValueError(f"kv_heads={kv_heads} not divisible by world size {world}")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def shard_attention(q, k_pool, v_pool, rank, world):
    """q [B,H,D], pools [NB,bs,KVH,D] -> this rank's contiguous head shards.
    The block tables are replicated (pages are shared by all heads)."""
    kvh = k_pool.shape[2]
    group = q.shape[1] // kvh
    g0, g1 = kv_head_range(kvh, rank, world)
    return (q[:, g0 * group:g1 * group].contiguous(), k_pool[:, :, g0:g1].contiguous(),
            v_pool[:, :, g0:g1].contiguous())


def gateup_row_index(I, rank, world):
    """Rows of W [2I, K] owned by this rank: its gate slice then its up slice."""
    if I % world:
        raise ValueError(f"I={I} not divisible by world size {world}")
    per = I // world
    gate = torch.arange(rank * per, (rank + 1) * per)
    return torch.cat([gate, gate + I])


def shard_gateup_weight(w, rank, world):
    I = w.shape[0] // 2
    return w.index_select(0, gateup_row_index(I, rank, world).to(w.device)).contiguous()


def gather_dim(x_local, dim, world, group=None):
    """all_gather the rank shards of x along ``dim`` (verification only)."""
    import torch.distributed as dist
    xs = x_local.movedim(dim, 0).contiguous()
    out = torch.empty((world * xs.shape[0],) + tuple(xs.shape[1:]), dtype=xs.dtype, device=xs.device)
    dist.all_gather_into_tensor(out, xs, group=group)
    return out.movedim(0, dim).contiguous()
