"""World-size-2 gloo (CPU) test of the multi-GPU partitioning logic: each rank
computes its kv-head shard of a cascade step and its column shard of the
SwiGLU GEMM with the CPU oracle, the shards are all_gathered, and the result
must equal the unsharded oracle exactly (the partition is exact: heads and
output columns are independent)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    from oracle import cascade_oracle as O
    rng = np.random.default_rng(0)
    B, H, KVH, bs = 6, 8, 4, 16
    pre, suf = 70, rng.integers(0, 60, size=B)
    npg = (pre + bs - 1) // bs + sum((int(s) + bs - 1) // bs for s in suf)
    perm = rng.permutation(npg)
    c = (pre + bs - 1) // bs
    bt_p = perm[:c][None].astype(np.int32)
    bt_s = np.zeros((B, 4), np.int32)
    for b in range(B):
        n = (int(suf[b]) + bs - 1) // bs
        bt_s[b, :n] = perm[c:c + n]
        c += n
    q = O.round_bf16(rng.standard_normal((B, H, 128)))
    k = O.round_bf16(rng.standard_normal((npg, bs, KVH, 128)))
    v = O.round_bf16(rng.standard_normal((npg, bs, KVH, 128)))
    x = O.round_bf16(rng.standard_normal((4, 64)))
    w = O.round_bf16(rng.standard_normal((2 * 32, 64)) * 0.02)
    return q, k, v, bt_p, [B], [pre], bt_s, suf, x, w


def _worker(rank, world, port, out_q):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "vllm-hust-cascade-kernel_b200"))
    import torch.distributed as dist
    from oracle import cascade_oracle as O
    from cascade_kernel import sharding as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, bt_p, gs, pl, bt_s, suf, x, w = _case()
        tq, tk, tv = S.shard_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), rank, world)
        o_loc, _ = O.cascade_step_ref(tq.numpy(), tk.numpy(), tv.numpy(), bt_p, gs, pl, bt_s, suf)
        o_all = S.gather_dim(torch.from_numpy(o_loc), 1, world)
        w_loc = S.shard_gateup_weight(torch.from_numpy(w), rank, world)
        d_loc = O.gateup_ref(x, w_loc.numpy(), mode=1)
        d_all = S.gather_dim(torch.from_numpy(d_loc), 1, world)
        if rank == 0:
            ref_o, _ = O.cascade_step_ref(q, k, v, bt_p, gs, pl, bt_s, suf)
            ref_d = O.gateup_ref(x, w, mode=1)
            out_q.put((bool(np.array_equal(o_all.numpy(), ref_o)), bool(np.array_equal(d_all.numpy(), ref_d))))
    finally:
        dist.destroy_process_group()


def test_kv_head_and_column_sharding_exact_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    attn_ok, mlp_ok = q.get(timeout=10)
    assert attn_ok and mlp_ok


def test_shard_index_helpers():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "vllm-hust-cascade-kernel_b200"))
    from cascade_kernel import sharding as S
    assert S.kv_head_range(8, 3, 4) == (6, 8)
    idx = S.gateup_row_index(8, 1, 2)
    assert idx.tolist() == [4, 5, 6, 7, 12, 13, 14, 15]
    with pytest.raises(ValueError):
        S.kv_head_range(8, 0, 3)
