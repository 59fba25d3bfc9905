"""Shared helpers for the GPU parity tests (device tensors <-> oracle arrays,
C-ABI call wrappers)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import cascade_oracle as O


def need_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def capi():
    from cascade_kernel import capi as C
    C.load()
    return C


def ops():
    import cascade_kernel  # noqa: F401  registers torch.ops.npu.*
    import torch
    return torch.ops.npu


def bits_to_dev(bits, dtype="bf16"):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == "bf16" else torch.float16).cuda()


def dev_to_f64(t):
    import torch
    return t.detach().float().cpu().numpy().astype(np.float64)


def load_fixture(name):
    z = np.load(os.path.join(GOLDEN, f"stage1_{name}.npz"))
    return z


def fixture_device_args(z):
    import torch
    q = bits_to_dev(z["q_bits"])
    k = bits_to_dev(z["k_bits"])
    v = bits_to_dev(z["v_bits"])
    bt = torch.from_numpy(z["block_table"]).cuda()
    qs = torch.from_numpy(z["q_seqlens"]).cuda()
    kvs = torch.from_numpy(z["kv_seqlens"]).cuda()
    return q, k, v, bt, qs, kvs


def fixture_host_args(z):
    return (O.bf16_bits_to_f64(z["q_bits"]), O.bf16_bits_to_f64(z["k_bits"]),
            O.bf16_bits_to_f64(z["v_bits"]), z["block_table"], z["q_seqlens"], z["kv_seqlens"])


def run_capi_paged(q, k, v, bt, qs, kvs, q_seqlen_value, suffix=False):
    """Call cascade_fa_fp32_stage1 / cascade_suffix_decode through the C ABI."""
    import torch
    C = capi()
    desc = C.paged_desc(q, k, v, bt, qs, kvs, q_seqlen_value)
    T, H, D = q.shape
    if suffix:
        out = torch.empty((T, H, D), dtype=q.dtype, device=q.device)
        lse = torch.empty((T * H,), dtype=torch.float32, device=q.device)
        n = C.suffix_workspace_size(desc)
    else:
        out = torch.empty((T, H, D), dtype=torch.float32, device=q.device)
        lse = torch.empty((T * H * 8,), dtype=torch.float32, device=q.device)
        n = C.stage1_workspace_size(desc)
    ws = torch.empty((max(n, 1),), dtype=torch.uint8, device=q.device) if n else None
    if suffix:
        C.suffix_decode(desc, out, lse, ws)
    else:
        C.fa_fp32_stage1(desc, out, lse, ws)
    torch.cuda.synchronize()
    assert C.device_error() == 0
    return out, lse


def kernel_structure(q_len, group, kv_cap_tokens, T, H, KVH, batch, block_cols, block_size, suffix=False):
    """(kernel id, oracle kwargs reproducing that kernel's quantisation structure)."""
    C = capi()
    desc = C.paged_desc(None, None, None, None, None, None, q_len,
                        shape=dict(num_tokens=T, num_heads=H, head_dim=128, num_blocks=1,
                                   block_size=block_size, kv_heads=KVH, batch=batch,
                                   block_cols=block_cols))
    desc.q_seqlen_value = 0
    p = C.plan(desc, q_len, suffix)
    if p.kernel in (0, 2):  # decode, one CTA per item or planned
        split = int(p.split_tokens)
        return 0, dict(segments=lambda kv: O.decode_segments(kv, split=split, tile=64, warps=4))
    return 1, dict(chunk=128, split=int(p.split_tokens))


def stage1_pieces(q_len, group, KVH, batch, cap_tokens, sms=148, min_run=8):
    """The equal-run schedule of the two-tile stage-1 (pp_pieces in capi.cu):
    None when the split grid is used, else a function (b, g, mp) -> list of
    (first tile, end tile) pieces of that unit, in 128-token KV tiles. Runs
    cut the concatenated (request, kv head) streams; every row-tile pair of a
    stream has the same pieces."""
    rows = q_len * group
    if q_len <= 0 or rows <= 128:
        return None
    pairs = -(-rows // 256)
    streams = KVH * batch
    tc = -(-max(1, cap_tokens) // 128)
    T = streams * tc
    G = min(sms // pairs, T)
    if G <= streams or T < G * min_run:
        return None
    starts = sorted(set([r * T // G for r in range(G)] + [T]))

    def pieces(b, g, mp):
        u = b * KVH + g
        lo, hi = u * tc, (u + 1) * tc
        cuts = [lo] + [x for x in starts if lo < x < hi] + [hi]
        return [(a - lo, e - lo) for a, e in zip(cuts[:-1], cuts[1:])]
    return pieces


def stage1_pieces_oracle(qf, kf, vf, bt, qs, kvs, group, pieces):
    """Kernel-structured fp64 stage-1 of the equal-run schedule: each (request,
    kv head, row-tile pair) unit runs the reference recurrence (128-token
    chunks) separately over each of its pieces, the pieces merged in LSE space
    -- paged_attention_ref per unit with that unit's segments. Returns (O,
    LSE, tie-band bound A)."""
    T, H, D = qf.shape
    KVH = H // group
    O_ = np.zeros((T, H, D))
    L_ = np.full((T, H), -np.inf)
    A_ = np.zeros((T, H, D))
    tok = 0
    for b in range(len(qs)):
        ql, kv = int(qs[b]), int(kvs[b])
        tok_per_pair = 256 // group
        for g in range(KVH):
            for mp in range(-(-ql * group // 256)):
                t0, t1 = tok + mp * tok_per_pair, tok + min(ql, (mp + 1) * tok_per_pair)
                segs = [[np.arange(t * 128, min((t + 1) * 128, kv)) for t in range(a, e) if t * 128 < kv]
                        for a, e in pieces(b, g, mp)]
                segs = [s for s in segs if s]
                hs = slice(g * group, (g + 1) * group)
                o, l, a = O.paged_attention_ref(qf[t0:t1, hs], kf[:, :, g:g + 1], vf[:, :, g:g + 1], bt[b:b + 1],
                                                np.array([t1 - t0]), np.array([kv]), segments=lambda _kv: segs,
                                                with_tieband=True, tieband_rule="rescaled")
                O_[t0:t1, hs], L_[t0:t1, hs], A_[t0:t1, hs] = o, l, a
        tok += ql
    return O_, L_, A_


def norm_inputs(m, k, dtype, seed, has_beta):
    """The seeded inputs of add_rms_norm_stats_cases.make_inputs
    (add_rms_norm_stats/test/add_rms_norm_stats_cases.py:33-43), drawn on the
    CPU in the same order: x1, x2 ~ 0.5 N(0,1); gamma ~ 1 + 0.1 N(0,1);
    beta ~ 0.05 N(0,1). Returns CPU tensors of ``dtype`` (beta None unless
    has_beta)."""
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    x1 = (torch.randn(m, k, generator=g, dtype=torch.float32) * 0.5).to(dtype)
    x2 = (torch.randn(m, k, generator=g, dtype=torch.float32) * 0.5).to(dtype)
    gamma = (1.0 + torch.randn(k, generator=g, dtype=torch.float32) * 0.1).to(dtype)
    beta = (torch.randn(k, generator=g, dtype=torch.float32) * 0.05).to(dtype) if has_beta else None
    return x1, x2, gamma, beta


def bits_to_f64(bits, dtype):
    """uint16 bit patterns of bf16 / fp16 values -> fp64."""
    if dtype == "bf16":
        return O.bf16_bits_to_f64(bits)
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float64)


def _step_oracle_head(item):
    """Process-pool worker: the fp64 cascade step of one kv head, from the
    per-head .npy files written by step_oracle_all_heads."""
    d, g, meta = item
    ld = lambda n: np.load(os.path.join(d, n))
    dt = meta["p_dtype"]
    conv = (lambda b: O.bf16_bits_to_f64(b)) if dt == "bf16" else \
        (lambda b: np.asarray(b, np.uint16).view(np.float16).astype(np.float64))
    q = conv(ld(f"q{g}.npy"))
    k = conv(ld(f"k{g}.npy"))[:, :, None, :]
    v = conv(ld(f"v{g}.npy"))[:, :, None, :]
    out, lse = O.cascade_step_ref(q, k, v, ld("bt_p.npy"), meta["group_sizes"], meta["prefix_lens"],
                                  ld("bt_s.npy"), ld("suf.npy"), p_dtype=dt, out_dtype=meta["out_dtype"],
                                  round_suffix=meta["round_suffix"])
    return g, out, lse


def step_oracle_all_heads(w, out_dtype="fp32", round_suffix=False):
    """The CPU oracle of a whole cascade step (oracle.cascade_step_ref) on
    EVERY kv head of workload ``w``, one spawned worker per kv head; each
    worker reads only its head's slice of q and of the pools from a temporary
    directory. Returns (out [B, H, D], lse [B, H])."""
    import multiprocessing as mp
    import shutil
    import tempfile
    import torch
    H, KVH = w.q.shape[1], w.k_pool.shape[2]
    grp = H // KVH
    p_dtype = "fp16" if w.q.dtype == torch.float16 else "bf16"
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    d = tempfile.mkdtemp(prefix="cascade_oracle_")
    try:
        for g in range(KVH):
            np.save(os.path.join(d, f"q{g}.npy"), bits(w.q[:, g * grp:(g + 1) * grp]))
            np.save(os.path.join(d, f"k{g}.npy"), bits(w.k_pool[:, :, g]))
            np.save(os.path.join(d, f"v{g}.npy"), bits(w.v_pool[:, :, g]))
        np.save(os.path.join(d, "bt_p.npy"), w.tables.prefix_block_table.cpu().numpy())
        np.save(os.path.join(d, "bt_s.npy"), w.tables.suffix_block_table.cpu().numpy())
        np.save(os.path.join(d, "suf.npy"), np.asarray(w.suffix_lens))
        meta = dict(p_dtype=p_dtype, out_dtype=out_dtype, round_suffix=round_suffix,
                    group_sizes=[int(x) for x in w.group_sizes], prefix_lens=[int(x) for x in w.prefix_lens])
        workers = max(1, min(KVH, os.cpu_count() or 1))
        with mp.get_context("spawn").Pool(workers) as pool:
            res = pool.map(_step_oracle_head, [(d, g, meta) for g in range(KVH)], chunksize=1)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    B = w.q.shape[0]
    out = np.zeros((B, H, w.q.shape[2]))
    lse = np.zeros((B, H))
    for g, o, l in res:
        out[:, g * grp:(g + 1) * grp] = o
        lse[:, g * grp:(g + 1) * grp] = l
    return out, lse
