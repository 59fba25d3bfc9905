"""GPU parity of the whole cascade decode step: the fused single-combine op
(npu.cascade_decode_step / C ABI cascade_decode_step) and the reference
consumer's three-op chain, against the CPU oracle of the composed step
(oracle.cascade_step_ref) and against each other at the benchmark shape."""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu


def _work(name, **kw):
    from cascade_kernel import workloads
    return workloads.make_cascade(name, device="cuda", **kw)


CASES = {
    # C1-like: 4 requests share a 512-token prefix, fp16, H=8/KVH=2
    "c1_like": dict(group_sizes=[4], prefix_lens=[512], suffix_lens=[64, 100, 200, 256], H=8, KVH=2, bs=128,
                    dtype="fp16", seed=1),
    # C2-like at reduced batch (the oracle must finish in seconds): bf16, 32/8 heads
    "c2_like_b16": dict(group_sizes=[16], prefix_lens=[1024], suffix_lens=list(range(128, 1024, 56)), H=32,
                        KVH=8, bs=128, dtype="bf16", seed=2),
    # ragged: several prefix groups, block size 16, zero-length suffixes, GQA 5
    "ragged_bs16": dict(group_sizes=[3, 3, 3], prefix_lens=[16, 300, 777], suffix_lens=[0, 5, 200, 0, 31, 64, 1, 0, 90],
                        H=10, KVH=2, bs=16, dtype="fp16", seed=3),
    # many rows per kv head: 40 requests x group 5 -> 200 rows (two 128-row tiles)
    "wide_group": dict(group_sizes=[40], prefix_lens=[640], suffix_lens=[7] * 40, H=10, KVH=2, bs=64,
                       dtype="bf16", seed=4),
}


def _oracle(w, round_suffix, out_dtype):
    f64 = lambda x: x.float().cpu().numpy().astype(np.float64)
    p_dtype = "bf16" if str(w.q.dtype) == "torch.bfloat16" else "fp16"
    return O.cascade_step_ref(f64(w.q), f64(w.k_pool), f64(w.v_pool), w.tables.prefix_block_table.cpu().numpy(),
                              w.group_sizes, w.prefix_lens, w.tables.suffix_block_table.cpu().numpy(),
                              w.suffix_lens, p_dtype=p_dtype, out_dtype=out_dtype, round_suffix=round_suffix)


@pytest.mark.parametrize("name", list(CASES))
def test_fused_step_and_chain_vs_oracle(name):
    import torch
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    kw = dict(CASES[name])
    kw["dtype"] = torch.float16 if kw["dtype"] == "fp16" else torch.bfloat16
    w = _work(name, **kw)
    dt = "fp16" if kw["dtype"] == torch.float16 else "bf16"
    fused = cascade_decode(w.q, w.k_pool, w.v_pool, w.tables, fused=True)
    chain = cascade_decode(w.q, w.k_pool, w.v_pool, w.tables, fused=False)
    torch.cuda.synchronize()
    assert Hh.capi().device_error() == 0
    ref_f, _ = _oracle(w, round_suffix=False, out_dtype="fp32")
    ref_c, _ = _oracle(w, round_suffix=True, out_dtype="fp32")
    got_f, got_c = Hh.dev_to_f64(fused), Hh.dev_to_f64(chain)
    assert np.isfinite(got_f).all() and np.isfinite(got_c).all()
    # BASELINE bar
    np.testing.assert_allclose(got_f, ref_f, atol=2e-2, rtol=2e-2)
    np.testing.assert_allclose(got_c, ref_c, atol=2e-2, rtol=2e-2)
    # tighter: one output ulp plus the P-rounding structure difference of the
    # attention kernels against the 512-chunk golden structure
    for got, ref in ((got_f, ref_f), (got_c, ref_c)):
        err = np.abs(got - ref)
        assert (err <= O.ulp(ref, dt) + 2e-3).all(), float((err - O.ulp(ref, dt)).max())


def _combine_case(form):
    """Step shapes of 2,560 (token, head) rows -- more than one wave of the
    two-blocks-per-SM combine grid -- whose plans (stage-1 planes n1, suffix
    splits n2) select each of the step combine's other forms: n1 + n2 = 3
    (4-deep dense), 6 (8-deep dense) and 16 (sparse: one 6,000-token suffix
    makes 12 splits that most rows leave empty; some suffixes are empty)."""
    rng = np.random.default_rng(11)
    if form == "dense4":
        return dict(group_sizes=[80], prefix_lens=[256], suffix_lens=list(rng.integers(1, 400, 80)), H=32, KVH=8,
                    bs=64, dtype="bf16", seed=5), 3
    if form == "dense8":
        return dict(group_sizes=[40, 40], prefix_lens=[1024, 600], suffix_lens=list(rng.integers(1, 2000, 80)),
                    H=32, KVH=8, bs=64, dtype="bf16", seed=6), 6
    suf = list(rng.integers(0, 300, 80))
    suf[7] = 6000
    return dict(group_sizes=[20] * 4, prefix_lens=[100, 2000, 37, 640], suffix_lens=suf, H=32, KVH=8, bs=16,
                dtype="fp16", seed=7), 16


@pytest.mark.parametrize("form", ["dense4", "dense8", "sparse"])
def test_step_combine_forms_vs_oracle(form):
    import torch
    from cascade_kernel import capi
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    kw, n_planes = _combine_case(form)
    dt = kw["dtype"]
    kw["dtype"] = torch.float16 if dt == "fp16" else torch.bfloat16
    w = _work(form, **kw)
    t = w.tables
    # the planes the step merges: stage-1's plan (prefix-first: at most 32
    # CTAs over the (kv head, row-tile pair) units) and the suffix splits
    dp = capi.paged_desc(w.q, w.k_pool, w.v_pool, t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens,
                         t.uniform_group)
    ds = capi.paged_desc(w.q, w.k_pool, w.v_pool, t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1)
    pa, pb = capi.plan(dp, t.uniform_group, False), capi.plan(ds, 1, True)
    cdiv = lambda a, b: -(-a // b)
    rows_pf = t.uniform_group * (kw["H"] // kw["KVH"])
    units = kw["KVH"] * len(kw["group_sizes"]) * cdiv(rows_pf, 256 if rows_pf > 128 else 128)
    n1 = pa.num_splits
    if pa.kernel == 1 and units <= 24:
        cap = dp.block_cols * dp.block_size
        split_tokens = cdiv(cdiv(cap, min(cdiv(32, units), cdiv(cap, 128))), 128) * 128
        n1 = cdiv(cap, split_tokens)
    assert w.q.shape[0] * w.q.shape[1] == 2560 and n1 + pb.num_splits == n_planes
    got = cascade_decode(w.q, w.k_pool, w.v_pool, w.tables, fused=True)
    torch.cuda.synchronize()
    assert Hh.capi().device_error() == 0
    ref, _ = _oracle(w, round_suffix=False, out_dtype="fp32")
    got = Hh.dev_to_f64(got)
    assert np.isfinite(got).all()
    err = np.abs(got - ref)
    assert (err <= O.ulp(ref, dt) + 2e-3).all(), float((err - O.ulp(ref, dt)).max())


def test_fused_equals_chain_at_benchmark_shape():
    """C2 (B=64, prefix 4096, suffix U[128,1024], 32/8 heads): the fused step and
    the three-op chain differ by the chain's rounding of the suffix partial to
    bf16 before the merge and by their stage-1 splits (the fused step's
    prefix-first schedule runs stage-1 with fewer, longer splits than the
    standalone op, which moves where P is rounded against the running max):
    within one bf16 ulp plus the P-rounding structure slack of the other
    structure tests (2e-3)."""
    import torch
    from cascade_kernel import workloads
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    w = workloads.c2_llama8b(seed=0)
    t = w.tables
    fused = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=True)
    chain = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=False)
    o2, _ = torch.ops.npu.cascade_suffix_decode(w.q, w.k_pool, w.v_pool, t.suffix_block_table,
                                                t.suffix_q_seqlens, t.suffix_kv_seqlens, 1)
    torch.cuda.synchronize()
    a, b = Hh.dev_to_f64(fused), Hh.dev_to_f64(chain)
    # each side rounds once to bf16 (<= 1 ulp apart) and the chain also rounds
    # the suffix partial (weight <= 1) before merging (<= half an ulp of o2)
    bound = O.ulp(np.maximum(np.abs(a), np.abs(b)), "bf16") + 0.5 * O.ulp(Hh.dev_to_f64(o2), "bf16") + 2e-3
    excess = np.abs(a - b) - bound
    assert (excess <= 0).all(), float(excess.max())


def test_decode_step_capi_and_partials_only_flag():
    import torch
    from cascade_kernel import workloads
    Hh.need_cuda()
    C = Hh.capi()
    npu = Hh.ops()
    w = workloads.c1_cpu_golden(seed=3)
    t = w.tables
    dp = C.paged_desc(w.q, w.k_pool, w.v_pool, t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens,
                      t.uniform_group)
    ds = C.paged_desc(w.q, w.k_pool, w.v_pool, t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1)
    n = C.decode_step_workspace_size(dp, ds)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(w.q)
    lse = torch.empty(w.q.shape[0] * w.q.shape[1], dtype=torch.float32, device="cuda")
    C.decode_step(dp, ds, out, lse, ws)
    ref = npu.cascade_decode_step(w.q, w.k_pool, w.v_pool, t.prefix_block_table, t.prefix_q_seqlens,
                                  t.prefix_kv_seqlens, t.suffix_block_table, t.suffix_q_seqlens,
                                  t.suffix_kv_seqlens, t.uniform_group, 3)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    _, l_ref = _oracle(w, round_suffix=False, out_dtype="fp16")
    assert np.abs(Hh.dev_to_f64(lse).reshape(l_ref.shape) - l_ref).max() < 1e-3
    # partials-only: the suffix kernel alone, no combine, out untouched
    dpo = C.paged_desc(w.q, w.k_pool, w.v_pool, t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1,
                       flags=C.FLAG_PARTIALS_ONLY)
    m = C.suffix_workspace_size(dpo)
    assert m > 0
    ws2 = torch.empty(m, dtype=torch.uint8, device="cuda")
    o2 = torch.full_like(w.q, 5.0)
    l2 = torch.empty_like(lse)
    C.suffix_decode(dpo, o2, l2, ws2)
    torch.cuda.synchronize()
    assert torch.all(o2 == 5.0)


def test_step_graph_replay_with_host_io():
    """CascadeStepGraph replays the step bit-identically to the eager op, and
    with host_io its replay also moves fresh host inputs in and the output
    out: changing the pinned host query between replays changes the result
    exactly as the eager step on the new query does."""
    import torch
    from cascade_kernel.cascade import CascadeStepGraph, CascadeTables, cascade_decode
    Hh.need_cuda()
    kw = dict(CASES["c2_like_b16"])
    kw["dtype"] = torch.bfloat16
    w = _work("graph_io", **kw)
    t = w.tables
    parts = [w.q, t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens, t.suffix_block_table,
             t.suffix_q_seqlens, t.suffix_kv_seqlens]
    offs, cur = [], 0
    for x in parts:
        offs.append(cur)
        cur += (x.numel() * x.element_size() + 255) // 256 * 256
    host_in = torch.zeros(cur, dtype=torch.uint8).pin_memory()
    def put(i, x):
        nb = x.numel() * x.element_size()
        host_in[offs[i]:offs[i] + nb].copy_(x.contiguous().view(-1).view(torch.uint8).cpu())
    for i, x in enumerate(parts):
        put(i, x)
    dev_in = torch.empty(cur, dtype=torch.uint8, device="cuda")
    views = [dev_in[o:o + x.numel() * x.element_size()].view(x.dtype).view(x.shape) for x, o in zip(parts, offs)]
    dev_in.copy_(host_in)
    tt = CascadeTables(*views[1:], uniform_group=t.uniform_group)
    out_h = torch.empty(w.q.shape, dtype=w.q.dtype).pin_memory()
    plain = CascadeStepGraph(views[0], w.k_pool, w.v_pool, tt)
    io = CascadeStepGraph(views[0], w.k_pool, w.v_pool, tt, host_io=(host_in, dev_in, out_h))
    eager = cascade_decode(w.q, w.k_pool, w.v_pool, t)
    assert torch.equal(plain.replay(), eager)
    for step in range(2):
        q_new = (torch.randn(w.q.shape, device="cuda") * (1.0 + step)).to(w.q.dtype)
        put(0, q_new)
        io.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_h, cascade_decode(q_new, w.k_pool, w.v_pool, t).cpu())


def test_vllm_kv_cache_layout_views():
    """vLLM keeps K and V in one tensor [2, numBlocks, blockSize, KVH, D]; its
    kv_cache[0] / kv_cache[1] are contiguous [numBlocks, blockSize, KVH, D]
    views, which the ops take as the K and V pools without a copy."""
    import torch
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    kw = dict(CASES["c2_like_b16"])
    kw["dtype"] = torch.bfloat16
    w = _work("vllm_layout", **kw)
    kv_cache = torch.stack([w.k_pool, w.v_pool])           # [2, NB, bs, KVH, D]
    k_view, v_view = kv_cache[0], kv_cache[1]
    assert k_view.is_contiguous() and v_view.is_contiguous()
    assert k_view.data_ptr() == kv_cache.data_ptr()        # a view, no copy
    a = cascade_decode(w.q, w.k_pool, w.v_pool, w.tables)
    b = cascade_decode(w.q, k_view, v_view, w.tables)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_layers_graph_steps_and_host_io():
    """CascadeLayersGraph: several steps, each on its own layer's q/K/V, in
    one graph. Every step's output equals the eager step on that layer, and
    with per-step host_io each step's pinned host output is its own result."""
    import torch
    from cascade_kernel.cascade import CascadeLayersGraph, CascadeTables, cascade_decode
    Hh.need_cuda()
    kw = dict(CASES["c1_like"])
    kw["dtype"] = torch.float16
    kw["group_sizes"], kw["suffix_lens"] = [4, 4], [64, 100, 200, 256, 0, 17, 128, 300]
    kw["prefix_lens"] = [512, 384]
    w = _work("layers", **kw)
    t = w.tables
    gen = torch.Generator(device="cuda").manual_seed(5)
    layers = [(w.q, w.k_pool, w.v_pool)] + [
        tuple(torch.randn(x.shape, device="cuda", generator=gen).to(x.dtype) for x in (w.q, w.k_pool, w.v_pool))
        for _ in range(2)]
    order = [0, 1, 2, 1]
    g = CascadeLayersGraph([layers[l] + (t,) for l in order])
    outs = g.replay()
    torch.cuda.synchronize()
    assert len(outs) == len(order)
    for o, l in zip(outs, order):
        assert torch.equal(o, cascade_decode(*layers[l], t))
    # per-step host io: the query of each step comes from its own pinned buffer
    ios, steps = [], []
    for l in order:
        q = layers[l][0]
        host_in = torch.empty(q.numel() * q.element_size(), dtype=torch.uint8).pin_memory()
        host_in.copy_(q.contiguous().view(-1).view(torch.uint8).cpu())
        dev_in = torch.empty_like(host_in, device="cuda")
        qv = dev_in.view(q.dtype).view(q.shape)
        out_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        ios.append((host_in, dev_in, out_h))
        steps.append((qv, layers[l][1], layers[l][2], t))
    gi = CascadeLayersGraph(steps, host_io=ios)
    gi.replay()
    torch.cuda.synchronize()
    for (_, _, out_h), l in zip(ios, order):
        assert torch.equal(out_h, cascade_decode(*layers[l], t).cpu())
    with pytest.raises(ValueError):
        CascadeLayersGraph(steps, host_io=ios[:1])


@pytest.mark.parametrize("use,io_group", [([0, 1, 0, 1], 1), ([0, 1, 0, 1], 4), ([0, 1, 2, 0, 1, 2, 0], 4),
                                          ([0, 1, 2, 3, 0, 1, 2, 3, 0], 2), ([0, 0, 1], 4)])
def test_layers_graph_overlapped_host_io_reuses_buffers_safely(use, io_group):
    """overlap_io=True where steps share device input buffers (e.g. steps 0
    and 2 load different host queries into the same dev_in): a step's
    host->device copy must wait until the earlier step on that buffer has
    read it, and a copy group ends before a buffer repeats, so every step's
    pinned output equals the eager step on its OWN query -- for copy groups
    of 1, 2 and 4 steps."""
    import torch
    from cascade_kernel.cascade import CascadeLayersGraph, cascade_decode
    Hh.need_cuda()
    kw = dict(CASES["c1_like"])
    kw["dtype"] = torch.float16
    w = _work("layers_ovl", **kw)
    t = w.tables
    gen = torch.Generator(device="cuda").manual_seed(9)
    k2, v2 = (torch.randn(x.shape, device="cuda", generator=gen).to(x.dtype) for x in (w.k_pool, w.v_pool))
    pools = [((w.k_pool, w.v_pool), (k2, v2))[(i * 5 // 3) % 2] for i in range(len(use))]
    nbytes = w.q.numel() * w.q.element_size()
    dins = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(max(use) + 1)]
    qs = [torch.randn(w.q.shape, device="cuda", generator=gen).to(w.q.dtype) for _ in use]
    steps, io = [], []
    for i, b in enumerate(use):
        hin = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        hin.copy_(qs[i].view(-1).view(torch.uint8).cpu())
        out_h = torch.empty(w.q.shape, dtype=w.q.dtype).pin_memory()
        steps.append((dins[b].view(w.q.dtype).view(w.q.shape), pools[i][0], pools[i][1], t))
        io.append((hin, dins[b], out_h))
    g = CascadeLayersGraph(steps, host_io=io, overlap_io=True, io_group=io_group)
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        for i in range(len(use)):
            assert torch.equal(io[i][2], cascade_decode(qs[i], pools[i][0], pools[i][1], t).cpu())


@pytest.mark.parametrize("suffix", ["long", "empty"])
def test_overlapped_stage1_other_shapes_vs_oracle(suffix):
    """The step's two-segment stage-1 away from the C4 shape: one group of 64
    requests, 64 q / 8 kv heads, a 24,576-token prefix (8 streams of 192
    tiles: the overlap is planned with 25 partial planes). Suffixes U[1000,
    2000] (98,819 tokens) give a segment A of 640 tiles (20 per run, no
    stream-aligned size within reach); near-empty suffixes (zeros and a few
    1-3 token ones) give none, the decode and segment B then doing all the
    work. Checked against
    the CPU oracle on every kv head."""
    import torch
    from cascade_kernel import capi
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    rng = np.random.default_rng(21)
    lens = (list(rng.integers(1000, 2001, 64)) if suffix == "long"
            else [0] * 60 + [1, 2, 3, 1])
    w = _work("ovl_" + suffix, group_sizes=[64], prefix_lens=[24576], suffix_lens=lens, H=64, KVH=8, bs=128,
              dtype=torch.bfloat16, seed=22)
    t = w.tables
    dp = capi.paged_desc(w.q, w.k_pool, w.v_pool, t.prefix_block_table, t.prefix_q_seqlens, t.prefix_kv_seqlens,
                         t.uniform_group)
    # the step writes split partials on both sides (the partials-only flag)
    ds = capi.paged_desc(w.q, w.k_pool, w.v_pool, t.suffix_block_table, t.suffix_q_seqlens, t.suffix_kv_seqlens, 1,
                         flags=capi.FLAG_PARTIALS_ONLY)
    pb = capi.plan(ds, 1, True)
    align = lambda n: -(-n // 256) * 256
    # the step's workspace holds the overlap's 25 stage-1 planes
    assert capi.decode_step_workspace_size(dp, ds) == align(25 * 64 * 64 * 129 * 4) + align(pb.workspace_bytes)
    got = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=True)
    torch.cuda.synchronize()
    assert Hh.capi().device_error() == 0
    a = Hh.dev_to_f64(got)
    assert np.isfinite(a).all()
    ref, _ = Hh.step_oracle_all_heads(w, out_dtype="fp32", round_suffix=False)
    err = np.abs(a - ref)
    assert (err <= O.ulp(ref, "bf16") + 2e-3).all(), float((err - O.ulp(ref, "bf16")).max())
