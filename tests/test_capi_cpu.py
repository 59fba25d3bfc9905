"""CPU-only checks of the native boundary: the C-ABI library loads and exports
every symbol include/cascade_b200.h declares; the torch extension registers
the reference's schemas byte-identically; the host-side planner and
validation behave like the reference op hosts. No CUDA calls."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "cascade_b200.h")


def _declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"CASCADE_API\s+[\w\s\*]+?\b(cascade_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    from cascade_kernel import capi
    lib = capi.load()
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(capi.EXPORTED) == names
    assert lib.cascade_version() == 100


def test_torch_schemas_match_reference():
    import torch
    import cascade_kernel  # noqa: F401
    want = {
        "lse_merge": "npu::lse_merge(Tensor o1, Tensor o2, Tensor lse1, Tensor lse2, int out_code=0) -> Tensor",
        "fa_fp32_stage1": "npu::fa_fp32_stage1(Tensor query, Tensor key, Tensor value, Tensor block_table, "
                          "Tensor actual_q_seqlens, Tensor actual_kv_seqlens, int q_seqlen_value=0) -> "
                          "(Tensor, Tensor)",
        "f3_gateup_epilogue": "npu::f3_gateup_epilogue(Tensor a, Tensor b, Tensor? workspace, Tensor? out_d, "
                              "int mode) -> (Tensor, Tensor)",
        "add_rms_norm_stats": "npu::add_rms_norm_stats(Tensor x1, Tensor x2, Tensor? gamma, Tensor? beta, "
                              "float eps, int mode) -> (Tensor, Tensor, Tensor)",
    }
    for name, schema in want.items():
        op = getattr(torch.ops.npu, name)
        assert str(op.default._schema) == schema


def test_cpu_tensor_has_no_fallback():
    import torch
    import cascade_kernel  # noqa: F401
    o = torch.zeros(2, 4, 16)
    with pytest.raises(NotImplementedError):
        torch.ops.npu.lse_merge(o, o.bfloat16(), torch.zeros(8), torch.zeros(8), 2)


def _desc(**kw):
    from cascade_kernel import capi
    shape = dict(num_tokens=64, num_heads=32, head_dim=128, num_blocks=1000, block_size=128, kv_heads=8,
                 batch=64, block_cols=8)
    qsv = kw.pop("q_seqlen_value", 1)
    dtype = kw.pop("dtype", capi.BF16)
    shape.update(kw)
    return capi.paged_desc(None, None, None, None, None, None, qsv, shape=shape, dtype=dtype)


def test_planner_kernel_choice_and_splits():
    from cascade_kernel import capi
    # C2 suffix: q_len 1, group 4 -> decode path, 512-token splits
    p = capi.plan(_desc(), 1, True)
    assert (p.kernel, p.rows_per_group, p.split_tokens, p.num_splits) == (0, 4, 512, 2)
    assert p.workspace_bytes == 2 * 64 * 32 * 129 * 4
    # C2 stage-1: one flattened request of 64 tokens -> 256 rows -> tcgen05 path
    p = capi.plan(_desc(num_tokens=64, batch=1, block_cols=32, q_seqlen_value=64), 64, False)
    assert p.kernel == 1 and p.rows_per_group == 256 and p.split_tokens % 128 == 0
    assert p.num_splits * p.split_tokens >= 32 * 128
    # two-tile form: 8 (kv head, tile pair) units x 16 splits = 128 CTAs
    assert (p.split_tokens, p.num_splits) == (256, 16)
    # C5-like stage-1 (32 groups x 16 requests, group 5, prefixes up to 4016
    # tokens at bs 16): 256 row tiles fill the SMs already, but the longest
    # prefixes are still cut in two
    p = capi.plan(_desc(num_tokens=512, batch=32, num_heads=40, block_size=16, block_cols=251, q_seqlen_value=16),
                  16, False)
    assert p.kernel == 1 and (p.split_tokens, p.num_splits) == (2048, 2)
    # C4-like (4 groups x 64 requests, group 8, prefix 16384): 64 tile pairs x 128 tiles cut into 148
    # equal runs of 55-56 tiles (pieces of at most 56 x 128 tokens; some unit spans 4 runs -> 4 planes)
    p = capi.plan(_desc(num_tokens=256, batch=4, num_heads=64, block_cols=128, q_seqlen_value=64), 64, False)
    assert p.kernel == 1 and (p.split_tokens, p.num_splits) == (7168, 4)
    # 128 rows or fewer per request: one row tile per CTA, 148 / units splits
    p = capi.plan(_desc(num_tokens=32, batch=1, num_heads=32, block_cols=32, q_seqlen_value=32), 32, False)
    assert p.kernel == 1 and (p.split_tokens, p.num_splits) == (256, 16)
    # 16 rows is still the decode path, 17 is not
    assert capi.plan(_desc(num_tokens=5, batch=1, q_seqlen_value=5, num_heads=32), 5, False).kernel == 1
    assert capi.plan(_desc(num_tokens=4, batch=1, q_seqlen_value=4, num_heads=16), 4, False).kernel == 0
    # workspace size: shape-only, covers both kernels on the legacy path
    lib = capi.load()
    for q_len in (1, 5):
        d = _desc(q_seqlen_value=0, num_tokens=64, batch=64 // q_len if q_len == 1 else 12)
        fast = _desc(q_seqlen_value=q_len, num_tokens=64 if q_len == 1 else 60, batch=64 if q_len == 1 else 12)
        want = capi.plan(fast, q_len, False).workspace_bytes
        assert lib.cascade_fa_fp32_stage1_workspace_size(ctypes.byref(d)) >= want


@pytest.mark.parametrize("kw,msg", [
    (dict(head_dim=64), "only head dim 128"),
    (dict(block_size=48), "blockSize must be one of"),
    (dict(num_heads=30), "multiple of kvHeads"),
    (dict(q_seqlen_value=2), "query.size\\(0\\) must equal batch \\* q_seqlen_value"),
    (dict(q_seqlen_value=-1), "q_seqlen_value must be >= 0"),
    (dict(dtype=2), "bf16 or fp16"),
])
def test_planner_validation_messages(kw, msg):
    from cascade_kernel import capi
    d = _desc(**kw)
    with pytest.raises(capi.CascadeError, match="fa_fp32_stage1: .*" + msg):
        capi.plan(d, 1, False)


def test_merge_validation_without_gpu():
    from cascade_kernel import capi
    lib = capi.load()
    rc = lib.cascade_lse_merge(None, 0, None, 0, None, 1, None, 1, None, 3, 4, 128, None)
    assert rc == capi.ERR_INVALID and "dtypes" in capi.last_error()
    rc = lib.cascade_lse_merge(None, 0, None, 0, None, 1, None, 1, None, 0, 4, 24, None)
    assert rc == capi.ERR_INVALID and "multiple of 16" in capi.last_error()
    rc = lib.cascade_lse_merge(None, 0, None, 0, None, 65, None, 1, None, 0, 4, 128, None)
    assert rc == capi.ERR_INVALID and "stride" in capi.last_error()
    assert lib.cascade_lse_merge(None, 0, None, 0, None, 1, None, 1, None, 0, 0, 128, None) == 0


def test_gateup_validation_without_gpu():
    from cascade_kernel import capi
    lib = capi.load()
    assert lib.cascade_f3_gateup_epilogue(None, None, None, None, 128, 16, 64, 128, 6, None) == capi.ERR_INVALID
    assert "mode must be" in capi.last_error()
    assert lib.cascade_f3_gateup_epilogue(None, None, None, None, 100, 16, 64, 100, 1, None) == capi.ERR_INVALID
    assert "N tile" in capi.last_error()
    assert lib.cascade_f3_gateup_epilogue(None, None, None, None, 128, 16, 48, 128, 1, None) == capi.ERR_INVALID
    assert lib.cascade_f3_gateup_epilogue(None, None, None, None, 128, 16, 64, 128, 2, None) == capi.ERR_WORKSPACE


def test_add_rms_norm_stats_validation_without_gpu():
    """The C ABI rejects, before any launch, what op_host/add_rms_norm_stats.cpp
    rejects (mode, eps, dtype, empty M, K range, K % 16), with its texts."""
    from cascade_kernel import capi
    lib = capi.load()
    def rc(M=4, K=128, dtype=capi.BF16, mode=0, eps=1e-6):
        return lib.cascade_add_rms_norm_stats(None, None, None, None, None, None, None, M, K, dtype, mode, eps, None)
    assert rc(mode=3) == capi.ERR_INVALID and "mode must be 0, 1 or 2" in capi.last_error()
    assert rc(eps=0.0) == capi.ERR_INVALID and "eps must be > 0" in capi.last_error()
    assert rc(dtype=capi.FP32) == capi.ERR_INVALID and "bf16 or fp16" in capi.last_error()
    assert rc(M=0) == capi.ERR_INVALID and "empty row count" in capi.last_error()
    assert rc(K=5136) == capi.ERR_INVALID and "(0, 5120]" in capi.last_error()
    assert rc(K=24) == capi.ERR_INVALID and "multiple of 16" in capi.last_error()
    assert rc() == capi.ERR_INVALID and "null pointer" in capi.last_error()


def test_planner_planned_decode_choice_and_workspace():
    """Kernel 2 (planned decode) exactly when the uniform-q one-CTA-per-item
    grid at 512-token splits would exceed 16384 CTAs; its workspace adds the
    item list [batch * splits], the count and one counter per kv head."""
    from cascade_kernel import capi
    def plan(B, cols, bs=16, KVH=8, q=1):
        d = _desc(num_tokens=B * q, batch=B, kv_heads=KVH, num_heads=KVH * 5, block_size=bs, block_cols=cols,
                  q_seqlen_value=q)
        return capi.plan(d, q, True)
    p = plan(512, 290)                       # C5-like: 4096 pairs x 10 splits
    assert (p.kernel, p.split_tokens, p.num_splits) == (2, 512, 10)
    rows = 512 * 40
    assert p.workspace_bytes == 10 * rows * 129 * 4 + (512 * 10 + 1 + 8) * 4
    assert plan(256, 16, bs=128).kernel == 0   # C4-like: 2048 pairs x 4 splits = 8192
    assert plan(512, 32, bs=16).kernel == 0    # one split only
    assert plan(64, 8, bs=128, KVH=8).kernel == 0
    d = _desc(num_tokens=512, batch=512, kv_heads=8, num_heads=40, block_size=16, block_cols=290, q_seqlen_value=0)
    assert capi.plan(d, 1, True).kernel == 0  # per-request q lengths: never planned


def _two_segment_pieces(T, tc, ga, gb, TA):
    """Restatement of the stage-1 wrapper's run map (prefix_tc.cu): runs
    [0, ga) cut [0, TA), runs [ga, ga + gb) cut [TA, T) (TA = T: one
    segment); a piece is a run's part inside one unit of tc tiles, written to
    plane run - run_of(unit's first tile). Returns {unit: [(start, end, plane)]}."""
    def bnd(r):
        return r * TA // ga if r <= ga else TA + (r - ga) * (T - TA) // gb

    def run_of(x):
        if x < TA:
            return ((x + 1) * ga + TA - 1) // TA - 1
        return ga + ((x - TA + 1) * gb + (T - TA) - 1) // (T - TA) - 1

    out = {}
    for run in range(ga + gb):
        x, hi = bnd(run), bnd(run + 1)
        while x < hi:
            u = x // tc
            end = min(hi, (u + 1) * tc)
            out.setdefault(u, []).append((x - u * tc, end - u * tc, run - run_of(u * tc)))
            x = end
    return out


def _overlap_tiles(tokens, kv_heads, ga, gb, T, tc):
    """Restatement of overlap_tiles (kernels.h): segment A's tiles from the
    suffix's kv tokens (6 TB/s decode, 3.3 us per stage-1 tile, runs of at
    least 16 tiles or none, at most 3/5 of the tiles); within 40% of that,
    the size whose segment-B runs are tc >> k tiles."""
    per_run = int(tokens * kv_heads * 512.0 / 6000.0 / 3300.0)
    per_run = min(per_run, (3 * T) // 5 // ga)
    if per_run < 16:
        return 0
    est = per_run * ga
    best = None
    for k in range(4):
        lb = tc >> k
        if lb < 8 or (lb << k) != tc:
            break
        ta = T - gb * lb
        if ta < 16 * ga or ta > (3 * T) // 5 or 5 * abs(ta - est) > 2 * est:
            continue
        if best is None or abs(ta - est) < abs(best - est):
            best = ta
    return est if best is None else best


@pytest.mark.parametrize("kv_heads", [8, 4, 2])
def test_overlapped_stage1_schedule_and_workspace(kv_heads):
    """The C4 step (4 groups x 64 requests, prefix 16384, suffix <= 2048 on the
    per-item decode) runs stage-1 in two segments around the decode: 32 runs
    (64 CTAs) over the first TA tiles, the 74-run equal schedule over the rest.
    For every TA the device can choose, each unit's pieces cover its tiles
    once, in order, on planes 0, 1, ... below the planner's bound, which the
    step's workspace size holds (9 planes on C4). kv_heads 4: the shard of 2
    ranks (13 planes); kv_heads 2 (4 ranks): too few tiles, the serial order."""
    from cascade_kernel import capi
    pre = _desc(num_tokens=256, num_heads=8 * kv_heads, kv_heads=kv_heads, batch=4, block_cols=128,
                q_seqlen_value=64, num_blocks=40000)
    suf = _desc(num_tokens=256, num_heads=8 * kv_heads, kv_heads=kv_heads, batch=256, block_cols=16,
                q_seqlen_value=1, num_blocks=40000)
    pa, pb = capi.plan(pre, 64, True), capi.plan(suf, 1, True)
    assert pa.kernel == 1 and pb.kernel == 0 and pb.num_splits == (2 if kv_heads == 8 else 4)
    tc, ga, gb = 128, 32, 74
    T = kv_heads * 4 * tc
    minrun = min(16, (T - 3 * T // 5) // gb)
    got = capi.decode_step_workspace_size(pre, suf)
    align = lambda n: -(-n // 256) * 256
    if minrun < 8:
        # segment B's runs would be shorter than 8 tiles (the 4-rank shard):
        # no overlap, the plan's own planes
        assert got == align(pa.workspace_bytes) + align(pb.workspace_bytes)
        return
    bound = -(-tc // minrun) + 1
    rows = 256 * 8 * kv_heads
    assert got == align(bound * rows * 129 * 4) + align(pb.workspace_bytes)
    # every TA the device can choose: a multiple of ga with runs of >= 16 tiles
    # up to 3/5 of the tiles, or T - gb * (tc >> k) in that range
    TAs = [0] + sorted(set([r * ga for r in range(16, (3 * T) // 5 // ga + 1)]
                           + [T - gb * (tc >> k) for k in range(4) if 16 * ga <= T - gb * (tc >> k) <= 3 * T // 5]))
    for TA in TAs:
        for u, ps in _two_segment_pieces(T, tc, ga, gb, TA).items():
            assert [p[2] for p in ps] == list(range(len(ps))), (TA, u)
            assert ps[0][0] == 0 and ps[-1][1] == tc and all(a[1] == b[0] for a, b in zip(ps, ps[1:]))
            assert len(ps) <= bound
    # the C4 suffix of bench.py's seed (304,653 tokens): 63 tiles per run
    # estimated (2,016 tiles); 32-tile segment-B runs (TA = 4096 - 74 * 32 =
    # 1,728) lie within 40% of it and are taken
    if kv_heads == 8:
        assert _overlap_tiles(304653, 8, ga, gb, T, tc) == 1728
    if kv_heads == 4:  # 31 tiles per run estimated (992); 16-tile segment-B runs: 2048 - 74 * 16 = 864
        assert _overlap_tiles(304653, 4, ga, gb, T, tc) == 864


def test_overlap_not_used_for_small_or_planned_steps():
    """C2 (prefix-first) keeps its workspace: no extra stage-1 planes."""
    from cascade_kernel import capi
    pre = _desc(num_tokens=64, batch=1, block_cols=32, q_seqlen_value=64)
    suf = _desc(num_tokens=64, batch=64, block_cols=8, q_seqlen_value=1)
    align = lambda n: -(-n // 256) * 256
    assert capi.decode_step_workspace_size(pre, suf) == (align(capi.plan(pre, 64, True).workspace_bytes)
                                                        + align(capi.plan(suf, 1, True).workspace_bytes))
