"""GPU parity of the paged-attention ops (stage-1 prefix and suffix decode)
against the CPU oracle and the reference golden fixtures, through the C ABI.

Gates (the reference's own, run_precision_suite.py:72-89):
  * reference parity: |O - O_golden| within the tolerance stated per test,
    LSE within 1e-3 absolute (BASELINE), -inf matching -inf;
  * kernel-structured oracle (same online-softmax chunks and KV splits as the
    kernel): |O - O_ks| <= A + 3e-6 (A = bf16 near-tie bound), LSE <= 1e-5.
"""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu

FIXTURES = ["min_b1_kv128", "kv_448_tail", "varlen_3req", "qlen2_b4", "h2_kvh1", "padded_block_cols",
            "flat_T17_g5", "flat_T64_g4", "b8_kvh1_g8", "perm_table_varlen"]

# stage-1 out is fp32: the reference parity tolerance is tighter than the
# BASELINE bf16 bound of 2e-2 (the only difference from the 512-chunk golden
# is where P is rounded to bf16)
O_TOL_REF = 5e-3
LSE_TOL = 1e-3


def _assert_within(o, ref, bound, kvs=None):
    excess = np.abs(o - ref) - bound
    if (excess > 0).any():
        i = np.unravel_index(np.argmax(excess), excess.shape)
        raise AssertionError(
            f"{int((excess > 0).sum())} elements out of bound; worst at {i} (kv={None if kvs is None else kvs[i[0]]}): "
            f"got {o[i]:.8g} ref {ref[i]:.8g} bound {bound[i]:.3g}")


def _check_stage1(z, out, lse, q_len_max):
    T = z["q_bits"].shape[0]
    H = int(z["H"])
    KVH = int(z["KVH"])
    o = Hh.dev_to_f64(out)
    l8 = Hh.dev_to_f64(lse).reshape(-1, 8)
    # the padded-row invariant: all 8 copies of a row identical
    assert np.array_equal(l8, np.repeat(l8[:, :1], 8, axis=1))
    l = l8[:, 0].reshape(T, H)
    # reference parity against the reference's own golden output
    assert np.abs(o - z["o_ref"]).max() < O_TOL_REF
    assert np.abs(l - z["lse_ref"]).max() < LSE_TOL
    # exact structure check against the kernel-structured oracle
    qh, kh, vh, bt, qs, kvs = Hh.fixture_host_args(z)
    _, kw = Hh.kernel_structure(q_len_max, H // KVH, None, T, H, KVH, len(qs), bt.shape[1], kh.shape[1])
    o_ks, l_ks, A = O.paged_attention_ref(qh, kh, vh, bt, qs, kvs, with_tieband=True,
                                          tieband_rule="rescaled", **kw)
    _assert_within(o, o_ks, A + 3e-6)
    assert np.abs(l - l_ks).max() < 1e-5


@pytest.mark.parametrize("name", FIXTURES)
@pytest.mark.parametrize("fast", [False, True], ids=["legacy", "fast"])
def test_stage1_golden_fixture(name, fast):
    Hh.need_cuda()
    z = Hh.load_fixture(name)
    args = Hh.fixture_device_args(z)
    q_len = int(z["q_len"])
    out, lse = Hh.run_capi_paged(*args, q_len if fast else 0)
    _check_stage1(z, out, lse, q_len)


@pytest.mark.parametrize("name", ["kv_448_tail", "varlen_3req", "flat_T64_g4", "perm_table_varlen"])
def test_stage1_fast_path_bit_identical_to_legacy(name):
    """test_q_seqlen_fastpath.py F1: q_seqlen_value=q_len is bit-identical."""
    Hh.need_cuda()
    z = Hh.load_fixture(name)
    args = Hh.fixture_device_args(z)
    o0, l0 = Hh.run_capi_paged(*args, 0)
    o1, l1 = Hh.run_capi_paged(*args, int(z["q_len"]))
    assert np.array_equal(o0.cpu().numpy().view(np.uint32), o1.cpu().numpy().view(np.uint32))
    assert np.array_equal(l0.cpu().numpy().view(np.uint32), l1.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("name", ["varlen_3req", "flat_T64_g4"])
def test_stage1_ten_run_bit_stability(name):
    """fa_fp32_stage1 S4 / F4: 10 runs bit-identical."""
    Hh.need_cuda()
    z = Hh.load_fixture(name)
    args = Hh.fixture_device_args(z)
    first = None
    for _ in range(10):
        o, l = Hh.run_capi_paged(*args, int(z["q_len"]))
        b = (o.cpu().numpy().tobytes(), l.cpu().numpy().tobytes())
        first = first or b
        assert b == first


def _rand_case(B, H, KVH, bs, kv_lens, q_len, dtype, seed, permute=True, cols_extra=0):
    import torch
    rng = np.random.default_rng(seed)
    pages = [(int(k) + bs - 1) // bs for k in kv_lens]
    n = sum(pages) + 3
    perm = rng.permutation(n).astype(np.int32) if permute else np.arange(n, dtype=np.int32)
    cols = max(1, max(pages)) + cols_extra
    bt = np.full((B, cols), -7, np.int32)  # garbage beyond each request's pages
    c = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[c:c + pages[b]]
        c += pages[b]
    qf = O.quantize(rng.standard_normal((B * q_len, H, 128)), dtype)
    kf = O.quantize(rng.standard_normal((n, bs, KVH, 128)), dtype)
    vf = O.quantize(rng.standard_normal((n, bs, KVH, 128)), dtype)
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    dev = [torch.from_numpy(x.astype(np.float32)).to(td).cuda() for x in (qf, kf, vf)]
    qs = np.full(B, q_len, np.int64)
    kvs = np.asarray(kv_lens, np.int64)
    dev += [torch.from_numpy(bt).cuda(), torch.from_numpy(qs).cuda(), torch.from_numpy(kvs).cuda()]
    return dev, (qf, kf, vf, bt, qs, kvs)


@pytest.mark.parametrize("H,kv_lens", [(32, [9600, 3000]), (64, [9728])], ids=["one_pair_ragged", "two_pairs"])
def test_stage1_equal_runs_exact_structure(H, kv_lens):
    """Two-tile stage-1 on the equal-run schedule (units' KV tiles cut into one
    run per SM, a run spanning two units, a unit's pieces on consecutive
    planes, pieces past a short prefix empty): against the kernel-structured
    oracle of exactly those pieces, and the fp64 single pass at the reference
    tolerance."""
    Hh.need_cuda()
    KVH, q_len, bs = 8, 64, 128
    group = H // KVH
    dev, (qf, kf, vf, bt, qs, kvs) = _rand_case(len(kv_lens), H, KVH, bs, kv_lens, q_len, "bf16", seed=11)
    pieces = Hh.stage1_pieces(q_len, group, KVH, len(kv_lens), bt.shape[1] * bs)
    assert pieces is not None  # the shape takes the equal-run schedule
    assert max(len(pieces(b, g, mp)) for b in range(len(kv_lens)) for g in range(KVH)
               for mp in range(q_len * group // 256)) >= 3
    out, lse = Hh.run_capi_paged(*dev, q_len)
    o = Hh.dev_to_f64(out)
    l = Hh.dev_to_f64(lse).reshape(-1, 8)[:, 0].reshape(o.shape[0], H)
    o_ks, l_ks, A = Hh.stage1_pieces_oracle(qf, kf, vf, bt, qs, kvs, group, pieces)
    _assert_within(o, o_ks, A + 3e-6)
    assert np.abs(l - l_ks).max() < 1e-5
    o_ref, l_ref = O.paged_attention_ref(qf, kf, vf, bt, qs, kvs, chunk=512)
    assert np.abs(o - o_ref).max() < O_TOL_REF
    assert np.abs(l - l_ref).max() < LSE_TOL


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("bs", [16, 32, 64, 128, 256])
def test_suffix_decode_block_sizes(dtype, bs):
    """Suffix decode (q_len=1, GQA 5) over every supported page size, ragged
    lengths including 0 and 1, random-permutation tables, garbage past the
    last page."""
    Hh.need_cuda()
    kv = [0, 1, 15, 16, 17, 200, 255, 256, 257, 700, 1024, 0, 3]
    dev, host = _rand_case(len(kv), 10, 2, bs, kv, 1, dtype, seed=bs)
    out, lse = Hh.run_capi_paged(*dev, 1, suffix=True)
    qf, kf, vf, bt, qs, kvs = host
    C = Hh.capi()
    split = C.plan(C.paged_desc(*dev, 1), 1, True).split_tokens
    seg = lambda n: O.decode_segments(n, split=split, tile=64, warps=4)
    o_ks, l_ks, A = O.paged_attention_ref(qf, kf, vf, bt, qs, kvs, segments=seg, p_dtype=dtype,
                                          with_tieband=True, tieband_rule="rescaled")
    o = Hh.dev_to_f64(out)
    l = Hh.dev_to_f64(lse).reshape(o_ks.shape[:2])
    # the fp32 result (within A + 3e-6 of the oracle) is rounded to the input
    # dtype: |round(x') - x| <= ulp(round(x'))/2 + |x' - x|
    half_ulp = 0.5 * np.maximum(O.ulp(o_ks, dtype), O.ulp(o, dtype))
    _assert_within(o, o_ks, A + half_ulp + 3e-6, kvs)
    z = kvs == 0
    assert np.all(np.isneginf(l[z])) and np.all(o[z] == 0)
    assert np.abs(l[~z] - l_ks[~z]).max() < 1e-5
    # BASELINE parity against the reference-structured oracle (chunk 512)
    o_ref, l_ref = O.paged_attention_ref(qf, kf, vf, bt, qs, kvs, p_dtype=dtype)
    np.testing.assert_allclose(o[~z], o_ref[~z], atol=2e-2, rtol=2e-2)
    assert np.abs(l[~z] - l_ref[~z]).max() < LSE_TOL


@pytest.mark.parametrize("q_len,H,dtype", [(1, 16, "bf16"), (1, 16, "fp16"), (2, 40, "fp16"), (4, 32, "bf16")])
def test_planned_suffix_decode_wide_ragged(q_len, H, dtype):
    """A wide ragged batch (512 requests x 8 kv heads, block size 16, lengths
    from 0 to 4000, most short: 8 splits x 4096 pairs > 16384 slots) takes
    the planned decode: the device lists only the non-empty (request, split)
    items and the empty split slots get -inf partials. Same gates as the
    per-item decode, with and without the combine (partials only); 2, 10
    and 16 query rows per (request, kv head) (the item slot's Q rows)."""
    import torch
    Hh.need_cuda()
    rng = np.random.default_rng(11)
    kv = np.clip(rng.lognormal(np.log(150), 1.0, 512), 1, 4000).astype(int)
    kv[rng.random(512) < 0.1] = 0
    kv[:3] = [4000, 1025, 512]
    dev, host = _rand_case(512, H, 8, 16, list(kv), q_len, dtype, seed=21 + q_len)
    C = Hh.capi()
    plan = C.plan(C.paged_desc(*dev, q_len), q_len, True)
    assert plan.kernel == 2 and plan.split_tokens == 512 and plan.num_splits == 8
    out, lse = Hh.run_capi_paged(*dev, q_len, suffix=True)
    qf, kf, vf, bt, qs, kvs = host
    seg = lambda n: O.decode_segments(n, split=512, tile=64, warps=4)
    o_ks, l_ks, A = O.paged_attention_ref(qf, kf, vf, bt, qs, kvs, segments=seg, p_dtype=dtype,
                                          with_tieband=True, tieband_rule="rescaled")
    o = Hh.dev_to_f64(out)
    l = Hh.dev_to_f64(lse).reshape(o_ks.shape[:2])
    half_ulp = 0.5 * np.maximum(O.ulp(o_ks, dtype), O.ulp(o, dtype))
    kv_tok = np.repeat(kvs, q_len)  # per query token
    _assert_within(o, o_ks, A + half_ulp + 3e-6, kv_tok)
    z = kv_tok == 0
    assert np.all(np.isneginf(l[z])) and np.all(o[z] == 0)
    assert np.abs(l[~z] - l_ks[~z]).max() < 1e-5
    # partials only: slot s of a request holds its split s (or -inf beyond its length)
    d = C.paged_desc(*dev, q_len, flags=C.FLAG_PARTIALS_ONLY)
    ws = torch.full((C.suffix_workspace_size(d),), 0x7F, dtype=torch.uint8, device="cuda")
    C.suffix_decode(d, None, None, ws)
    torch.cuda.synchronize()
    assert C.device_error() == 0
    rows = 512 * q_len * H
    part_lse = ws[8 * 4 * rows * 128:8 * 4 * rows * 129].view(torch.float32).view(8, 512, q_len * H).cpu().numpy()
    used = np.minimum(8, -(-kvs // 512))
    for s in range(8):
        assert np.all(np.isneginf(part_lse[s][s >= used])), s
        assert np.all(np.isfinite(part_lse[s][s < used])), s


def test_block_table_indexing_exact():
    """V pages filled with their physical page id and one-hot scores: the
    output must equal the selected page id exactly (indexing is bit-exact)."""
    import torch
    Hh.need_cuda()
    B, H, KVH, bs = 6, 4, 1, 16
    kv = [1, 16, 17, 100, 333, 1000]
    dev, host = _rand_case(B, H, KVH, bs, kv, 1, "bf16", seed=5)
    q, k, v, bt, qs, kvs = dev
    n = k.shape[0]
    v.copy_(torch.arange(n, device="cuda", dtype=torch.float32).view(n, 1, 1, 1).expand_as(v).to(torch.bfloat16))
    # one-hot: every key zero except the chosen token of each request, aligned with q
    k.zero_()
    bt_h = host[3]
    chosen = [int(x) - 1 for x in kv]  # the last valid token
    for b in range(B):
        t = chosen[b]
        page = int(bt_h[b, t // bs])
        k[page, t % bs, 0, :] = q[b, 0, :] * 64.0
    q[:, 1:, :] = q[:, :1, :]
    out, lse = Hh.run_capi_paged(q, k, v, bt, qs, kvs, 1, suffix=True)
    o = out.float().cpu().numpy()
    assert k.shape[0] <= 256  # page ids exact in bf16
    for b in range(B):
        page = int(bt_h[b, chosen[b] // bs])
        # the chosen token's weight is exactly 1, every other exp underflows to 0
        assert np.all(o[b] == page), (b, o[b, :, 0], page)


def test_stage1_negative_checks():
    """run_precision_suite.py:96-138 and test_q_seqlen_fastpath.py F3: rejected
    before launch with the op name in the message."""
    Hh.need_cuda()
    C = Hh.capi()
    dev, host = _rand_case(4, 8, 2, 128, [512] * 4, 1, "bf16", seed=1, permute=False)
    q, k, v, bt, qs, kvs = dev
    with pytest.raises(C.CascadeError, match="fa_fp32_stage1.*sum"):
        Hh.run_capi_paged(q[:-1], k, v, bt, qs, kvs, 0)
    with pytest.raises(C.CascadeError, match="fa_fp32_stage1.*cols too small"):
        Hh.run_capi_paged(q, k, v, bt[:, :1].contiguous(), qs, kvs, 0)
    kv0 = kvs.clone()
    kv0[-1] = 0
    with pytest.raises(C.CascadeError, match="fa_fp32_stage1.*>= 1"):
        Hh.run_capi_paged(q, k, v, bt, qs, kv0, 0)
    with pytest.raises(C.CascadeError, match="q_seqlen_value"):
        Hh.run_capi_paged(q, k, v, bt, qs, kvs, 2)


def test_torch_op_matches_capi_and_rejects_like_reference():
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    z = Hh.load_fixture("varlen_3req")
    args = Hh.fixture_device_args(z)
    o_c, l_c = Hh.run_capi_paged(*args, 1)
    o_t, l_t = npu.fa_fp32_stage1(*args, 1)
    torch.cuda.synchronize()
    assert torch.equal(o_c, o_t) and torch.equal(l_c, l_t)
    q, k, v, bt, qs, kvs = args
    with pytest.raises(RuntimeError, match="fa_fp32_stage1: query must be bf16"):
        npu.fa_fp32_stage1(q.half(), k, v, bt, qs, kvs, 1)
    with pytest.raises(RuntimeError, match="fa_fp32_stage1: all inputs must be contiguous"):
        npu.fa_fp32_stage1(q.transpose(0, 1), k, v, bt, qs, kvs, 1)
    with pytest.raises(RuntimeError, match="fa_fp32_stage1: block_table must be int32"):
        npu.fa_fp32_stage1(q, k, v, bt.long(), qs, kvs, 1)
    with pytest.raises(RuntimeError, match="only paged blockSize 128"):
        npu.fa_fp32_stage1(q, k.view(-1, 64, k.shape[2], 128), v.view(-1, 64, k.shape[2], 128), bt, qs, kvs, 1)
    # empty batch -> empty outputs (op_host/fa_fp32_stage1.cpp:209-213)
    e = torch.empty((0,), dtype=torch.int64, device="cuda")
    o, l = npu.fa_fp32_stage1(q[:0], k, v, bt[:0], e, e, 0)
    assert o.shape == (0, q.shape[1], 128) and l.numel() == 0
