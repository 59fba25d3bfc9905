"""The reference's fa_fp32_stage1 precision suite on the GPU, at full size.

15 shapes x seeds {0, 1} (ascend-kernel/csrc/ops/fa_fp32_stage1/test/
run_precision_suite.py:19-37, H=40/KVH=8 up to 64 x 8192 and 2 x 16384
tokens), inputs from the restated gen_inputs (pinned bit for bit on the CPU),
run through torch.ops.npu.fa_fp32_stage1 in the default mode the suite uses
(seqlens read back, :53-61) and in the fast q_seqlen_value mode, which must be
bit-identical. Gates, per case and seed, over every kv head:
  * the suite's padded-LSE stride invariant (all 8 copies of a row equal, :65-68);
  * its tie-band gate |O - O_ref| <= A + 3e-6 (:76-89), with O_ref and A from
    the oracle run in the kernel's own quantisation structure (the decode
    kernel's 16-token chunks per warp and its KV splits; A = the bf16 near-tie
    bound, carried like the accumulator);
  * LSE within 1e-3 of the reference's OWN fp64 golden (stored by
    tests/golden/make_golden.py) and within 1e-5 of the kernel-structured
    oracle;
  * the BASELINE bar, |O - O_ref| <= 2e-2 + 2e-2 |O_ref|;
and the suite's three host rejections (:93-138) at its own shape.
The fp64 oracle runs in a spawned process pool, one item per (case, seed,
kv head)."""
import multiprocessing as mp
import os

import numpy as np
import pytest

import helpers as Hh
from conftest import GOLDEN
from suite_cases import CASES, SEEDS, oracle_head, spec, suite_inputs

pytestmark = pytest.mark.gpu

FLOOR = 3e-6       # run_precision_suite.py:81, fp32 accumulation floor
LSE_TOL = 1e-3     # run_precision_suite.py:87


def _plan(name, seed):
    q16, k16, v16, bt, qs, kvs, T, (_, batch, _, H, KVH, q_len, _) = suite_inputs(name, seed)
    C = Hh.capi()
    desc = C.paged_desc(None, None, None, None, None, None, q_len,
                        shape=dict(num_tokens=T, num_heads=H, head_dim=128, num_blocks=k16.shape[0], block_size=128,
                                   kv_heads=KVH, batch=batch, block_cols=bt.shape[1]))
    p = C.plan(desc, q_len, False)
    return int(p.kernel), int(p.split_tokens)


@pytest.fixture(scope="module")
def oracle_results():
    items = []
    for c in CASES:
        for seed in SEEDS:
            kernel, split = _plan(c[0], seed)
            assert kernel == 0          # every suite shape has <= 16 rows per (request, kv head)
            items += [(c[0], seed, g, split) for g in range(c[4])]
    items.sort(key=lambda it: -sum(spec(it[0])[2]))   # biggest first: a short tail
    workers = max(1, min(len(items), os.cpu_count() or 1))
    with mp.get_context("spawn").Pool(workers) as pool:
        res = pool.map(oracle_head, items, chunksize=1)
    return {(n, s, g): (o, l, A) for n, s, g, o, l, A in res}


def _run_op(name, seed, fast):
    import torch
    npu = Hh.ops()
    q16, k16, v16, bt, qs, kvs, T, c = suite_inputs(name, seed)
    args = (Hh.bits_to_dev(q16), Hh.bits_to_dev(k16), Hh.bits_to_dev(v16), torch.from_numpy(bt).cuda(),
            torch.from_numpy(qs).cuda(), torch.from_numpy(kvs).cuda())
    out, lse = npu.fa_fp32_stage1(*args, c[5]) if fast else npu.fa_fp32_stage1(*args)
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_precision_suite_case(name, seed, oracle_results):
    Hh.need_cuda()
    C = Hh.capi()
    out, lse = _run_op(name, seed, fast=False)
    out_f, lse_f = _run_op(name, seed, fast=True)
    assert C.device_error() == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint32), out_f.cpu().numpy().view(np.uint32))
    assert np.array_equal(lse.cpu().numpy().view(np.uint32), lse_f.cpu().numpy().view(np.uint32))
    _, batch, kvs, H, KVH, q_len, _ = spec(name)
    T = batch * q_len
    o = Hh.dev_to_f64(out)
    l8 = Hh.dev_to_f64(lse).reshape(-1, 8)
    assert np.array_equal(l8, np.repeat(l8[:, :1], 8, axis=1)), "padded-LSE stride invariant"
    l = l8[:, 0].reshape(T, H)
    grp = H // KVH
    golden = np.load(os.path.join(GOLDEN, "precision_suite_golden.npz"))
    assert np.abs(l - golden[f"{name}|{seed}|lse"]).max() <= LSE_TOL
    worst = 0.0
    for g in range(KVH):
        o_ks, l_ks, A = oracle_results[(name, seed, g)]
        og = o[:, g * grp:(g + 1) * grp]
        excess = np.abs(og - o_ks) - (A + FLOOR)
        assert (excess <= 0).all(), f"kv head {g}: {int((excess > 0).sum())} beyond the tie band, worst {excess.max():.3g}"
        assert np.abs(l[:, g * grp:(g + 1) * grp] - l_ks).max() <= 1e-5
        assert (np.abs(og - o_ks) <= 2e-2 + 2e-2 * np.abs(o_ks)).all()
        worst = max(worst, float(np.abs(og - o_ks).max()))
    print(f"{name} seed{seed}: O maxAbs vs kernel-structured oracle {worst:.3e}")


def test_precision_suite_negative_checks():
    """run_precision_suite.py:93-138 at its own shape (4 requests x 4096 tokens,
    H=40/KVH=8): T != sum(q_seqlens), block_table cols too small, a kv length
    of 0 -- each rejected before launch with the op name in the message."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    q16, k16, v16, bt, qs, kvs, T, _ = suite_inputs("probe_shape_b4", 0)
    q, k, v = Hh.bits_to_dev(q16), Hh.bits_to_dev(k16), Hh.bits_to_dev(v16)
    dev = lambda a: torch.from_numpy(np.asarray(a)).cuda()
    cases = [
        (q[:-1], k, v, dev(bt), dev(qs), dev(kvs)),                                   # T mismatch
        (q, k, v, dev(bt[:, :1].copy()), dev(qs), dev(kvs)),                          # cols too small
        (q, k, v, dev(bt), dev(np.ones(4, np.int64)), dev(np.array([4096, 4096, 4096, 0]))),  # kv seqlen 0
    ]
    for args in cases:
        with pytest.raises(RuntimeError, match="fa_fp32_stage1"):
            npu.fa_fp32_stage1(*args)
            torch.cuda.synchronize()
