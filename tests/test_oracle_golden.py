"""Pin the CPU oracle against the reference's own golden outputs (no GPU).

The fixtures under tests/golden/ were produced by running the reference's
fa_fp32_ref.py / lse_merge_cases.py (see tests/golden/make_golden.py)."""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import cascade_oracle as O

STAGE1 = sorted(glob.glob(os.path.join(GOLDEN, "stage1_*.npz")))


def load_stage1(path):
    z = np.load(path)
    q = O.bf16_bits_to_f64(z["q_bits"])
    k = O.bf16_bits_to_f64(z["k_bits"])
    v = O.bf16_bits_to_f64(z["v_bits"])
    return z, q, k, v


def test_fixtures_present():
    assert len(STAGE1) >= 10
    assert os.path.exists(os.path.join(GOLDEN, "lse_merge_cases.npz"))


@pytest.mark.parametrize("path", STAGE1, ids=[os.path.basename(p)[7:-4] for p in STAGE1])
def test_stage1_oracle_matches_reference_golden(path):
    z, q, k, v = load_stage1(path)
    o, lse, a = O.paged_attention_ref(q, k, v, z["block_table"], z["q_seqlens"],
                                      z["kv_seqlens"], chunk=512, with_tieband=True)
    np.testing.assert_allclose(o, z["o_ref"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(lse, z["lse_ref"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(a, z["A_tb"], rtol=1e-6, atol=1e-12)


def test_stage1_split_equals_unsplit_without_quantisation():
    """Split-KV merged in LSE space is exact when P is not quantised."""
    z, q, k, v = load_stage1(os.path.join(GOLDEN, "stage1_varlen_3req.npz"))
    args = (q, k, v, z["block_table"], z["q_seqlens"], z["kv_seqlens"])
    o1, l1 = O.paged_attention_ref(*args, chunk=128, p_dtype="fp32")
    o2, l2 = O.paged_attention_ref(*args, chunk=64, split=192, p_dtype="fp32")
    np.testing.assert_allclose(o1, o2, rtol=0, atol=1e-6)
    np.testing.assert_allclose(l1, l2, rtol=0, atol=1e-12)


def test_stage1_kernel_structure_within_reference_tolerance():
    """The kernel-structured oracle (128-token steps, split KV) stays well inside
    the reference tolerance of the reference-structured one."""
    z, q, k, v = load_stage1(os.path.join(GOLDEN, "stage1_perm_table_varlen.npz"))
    args = (q, k, v, z["block_table"], z["q_seqlens"], z["kv_seqlens"])
    o, l = O.paged_attention_ref(*args, chunk=128, split=256)
    assert np.abs(o - z["o_ref"]).max() < 2e-3
    assert np.abs(l - z["lse_ref"]).max() < 1e-6


def test_kv_zero_contract():
    rng = np.random.default_rng(0)
    k = O.round_bf16(rng.standard_normal((2, 16, 1, 128)))
    q = O.round_bf16(rng.standard_normal((2, 2, 128)))
    bt = np.array([[0], [1]], np.int32)
    o, l = O.paged_attention_ref(q, k, k, bt, [1, 1], [0, 5])
    assert np.all(o[0] == 0) and np.all(np.isneginf(l[0]))
    assert np.all(np.isfinite(l[1]))


def test_merge_oracle_matches_reference_golden():
    z = np.load(os.path.join(GOLDEN, "lse_merge_cases.npz"))
    keys = sorted({k.rsplit("|", 1)[0] for k in z.files})
    assert len(keys) >= 20
    for key in keys:
        o1 = z[key + "|o1"]
        o1 = O.bf16_bits_to_f64(o1) if o1.dtype == np.uint16 else o1.astype(np.float64)
        o2 = O.bf16_bits_to_f64(z[key + "|o2"])
        rows = o1.size // o1.shape[-1]
        l1 = z[key + "|l1"].reshape(rows, -1)[:, 0].reshape(o1.shape[:-1])
        l2 = z[key + "|l2"].reshape(rows, -1)[:, 0].reshape(o1.shape[:-1])
        out, _ = O.lse_merge_ref(o1, o2, l1, l2)
        np.testing.assert_allclose(out, z[key + "|ref"], rtol=1e-13, atol=1e-13, err_msg=key)


def test_merge_neg_inf_sides():
    o1 = np.ones((3, 16))
    o2 = np.full((3, 16), 2.0)
    o2[1] = np.nan  # a -inf side's O is never read
    l1 = np.array([0.0, 0.0, -np.inf])
    l2 = np.array([-np.inf, -np.inf, -np.inf])
    out, lse = O.lse_merge_ref(o1, o2, l1, l2)
    assert np.all(out[0] == 1) and np.all(out[1] == 1) and np.all(out[2] == 0)
    assert lse[0] == 0 and np.isneginf(lse[2])


def test_bf16_rounding_matches_ml_dtypes():
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(100000) * 10.0 ** rng.integers(-8, 8, 100000)).astype(np.float32)
    ref = x.astype(ml.bfloat16).astype(np.float64)
    np.testing.assert_array_equal(O.round_bf16(x), ref)
    np.testing.assert_array_equal(O.bf16_bits(x), x.astype(ml.bfloat16).view(np.uint16))


def test_swiglu_oracle_small():
    rng = np.random.default_rng(2)
    x = O.round_bf16(rng.standard_normal((4, 64)))
    w = O.round_bf16(rng.standard_normal((2 * 32, 64)) * 0.02)
    d = O.gateup_ref(x, w, mode=1)
    exact = O.gateup_ref_fp64(x, w)
    assert d.shape == (4, 32)
    assert np.abs(d - exact).max() <= 2 ** -8 * np.abs(exact).max() + 1e-6
