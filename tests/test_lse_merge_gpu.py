"""GPU parity of lse_merge against the reference golden fixtures and the
oracle, with the reference's own thresholds (test_lse_merge_precision.py:16-66):
MERE / MARE per mode, abs bound 1e-5 (fp32 out) / 2e-2 (bf16 out)."""
import os

import numpy as np
import pytest

import helpers as Hh
from conftest import GOLDEN
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu

# mode -> (MERE tol, MARE tol, MARE floor)   lse_merge_cases.py:14-20
TOLS = {
    "A_tier0": (7.81e-3, 7.81e-2, 0.0),
    "B_fp32out": (1.22e-4, 1.22e-3, 1e-2),
    "Bp_fp32out_pad": (1.22e-4, 1.22e-3, 1e-2),
    "C_hybrid_bf16": (7.81e-3, 7.81e-2, 0.0),
}


def _metrics(out, ref, floor):
    rel = np.abs(out - ref) / (np.abs(ref) + 1e-7)
    if floor > 0:
        dom = np.abs(ref) >= floor
        mare = (rel * dom).max() if dom.any() else 0.0
    else:
        mare = rel.max()
    return rel.mean(), mare, np.abs(out - ref).max()


def _cases():
    z = np.load(os.path.join(GOLDEN, "lse_merge_cases.npz"))
    return z, sorted({k.rsplit("|", 1)[0] for k in z.files})


def _dev(arr):
    import torch
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(arr).cuda()


@pytest.mark.parametrize("key", _cases()[1])
def test_merge_golden(key):
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    z, _ = _cases()
    mode = key.split("|")[1]
    o1, o2 = _dev(z[key + "|o1"]), _dev(z[key + "|o2"])
    l1, l2 = _dev(z[key + "|l1"]), _dev(z[key + "|l2"])
    code = int(z[key + "|out_code"])
    out = npu.lse_merge(o1, o2, l1, l2, code)
    torch.cuda.synchronize()
    ref_f64 = z[key + "|ref"]
    # the reference compares against its fp64 golden cast to the output dtype
    ref = O.quantize(ref_f64, "bf16") if out.dtype == torch.bfloat16 else ref_f64.astype(np.float32)
    mere, mare, mabs = _metrics(Hh.dev_to_f64(out), ref.astype(np.float64), TOLS[mode][2])
    bound = 1e-5 if out.dtype == torch.float32 else 2e-2
    assert mere < TOLS[mode][0] and mare < TOLS[mode][1] and mabs < bound, (mere, mare, mabs)


def test_padded_lse_matches_compact_bitwise():
    """test_lse_merge_precision.py:80-93 on the production shape."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    T, H, D = 64, 40, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    o1 = torch.randn(T, H, D, device="cuda", generator=g).to(torch.bfloat16)
    o2 = torch.randn(T, H, D, device="cuda", generator=g).to(torch.bfloat16)
    l1 = torch.randn(T, H, device="cuda", generator=g)
    l2 = torch.randn(T, H, device="cuda", generator=g)
    l1p = l1.unsqueeze(-1).expand(T, H, 8).contiguous().reshape(T, H * 8)
    l2p = l2.unsqueeze(-1).expand(T, H, 8).contiguous().reshape(T, H * 8)
    a = npu.lse_merge(o1, o2, l1, l2, 2)
    b = npu.lse_merge(o1, o2, l1p, l2p, 2)
    assert torch.equal(a, b)


def test_out_code_validation_like_reference():
    """test_lse_merge_precision.py:69-77: out_code 3 and fp32 o2 are rejected
    by the reference op; the extended sibling accepts them."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    o1 = torch.randn(2, 4, 16, dtype=torch.bfloat16, device="cuda")
    o2 = torch.randn_like(o1)
    l1 = torch.randn(2, 4, dtype=torch.float32, device="cuda")
    l2 = torch.randn_like(l1)
    with pytest.raises(RuntimeError, match="lse_merge: out_code"):
        npu.lse_merge(o1, o2, l1, l2, 3)
    with pytest.raises(RuntimeError, match="lse_merge: o2 must be bf16"):
        npu.lse_merge(o1.float(), o2.float(), l1, l2)
    with pytest.raises(RuntimeError, match="head dim must be a multiple of 16"):
        npu.lse_merge(o1[..., :8].contiguous(), o2[..., :8].contiguous(), l1, l2)
    out = npu.cascade_lse_merge(o1.half(), o2.float(), l1, l2, 3)
    assert out.dtype == torch.float16


@pytest.mark.parametrize("o1_dt,o2_dt,code", [("fp32", "bf16", 1), ("fp32", "fp16", 3), ("bf16", "bf16", 0),
                                              ("fp32", "bf16", 2), ("fp16", "fp16", 2)])
def test_merge_neg_inf_and_mixed_dtypes(o1_dt, o2_dt, code):
    """-inf LSE sides (zero-length suffix / empty prefix) get zero weight, even
    when the other side's O holds NaN; matches the oracle."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    tmap = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
    T, H, D = 37, 8, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    o1 = torch.randn(T, H, D, device="cuda", generator=g).to(tmap[o1_dt])
    o2 = torch.randn(T, H, D, device="cuda", generator=g).to(tmap[o2_dt])
    l1 = torch.randn(T, H, device="cuda", generator=g) * 5
    l2 = torch.randn(T, H, device="cuda", generator=g) * 5
    l2[::3] = -float("inf")
    o2[::3] = float("nan")
    l1[::5] = -float("inf")
    l1p = l1.unsqueeze(-1).expand(T, H, 8).contiguous().reshape(-1)
    out = npu.cascade_lse_merge(o1, o2, l1p, l2.reshape(-1), code)
    torch.cuda.synchronize()
    ref, _ = O.lse_merge_ref(Hh.dev_to_f64(o1), Hh.dev_to_f64(o2), Hh.dev_to_f64(l1), Hh.dev_to_f64(l2))
    got = Hh.dev_to_f64(out)
    assert np.isfinite(got).all()
    dt = {torch.float32: "fp32", torch.bfloat16: "bf16", torch.float16: "fp16"}[out.dtype]
    tol = 1e-5 if dt == "fp32" else 0.5 * O.ulp(ref, dt) + 1e-6
    assert (np.abs(got - ref) <= tol).all()


def test_merge_capi_matches_op():
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    npu = Hh.ops()
    T, H, D = 64, 32, 128
    o1 = torch.randn(T, H, D, device="cuda")
    o2 = torch.randn(T, H, D, device="cuda").to(torch.bfloat16)
    l1 = torch.randn(T * H * 8, device="cuda")
    l2 = torch.randn(T * H, device="cuda")
    ref = npu.lse_merge(o1, o2, l1, l2, 1)
    out = torch.empty(T, H, D, device="cuda", dtype=torch.bfloat16)
    C.lse_merge(o1, o2, l1, 8, l2, 1, out, T * H, D)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
