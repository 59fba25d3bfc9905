"""CPU oracle for add_rms_norm_stats -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module; the CUDA op never calls into it.

Restates in numpy fp64 the reference's golden for the op
(ascend-kernel/csrc/ops/add_rms_norm_stats/test/add_rms_norm_stats_ref.py:130-156,
semantics in design.md section 1):

    x_out = round_dtype(x1 + x2)                    (mode 0 / 2; mode 1: x_out = x1)
    rstd  = 1 / sqrt(mean_k(x_out ** 2) + eps)      statistics of the ROUNDED value
    y     = round_dtype(round_dtype(x_out * rstd) * gamma + beta)      (mode 1)

and its acceptance rule, the mixed tolerance of the ops-precision standard
(same file :36-49 table, :92-133 metrics / verdict): per element
``|a - g| <= atol + rtol |g|``, matched ratio >= 0.99 and max abs error <=
max(fixed_limit, 32 ulp(1)).  Rounding to bf16 / fp16 goes through fp32
first, as torch's fp64 -> 16-bit conversion does.

Pinned by tests/test_rms_norm_oracle.py against fixtures produced by the
reference's own ``cpu_ref`` (tests/golden/make_golden.py) and against the
element records of the reference's device self-check
(test/f2_golden_selfcheck.json, extracted into
tests/golden/add_rms_norm_stats_selfcheck.json).
"""

from __future__ import annotations

import numpy as np

from .cascade_oracle import round_bf16, round_fp16

# add_rms_norm_stats_ref.py:36-44, keyed by the OUTPUT dtype
STD = {
    "fp16": {"atol": 2.0 ** -9, "rtol": 2.0 ** -9, "required_matched_ratio": 0.99, "fixed_limit": 1e-1,
             "ulp_at_one": 2.0 ** -10},
    "bf16": {"atol": 2.0 ** -6, "rtol": 2.0 ** -6, "required_matched_ratio": 0.99, "fixed_limit": 1e-0,
             "ulp_at_one": 2.0 ** -7},
    "fp32": {"atol": 2.0 ** -16, "rtol": 2.0 ** -10, "required_matched_ratio": 0.99, "fixed_limit": 1e-2,
             "ulp_at_one": 2.0 ** -23},
}
# add_rms_norm_stats_ref.py:50-53: CANN's own test tier, every element
CANN_TEST_TIER = {"bf16": (7.9345703125e-03, 7.9345703125e-03), "fp16": (1.0986328125e-03, 1.0986328125e-03)}


def _round(dtype):
    return round_bf16 if dtype == "bf16" else round_fp16


def add_rms_norm_stats_ref(x1, x2, gamma, beta, eps, mode, dtype):
    """(x_out, rstd, y) in fp64; x_out / y are None where ``mode`` does not
    produce them.  Inputs are fp64 arrays holding values of the ``dtype``
    grid: x1, x2 [M, K], gamma, beta [K] (beta may be None).  rstd is [M],
    rounded to fp32 like the reference's ``rstd.float()``."""
    q = _round(dtype)
    x1 = np.asarray(x1, dtype=np.float64)
    xo = x1 if mode == 1 else q(x1 + np.asarray(x2, dtype=np.float64))
    rstd = 1.0 / np.sqrt(np.mean(xo * xo, axis=-1) + eps)
    x_out = xo if mode == 0 else None
    y = None
    if mode == 1:
        mid = q(xo * rstd[:, None])
        acc = mid * np.asarray(gamma, dtype=np.float64)[None, :]
        if beta is not None:
            acc = acc + np.asarray(beta, dtype=np.float64)[None, :]
        y = q(acc)
    return x_out, rstd.astype(np.float32).astype(np.float64), y


def std_spec(out_dtype):
    """The standard's row for one output dtype with its abs-error ceiling
    (add_rms_norm_stats_ref.py:56-59)."""
    t = dict(STD[out_dtype])
    t["max_abs_error_limit"] = max(t["fixed_limit"], 32.0 * t["ulp_at_one"])
    return t


def metrics(out, ref, atol, rtol):
    """Element counts and errors of one output (ref = the fp64 side); refuses
    a shape-broadcast pairing like add_rms_norm_stats_ref.py:75-113."""
    a = np.asarray(out, dtype=np.float64).reshape(-1)
    b = np.asarray(ref, dtype=np.float64).reshape(-1)
    if a.size != b.size:
        raise ValueError(f"element count mismatch {a.size} vs {b.size}")
    d = np.abs(a - b)
    n_viol = int((d > atol + rtol * np.abs(b)).sum())
    return {"n_el": a.size, "n_viol": n_viol, "matched_ratio": 1.0 - n_viol / max(a.size, 1),
            "MaxAbsErr": float(d.max()) if a.size else 0.0}


def verdict(m, spec):
    """The standard's two-part rule (add_rms_norm_stats_ref.py:116-133)."""
    return m["matched_ratio"] >= spec["required_matched_ratio"] and m["MaxAbsErr"] <= spec["max_abs_error_limit"]
