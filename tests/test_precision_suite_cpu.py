"""The reference's fa_fp32_stage1 precision suite, CPU side (no CUDA).

The suite (ascend-kernel/csrc/ops/fa_fp32_stage1/test/run_precision_suite.py:
19-37) is 15 shapes x seeds {0, 1}; its inputs come from the reference's
gen_inputs (fa_fp32_ref.py:30-60). tests/golden/make_golden.py ran the
reference's own generator and fp64 golden for all 30 cases in the build
container and stored an input fingerprint plus the golden LSE and per-row O
sums. Here: the case list in the GPU test is the reference's, the restated
generator (oracle.gen_paged_inputs) draws bit-identical inputs for every case,
and the oracle reproduces the golden on the cases small enough for a CPU test.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import cascade_oracle as O
from suite_cases import CASES, SEEDS, suite_inputs


def _meta():
    return json.load(open(os.path.join(GOLDEN, "precision_suite.json")))


def _fingerprint(q16, k16, v16, bt, qs, kvs):
    h = hashlib.sha256()
    for a in (q16, k16, v16, np.asarray(bt, np.int32), np.asarray(qs, np.int64), np.asarray(kvs, np.int64)):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_case_list_is_the_references():
    m = _meta()
    assert [list(c) for c in CASES] == [[c[0], c[1], list(c[2]), c[3], c[4], c[5], c[6]] for c in m["cases"]]
    assert list(SEEDS) == m["seeds"]
    assert len(CASES) == 15 and len(SEEDS) == 2


@pytest.mark.parametrize("case", [c[0] for c in CASES])
def test_restated_generator_matches_reference_inputs(case):
    m = _meta()
    for seed in SEEDS:
        q16, k16, v16, bt, qs, kvs, T, spec = suite_inputs(case, seed)
        assert _fingerprint(q16, k16, v16, bt, qs, kvs) == m["sha256"][f"{case}|{seed}"]


SMALL = ["min_b1_kv128", "kv_448_tail", "varlen_3req", "h2_kvh1", "b64_kv128", "qlen2_b4", "b8_h8_kvh1"]


@pytest.mark.parametrize("case", SMALL)
def test_oracle_reproduces_reference_golden(case):
    g = np.load(os.path.join(GOLDEN, "precision_suite_golden.npz"))
    for seed in SEEDS:
        q16, k16, v16, bt, qs, kvs, T, spec = suite_inputs(case, seed)
        o, lse = O.paged_attention_ref(O.bf16_bits_to_f64(q16), O.bf16_bits_to_f64(k16), O.bf16_bits_to_f64(v16),
                                       bt, qs, kvs)
        assert np.abs(lse - g[f"{case}|{seed}|lse"]).max() <= 1e-12
        assert np.abs(o.sum(axis=2) - g[f"{case}|{seed}|o_rowsum"]).max() <= 1e-9
