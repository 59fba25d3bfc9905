"""Generate the committed golden fixtures from the reference's OWN golden code.

Run where a checkout of the reference is available (read-only is enough):

    python tests/golden/make_golden.py <reference checkout> [stage1 merge norm precision]

It imports, unmodified, the reference's CPU goldens
  * ascend-kernel/csrc/ops/fa_fp32_stage1/test/fa_fp32_ref.py
    (gen_inputs, fa_fp64_ref, fa_fp64_ref_tieband)
  * ascend-kernel/csrc/ops/lse_merge/test/lse_merge_cases.py
    (make_inputs, fp64_ref, boundary_cases)
  * ascend-kernel/csrc/ops/add_rms_norm_stats/test/add_rms_norm_stats_cases.py
    and add_rms_norm_stats_ref.py (make_inputs, cpu_ref)
runs them on small seeded cases and writes their inputs/outputs to
``tests/golden/*.npz``.  For the reference's precision suite
(fa_fp32_stage1/test/run_precision_suite.py:19-37: 15 shapes x seeds 0, 1,
read from that file's text because it imports the NPU runtime) it stores,
per case and seed, a SHA-256 fingerprint of the inputs the reference's own
gen_inputs draws (bf16 q/k/v bytes, block table, seqlens) and the fp64
golden's LSE and per-row O sums (fa_fp64_ref), so the full-size inputs can
be regenerated on the GPU box by the restated generator and checked there.  It also copies, from the reference's device
self-check record add_rms_norm_stats/test/f2_golden_selfcheck.json, the
per-element dumps (row, col, fp64 golden, CANN's value and rstd, gamma) and
the per-case error statistics into
``tests/golden/add_rms_norm_stats_selfcheck.json``.  The GPU box never reads the reference; the tests read
only these fixtures.  Case shapes are scaled-down members of the reference's
own case lists (run_precision_suite.py:19-36, test_lse_flatten_regression.py:31-47,
lse_merge_cases.py:14-70) so the fixtures stay small.
"""

import os
import sys
import zlib

import numpy as np


def stage1_cases():
    # (name, batch, kv_seqlens, H, KVH, q_len, block_cols_extra, share_blocks, permute)
    return [
        ("min_b1_kv128", 1, [128], 8, 2, 1, 0, True, False),
        ("kv_448_tail", 3, [448] * 3, 8, 2, 1, 0, True, False),
        ("varlen_3req", 3, [129, 640, 1024], 4, 1, 1, 0, False, False),
        ("qlen2_b4", 4, [384] * 4, 8, 2, 2, 0, True, False),
        ("h2_kvh1", 4, [512] * 4, 2, 1, 1, 0, True, False),
        ("padded_block_cols", 2, [300, 700], 4, 1, 1, 3, False, False),
        ("flat_T17_g5", 1, [600], 5, 1, 17, 0, True, False),
        ("flat_T64_g4", 1, [1100], 4, 1, 64, 0, True, False),
        ("b8_kvh1_g8", 8, [256] * 8, 8, 1, 1, 0, True, False),
        ("perm_table_varlen", 5, [77, 513, 1, 260, 1030], 4, 1, 1, 1, False, True),
    ]


def make_stage1(ref_dir, out_dir):
    sys.path.insert(0, os.path.join(ref_dir, "ascend-kernel/csrc/ops/fa_fp32_stage1/test"))
    import fa_fp32_ref as R  # the reference's own golden module

    for (name, batch, kvs, H, KVH, qlen, extra, share, permute) in stage1_cases():
        seed = zlib.crc32(name.encode()) % 2**31
        cols = None if extra == 0 else max((kv + 127) // 128 for kv in kvs) + extra
        q, k, v, bt, qs, kvarr, T = R.gen_inputs(batch, kvs, H, KVH, 128, seed=seed,
                                               q_len=qlen, block_cols=cols,
                                               share_blocks=share)
        if permute:
            # random-permutation physical pages; the
            # reference golden accepts any table (fa_fp32_ref.py:68-79)
            rng = np.random.default_rng(seed + 1)
            perm = rng.permutation(k.shape[0]).astype(np.int32)
            used = bt.copy()
            for b in range(batch):
                nb = (kvs[b] + 127) // 128
                used[b, :nb] = perm[bt[b, :nb]]
            bt = used
        q16, k16, v16 = R.to_bf16_bytes(q), R.to_bf16_bytes(k), R.to_bf16_bytes(v)
        qf, kf, vf = (x.astype(np.float64) for x in (q16, k16, v16))
        o, lse = R.fa_fp64_ref(qf, kf, vf, bt, qs, kvarr, 128, H, KVH)
        o_t, lse_t, A = R.fa_fp64_ref_tieband(qf, kf, vf, bt, qs, kvarr, 128, H, KVH)
        # the tie-band variant recomputes the same O/LSE; store its bound only
        assert np.array_equal(o_t, o) and np.array_equal(lse_t, lse)
        np.savez_compressed(
            os.path.join(out_dir, f"stage1_{name}.npz"),
            q_bits=q16.view(np.uint16), k_bits=k16.view(np.uint16), v_bits=v16.view(np.uint16),
            block_table=bt, q_seqlens=qs, kv_seqlens=kvarr,
            H=H, KVH=KVH, q_len=qlen,
            o_ref=o, lse_ref=lse, A_tb=A.astype(np.float32))
        print("stage1", name, "T", T, "blocks", k.shape[0])


def precision_suite_cases(ref_dir):
    """CASES and SEEDS of run_precision_suite.py, parsed from its text (never
    executed): literals, lists/tuples of them and list * int."""
    import ast

    def value(n):
        if isinstance(n, ast.Constant):
            return n.value
        if isinstance(n, (ast.List, ast.Tuple)):
            items = [value(e) for e in n.elts]
            return items if isinstance(n, ast.List) else tuple(items)
        if isinstance(n, ast.BinOp) and isinstance(n.op, ast.Mult):
            a, b = value(n.left), value(n.right)
            if isinstance(a, list) and isinstance(b, int):
                return a * b
        raise ValueError(f"unexpected expression in the case list: {ast.dump(n)[:80]}")

    path = os.path.join(ref_dir, "ascend-kernel/csrc/ops/fa_fp32_stage1/test/run_precision_suite.py")
    tree = ast.parse(open(path).read())
    found = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            if node.targets[0].id in ("CASES", "SEEDS"):
                found[node.targets[0].id] = value(node.value)
    return found["CASES"], found["SEEDS"]


def input_fingerprint(q16, k16, v16, bt, qs, kvs):
    import hashlib
    h = hashlib.sha256()
    for a in (q16.view(np.uint16), k16.view(np.uint16), v16.view(np.uint16), np.asarray(bt, np.int32),
              np.asarray(qs, np.int64), np.asarray(kvs, np.int64)):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def make_precision_suite(ref_dir, out_dir):
    import json
    sys.path.insert(0, os.path.join(ref_dir, "ascend-kernel/csrc/ops/fa_fp32_stage1/test"))
    import fa_fp32_ref as R  # the reference's own golden module
    cases, seeds = precision_suite_cases(ref_dir)
    out, meta = {}, {"source": "ascend-kernel/csrc/ops/fa_fp32_stage1/test/run_precision_suite.py:19-37",
                     "fields": ["name", "batch", "kv_seqlens", "H", "KVH", "q_len", "block_cols_extra"],
                     "cases": [list(c) for c in cases], "seeds": list(seeds), "sha256": {}}
    for (name, batch, kvs, H, KVH, qlen, extra) in cases:
        for seed in seeds:
            # exactly as run_case() draws them (run_precision_suite.py:47-51)
            cols = None if extra == 0 else max((kv + 127) // 128 for kv in kvs) + extra
            q, k, v, bt, qs, kvarr, T = R.gen_inputs(batch, kvs, H, KVH, 128, seed=seed, q_len=qlen,
                                                   block_cols=cols, share_blocks=True)
            q16, k16, v16 = R.to_bf16_bytes(q), R.to_bf16_bytes(k), R.to_bf16_bytes(v)
            key = f"{name}|{seed}"
            meta["sha256"][key] = input_fingerprint(q16, k16, v16, bt, qs, kvarr)
            o, lse = R.fa_fp64_ref(q16.astype(np.float64), k16.astype(np.float64), v16.astype(np.float64),
                                   bt, qs, kvarr, 128, H, KVH)
            out[key + "|lse"] = lse
            out[key + "|o_rowsum"] = o.sum(axis=2)
            print("precision suite", key, "T", T, "blocks", k.shape[0])
    np.savez_compressed(os.path.join(out_dir, "precision_suite_golden.npz"), **out)
    with open(os.path.join(out_dir, "precision_suite.json"), "w") as f:
        json.dump(meta, f, indent=1)


def make_merge(ref_dir, out_dir):
    import torch
    sys.path.insert(0, os.path.join(ref_dir, "ascend-kernel/csrc/ops/lse_merge/test"))
    import lse_merge_cases as C  # the reference's own case module
    C.DEV = "cpu"                # the module only uses DEV as a .to() target

    shapes = [("tiny", (7, 4, 16)), ("odd-rows", (13, 4, 128)), ("single-row", (1, 8, 128))]
    modes = ["A_tier0", "B_fp32out", "Bp_fp32out_pad", "C_hybrid_bf16"]
    out = {}
    for cat, (T, H, D) in shapes:
        for mode in modes:
            o1_dtype, _, out_code, padded, *_ = C.MODES[mode]
            seed = zlib.crc32(f"{cat}/{mode}".encode()) % 2**31
            o1, o2, l1c, l2c, l1, l2 = C.make_inputs(T, H, D, o1_dtype, padded, seed=seed)
            ref = C.fp64_ref(o1, o2, l1, l2)
            key = f"{cat}|{mode}"
            out[key + "|o1"] = (o1.view(torch.int16).numpy().view(np.uint16)
                                if o1.dtype == torch.bfloat16 else o1.numpy())
            out[key + "|o2"] = o2.view(torch.int16).numpy().view(np.uint16)
            out[key + "|l1"] = l1c.numpy()
            out[key + "|l2"] = l2c.numpy()
            out[key + "|out_code"] = np.int64(out_code)
            out[key + "|ref"] = ref.numpy()
    # boundary mutators on a reduced production-like shape
    T, H, D = 2, 8, 128
    for bname, bfn in C.boundary_cases():
        for mode in ["B_fp32out", "C_hybrid_bf16"]:
            o1_dtype, _, out_code, padded, *_ = C.MODES[mode]
            o1, o2, l1c, l2c, l1, l2 = C.make_inputs(T, H, D, o1_dtype, padded,
                                                     seed=zlib.crc32(bname.encode()) % 2**31)
            bfn(o1, o2, l1, l2)
            ref = C.fp64_ref(o1, o2, l1, l2)
            key = f"boundary-{bname}|{mode}"
            out[key + "|o1"] = o1.numpy()
            out[key + "|o2"] = o2.view(torch.int16).numpy().view(np.uint16)
            out[key + "|l1"] = l1.numpy()
            out[key + "|l2"] = l2.numpy()
            out[key + "|out_code"] = np.int64(out_code)
            out[key + "|ref"] = ref.numpy()
    np.savez_compressed(os.path.join(out_dir, "lse_merge_cases.npz"), **out)
    print("lse_merge", len(out) // 6, "cases")


def norm_cases():
    # scaled-down members of add_rms_norm_stats_cases.py:21-30 (same boundary kinds)
    return [("odd-rows-77", (77, 128)), ("k-min", (7, 16)), ("single-row", (1, 5120)),
            ("k-not-pow2", (3, 5008)), ("k-2048", (5, 2048))]


def make_norm(ref_dir, out_dir):
    import json
    import torch
    tdir = os.path.join(ref_dir, "ascend-kernel/csrc/ops/add_rms_norm_stats/test")
    sys.path.insert(0, tdir)
    import add_rms_norm_stats_cases as C  # the reference's own case module
    import add_rms_norm_stats_ref as R    # the reference's own golden
    C.DEV = "cpu"                          # the module only uses DEV as a .to() target
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    out = {}
    for dtype, dname in ((torch.bfloat16, "bf16"), (torch.float16, "fp16")):
        for name, (m, k) in norm_cases():
            for mode in (0, 1, 2):
                for has_beta in ((False, True) if mode == 1 else (False,)):
                    seed = zlib.crc32(f"norm/{dname}/{name}/{mode}/{has_beta}".encode()) % 2**31
                    x1, x2, gamma, beta = C.make_inputs(m, k, dtype, seed, has_beta)
                    x_out, rstd, y = R.cpu_ref(x1, x2, gamma, beta, 1e-6, mode)
                    key = f"{dname}|{name}|{mode}|{int(has_beta)}"
                    out[key + "|x1"] = bits(x1)
                    out[key + "|x2"] = bits(x2)
                    out[key + "|gamma"] = bits(gamma)
                    if beta is not None:
                        out[key + "|beta"] = bits(beta)
                    out[key + "|rstd"] = rstd.reshape(-1).numpy()
                    if x_out is not None:
                        out[key + "|x_out"] = bits(x_out)
                    if y is not None:
                        out[key + "|y"] = bits(y)
    np.savez_compressed(os.path.join(out_dir, "add_rms_norm_stats_cases.npz"), **out)
    sc = json.load(open(os.path.join(tdir, "f2_golden_selfcheck.json")))
    keep = {"source": "add_rms_norm_stats/test/f2_golden_selfcheck.json (reference device run: "
                      + sc["env"] + ", " + sc["date"] + ")",
            "eps": 1e-6, "mode": 1, "has_beta": False,
            "seed_rule": "zlib.crc32(f'golden/{torch_dtype}/{case}') % 2**31 "
                         "(run_golden_selfcheck.py dump_strict_violations)",
            "element_dumps": [{"dtype": r["dtype"], "case": r["case"], "shape": r["shape"],
                               "elements": [{f: e[f] for f in ("row", "col", "ref", "cann", "rstd_cann", "gamma")}
                                            for e in r["elements"]]}
                              for r in sc["violating_element_dumps"]],
            "cases": [{"dtype": c["dtype"], "case": c["case"], "shape": c["shape"],
                       "cann_vs_ref": c["checks"]["cann_vs_ref"], "ours_vs_ref": c["checks"]["ours_vs_ref"]}
                      for c in sc["cases"]]}
    with open(os.path.join(out_dir, "add_rms_norm_stats_selfcheck.json"), "w") as f:
        json.dump(keep, f, indent=1)
    print("add_rms_norm_stats", len(norm_cases()) * 8, "cases")


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout> [stage1 merge norm precision]")
    ref_dir = sys.argv[1]
    out_dir = os.path.dirname(os.path.abspath(__file__))
    only = sys.argv[2:]  # optional subset: stage1 merge norm precision
    if not only or "stage1" in only:
        make_stage1(ref_dir, out_dir)
    if not only or "merge" in only:
        make_merge(ref_dir, out_dir)
    if not only or "norm" in only:
        make_norm(ref_dir, out_dir)
    if not only or "precision" in only:
        make_precision_suite(ref_dir, out_dir)


if __name__ == "__main__":
    main()
