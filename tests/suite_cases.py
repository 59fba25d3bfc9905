"""The reference's fa_fp32_stage1 precision-suite cases and their inputs.

CASES and SEEDS are run_precision_suite.py:19-37 of
ascend-kernel/csrc/ops/fa_fp32_stage1/test, verbatim (name, batch,
kv_seqlens, H, KVH, q_len, block_cols_extra); every case is generated with
share_blocks=True as run_case() does (:47-51). ``suite_inputs`` draws them
with the restated generator oracle.gen_paged_inputs, which
tests/test_precision_suite_cpu.py pins against fingerprints of the
reference's own gen_inputs."""
from oracle import cascade_oracle as O

CASES = [
    # (name, batch, kv_seqlens, H, KVH, q_len, block_cols_extra)
    ("main_14b_b64",      64, [8192] * 64, 40, 8, 1, 0),
    ("probe_shape_b4",    4,  [4096] * 4,  40, 8, 1, 0),
    ("b16_h32",           16, [4096] * 16, 32, 8, 1, 0),
    ("b8_h8_kvh1",        8,  [2048] * 8,  8,  1, 1, 0),
    ("b32_kv8192",        32, [8192] * 32, 40, 8, 1, 0),
    ("min_b1_kv128",      1,  [128],       40, 8, 1, 0),
    ("kv_448_tail",       3,  [448] * 3,    40, 8, 1, 0),
    ("varlen_3req",       3,  [129, 640, 1024], 40, 8, 1, 0),
    ("qlen2_b4",          4,  [2048] * 4,   40, 8, 2, 0),
    ("b7_kv4096",         7,  [4096] * 7,   40, 8, 1, 0),
    ("b2_kv16384",        2,  [16384] * 2,  40, 8, 1, 0),
    ("b64_kv128",         64, [128] * 64,   40, 8, 1, 0),
    ("h2_kvh1",           4,  [512] * 4,    2,  1, 1, 0),
    ("padded_block_cols", 4,  [4096] * 4,   40, 8, 1, 3),
    ("varlen_6req",       6,  [4095, 2048, 8192, 512, 128, 4096], 40, 8, 1, 0),
]

SEEDS = [0, 1]


def spec(name):
    for c in CASES:
        if c[0] == name:
            return c
    raise KeyError(name)


def suite_inputs(name, seed):
    """(q16, k16, v16 uint16 bf16 bits, block_table, q_seqlens, kv_seqlens, T, case)."""
    c = spec(name)
    _, batch, kvs, H, KVH, q_len, extra = c
    cols = None if extra == 0 else max((kv + 127) // 128 for kv in kvs) + extra
    q, k, v, bt, qs, kvarr, T = O.gen_paged_inputs(batch, kvs, H, KVH, 128, seed=seed, q_len=q_len,
                                                   block_cols=cols, share_blocks=True)
    return O.bf16_bits(q), O.bf16_bits(k), O.bf16_bits(v), bt, qs, kvarr, T, c


def oracle_head(item):
    """Kernel-structured oracle of one kv head of one suite case: the decode
    kernel's 16-token chunks per warp and its ``split``-token KV splits, with
    the tie-band bound. item = (name, seed, kv head, split). A process-pool
    worker: returns (name, seed, head, O [T, group, D], LSE [T, group], A)."""
    name, seed, g, split = item
    q16, k16, v16, bt, qs, kvs, T, (_, _, _, H, KVH, _, _) = suite_inputs(name, seed)
    grp = H // KVH
    q = O.bf16_bits_to_f64(q16)[:, g * grp:(g + 1) * grp]
    k = O.bf16_bits_to_f64(k16[:, :, g:g + 1])
    v = O.bf16_bits_to_f64(v16[:, :, g:g + 1])
    o, l, A = O.paged_attention_ref(q, k, v, bt, qs, kvs, with_tieband=True, tieband_rule="rescaled",
                                    segments=lambda n: O.decode_segments(n, split=split, tile=64, warps=4))
    return name, seed, g, o, l, A
