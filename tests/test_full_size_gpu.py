"""The cascade step at the full sizes of the BASELINE configs, with the seeds
bench.py times: the Llama-3-8B step (C2: 64 requests sharing a 4096-token
prefix, suffix U[128,1024], 32/8 heads), the Llama-3-70B-shaped step (C4: 4
prefix groups x 64 requests, 16384-token prefixes, suffix U[256,2048], 64/8
heads) and the ragged stress case (C5: 32 groups, lognormal prefixes up to
32768 tokens, block size 16, fp16, GQA 5, zero-length suffixes).

Checks: the fused single-combine step and the reference consumer's three-op
chain agree to within the chain's extra rounding (plus, on C2 and C4, the
P-rounding structure of the fused step's own stage-1 pieces: prefix-first
splits, or two segments around the suffix decode) and are finite; the CPU
oracle of the whole step, run on EVERY kv head (one spawned worker per kv
head), matches the fused step at the BASELINE tolerance (2e-2) and at one
output ulp plus the P-rounding structure slack."""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["c2", "c4", "c5"])
def test_full_size_step(name):
    import torch
    from cascade_kernel import workloads
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    w = workloads.CONFIGS[name](seed=0)     # the seed bench.py times
    t = w.tables
    dt = "fp16" if w.q.dtype == torch.float16 else "bf16"
    fused = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=True)
    chain = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=False)
    o2, _ = torch.ops.npu.cascade_suffix_decode(w.q, w.k_pool, w.v_pool, t.suffix_block_table,
                                                t.suffix_q_seqlens, t.suffix_kv_seqlens, 1)
    torch.cuda.synchronize()
    assert Hh.capi().device_error() == 0
    a, b = Hh.dev_to_f64(fused), Hh.dev_to_f64(chain)
    assert np.isfinite(a).all() and np.isfinite(b).all()
    # the chain rounds the suffix partial once more; on C2 the fused step also
    # runs stage-1 with its prefix-first splits (fewer, longer than the
    # standalone op's), and on C4 with its two segments around the suffix
    # decode (other piece boundaries), which moves where P is rounded: the
    # structure slack
    slack = 2e-3 if name in ("c2", "c4") else 1e-7
    bound = O.ulp(np.maximum(np.abs(a), np.abs(b)), dt) + 0.5 * O.ulp(Hh.dev_to_f64(o2), dt) + slack
    assert (np.abs(a - b) <= bound).all(), float((np.abs(a - b) - bound).max())

    # the oracle on every kv head
    ref, ref_lse = Hh.step_oracle_all_heads(w, out_dtype="fp32", round_suffix=False)
    np.testing.assert_allclose(a, ref, atol=2e-2, rtol=2e-2)
    err = np.abs(a - ref)
    assert (err <= O.ulp(ref, dt) + 2e-3).all(), float((err - O.ulp(ref, dt)).max())
    print(f"{name}: max |out - oracle| {err.max():.3e} over {a.size} outputs, all kv heads")


def test_full_size_c4_shard_of_two_ranks():
    """Rank 0's shard of C4 over 2 ranks (4 kv heads / 32 q heads, tables
    replicated), the shard bench.py's strong-scaling block runs on each GPU:
    its step takes the overlapped stage-1 with a 864-tile segment A and 16-tile
    segment-B runs. The fused step and the three-op chain agree within the
    chain's extra rounding plus the stage-1 structure slack, and the fused
    step matches the CPU oracle on every kv head of the shard."""
    import torch
    from cascade_kernel import sharding, workloads
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    w = workloads.c4_llama70b(seed=0)
    w.q, w.k_pool, w.v_pool = sharding.shard_attention(w.q, w.k_pool, w.v_pool, 0, 2)
    t = w.tables
    fused = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=True)
    chain = cascade_decode(w.q, w.k_pool, w.v_pool, t, fused=False)
    o2, _ = torch.ops.npu.cascade_suffix_decode(w.q, w.k_pool, w.v_pool, t.suffix_block_table,
                                                t.suffix_q_seqlens, t.suffix_kv_seqlens, 1)
    torch.cuda.synchronize()
    assert Hh.capi().device_error() == 0
    a, b = Hh.dev_to_f64(fused), Hh.dev_to_f64(chain)
    assert np.isfinite(a).all() and np.isfinite(b).all()
    bound = O.ulp(np.maximum(np.abs(a), np.abs(b)), "bf16") + 0.5 * O.ulp(Hh.dev_to_f64(o2), "bf16") + 2e-3
    assert (np.abs(a - b) <= bound).all(), float((np.abs(a - b) - bound).max())
    ref, _ = Hh.step_oracle_all_heads(w, out_dtype="fp32", round_suffix=False)
    np.testing.assert_allclose(a, ref, atol=2e-2, rtol=2e-2)
    err = np.abs(a - ref)
    assert (err <= O.ulp(ref, "bf16") + 2e-3).all(), float((err - O.ulp(ref, "bf16")).max())
