"""The cascade step at the full sizes of the BASELINE configs that the bench
does not time: the Llama-3-70B-shaped shard (4 prefix groups x 64 requests,
16384-token prefixes, suffix U[256,2048], 64/8 heads) and the ragged stress
case (32 groups, lognormal prefixes up to 32768 tokens, block size 16, fp16,
GQA 5, zero-length suffixes).

Size-independent checks at full size: the fused single-combine step and the
reference consumer's three-op chain agree to within the chain's extra
rounding; both are finite. The oracle, which is too slow for every head at
these sizes, checks one kv head (all requests, all pages) at the BASELINE
tolerance and at one output ulp plus the P-rounding structure slack."""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["c4", "c5"])
def test_full_size_step(name):
    import torch
    from cascade_kernel import workloads
    from cascade_kernel.cascade import cascade_decode
    Hh.need_cuda()
    w = workloads.CONFIGS[name](seed=5)
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
    bound = O.ulp(np.maximum(np.abs(a), np.abs(b)), dt) + 0.5 * O.ulp(Hh.dev_to_f64(o2), dt) + 1e-7
    assert (np.abs(a - b) <= bound).all(), float((np.abs(a - b) - bound).max())

    # oracle on kv head 0: its q heads, its slice of the pools
    H, KVH = w.q.shape[1], w.k_pool.shape[2]
    group = H // KVH
    f64 = lambda x: x.float().cpu().numpy().astype(np.float64)
    ref, _ = O.cascade_step_ref(f64(w.q[:, :group]), f64(w.k_pool[:, :, :1]), f64(w.v_pool[:, :, :1]),
                                t.prefix_block_table.cpu().numpy(), w.group_sizes, w.prefix_lens,
                                t.suffix_block_table.cpu().numpy(), w.suffix_lens, p_dtype=dt, out_dtype="fp32",
                                round_suffix=False)
    got = a[:, :group]
    np.testing.assert_allclose(got, ref, atol=2e-2, rtol=2e-2)
    err = np.abs(got - ref)
    assert (err <= O.ulp(ref, dt) + 2e-3).all(), float((err - O.ulp(ref, dt)).max())
