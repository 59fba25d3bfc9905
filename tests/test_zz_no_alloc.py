"""The allocation-free suffix decode entry point (cascade_suffix_decode_noalloc).

It exists for callers that cannot allocate device memory when they run the
attention step (a host binding the C ABI without a device allocator, or a
serving loop whose memory is fixed up front); it keeps its split-KV partials in
a fixed 16 MiB scratch array inside the library. These checks call it through
the C ABI and compare it with the allocating entry point, cascade_suffix_decode,
on several different calls in a row (each reuses the scratch the one before
left behind), cover both the per-item decode and the planned decode (whose
scratch also holds the device-built item list and its counters), and check
that oversized or per-request-q-length calls are refused before anything runs.

Ordering: pytest collects test files in name order, and this file's name puts
it last, so a run that stops at the first failure (``-x``) has already run every
other test when a failure here stops it. Nothing here depends on that order:
the first call on a device looks up the scratch array's address whether or not
other tests ran before, and the file passes alone in a fresh process as well
as after the rest of the suite.
"""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu


def _case(seed, B, kv_max, H=32, KVH=8, bs=128, kv_typ=None):
    """Seeded suffix-decode inputs: kv lengths U[0, kv_typ or kv_max], the
    first request at kv_max (so the block table spans kv_max tokens)."""
    import torch
    rng = np.random.default_rng(seed)
    kv = rng.integers(0, (kv_typ or kv_max) + 1, size=B)
    kv[0] = kv_max                      # at least one request uses every split
    pages = [(int(k) + bs - 1) // bs for k in kv]
    n = sum(pages) + 1
    perm = rng.permutation(n).astype(np.int32)
    bt = np.zeros((B, max(pages)), np.int32)
    c = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[c:c + pages[b]]
        c += pages[b]
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(n, bs, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(n, bs, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    i64 = dict(dtype=torch.int64, device="cuda")
    return (q, k, v, torch.from_numpy(bt).cuda(), torch.ones(B, **i64), torch.from_numpy(kv).to(**i64))


def _noalloc(args):
    import torch
    C = Hh.capi()
    q = args[0]
    desc = C.paged_desc(*args, 1)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[0] * q.shape[1], dtype=torch.float32, device="cuda")
    C.suffix_decode_noalloc(desc, out, lse)
    torch.cuda.synchronize()
    assert C.device_error() == 0
    return out, lse


def test_noalloc_matches_allocating_entry_on_two_calls():
    Hh.need_cuda()
    C = Hh.capi()
    # three different problems, all split into several KV partials: two take
    # the per-item decode, the third (256 requests x 8 kv heads over a
    # 4608-token block table) the planned decode, whose scratch also holds
    # the item list, its count and the per-kv-head counters
    cases = [_case(11, B=64, kv_max=1024), _case(12, B=40, kv_max=768, H=40),
             _case(13, B=256, kv_max=4608, H=8, KVH=8, kv_typ=600)]
    kernels = []
    for args in cases:
        desc = C.paged_desc(*args, 1)
        assert C.suffix_workspace_size(desc) > 0       # the scratch is really used
        kernels.append(C.plan(desc, 1, True).kernel)
        ref_out, ref_lse = Hh.run_capi_paged(*args, 1, suffix=True)
        out, lse = _noalloc(args)
        o, r = Hh.dev_to_f64(out), Hh.dev_to_f64(ref_out)
        # same kernels, same plan: within the suffix tests' bound (half a bf16
        # ulp), in practice bit-identical
        assert (np.abs(o - r) <= 0.5 * O.ulp(r, "bf16") + 1e-6).all()
        l, lr = Hh.dev_to_f64(lse), Hh.dev_to_f64(ref_lse)
        fin = np.isfinite(lr)
        assert np.array_equal(np.isneginf(l), np.isneginf(lr))
        assert np.abs(l[fin] - lr[fin]).max() <= 1e-5
    assert kernels == [0, 0, 2]


def test_noalloc_refuses_oversized_and_legacy_calls():
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    small = _case(14, B=4, kv_max=300)
    out = torch.full_like(small[0], 3.0)
    lse = torch.empty(small[0].shape[0] * small[0].shape[1], dtype=torch.float32, device="cuda")
    # 512 requests x 32 heads x several splits of 4096 tokens x 516 B > 16 MiB; the
    # size check runs on the shapes before anything is launched
    big = C.paged_desc(None, None, None, None, None, None, 1,
                       shape=dict(num_tokens=512, num_heads=32, head_dim=128, num_blocks=1, block_size=128,
                                  kv_heads=8, batch=512, block_cols=32))
    assert C.suffix_workspace_size(big) > (16 << 20)
    with pytest.raises(C.CascadeError, match="above the fixed"):
        C.suffix_decode_noalloc(big, out, lse)
    torch.cuda.synchronize()
    assert torch.all(out == 3.0)                       # nothing ran
    d = C.paged_desc(*small, 0)
    with pytest.raises(C.CascadeError, match="q_seqlen_value > 0"):
        C.suffix_decode_noalloc(d, out, lse)
