"""Bounded waits end a stalled pipeline with an error status, not a hang.

Each case runs an attention kernel with CASCADE_FLAG_DEBUG_STALL: its
consumer warps first wait on an mbarrier that nothing ever completes, with a
1 ms limit. The wait runs out, the CTA raises its abort flag, every other
wait of the CTA returns at once, producers stop issuing and wait (bounded)
for their copies in flight, an MMA issuer waits for its last MMAs, TMEM is
freed and the kernel exits. The checks: the call returns promptly, bit 1 of
the device error word is set, and the context is still usable -- the same
call without the flag gives the same result as before and a clean error word.
No case faults, traps or hangs a GPU: the stalled wait is an ordinary
bounded mbarrier wait on a barrier of the CTA's own shared memory.
Also: the debug mode that reads the block table back before launching
(CASCADE_FLAG_CHECK_BLOCK_IDS) accepts valid tables and changes nothing; the
rejection of bad ids is covered on the CPU (no kernel ever sees one here).
"""
import time

import numpy as np
import pytest

import helpers as Hh

pytestmark = pytest.mark.gpu


def _inputs(seed, B, kv_max, H, KVH, bs=128, q_len=1, kv_typ=None, shared=False):
    import torch
    rng = np.random.default_rng(seed)
    kv = rng.integers(1, (kv_typ or kv_max) + 1, size=B)
    kv[0] = kv_max
    pages = [(int(k) + bs - 1) // bs for k in kv]
    n = (max(pages) if shared else sum(pages)) + 1
    bt = np.zeros((B, max(pages)), np.int32)
    perm = rng.permutation(n).astype(np.int32)
    c = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[:pages[b]] if shared else perm[c:c + pages[b]]
        c += pages[b]
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B * q_len, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(n, bs, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(n, bs, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    i64 = dict(dtype=torch.int64, device="cuda")
    return (q, k, v, torch.from_numpy(bt).cuda(), torch.full((B,), q_len, **i64),
            torch.from_numpy(kv).to(**i64))


def _call(args, q_len, suffix, flags):
    import torch
    C = Hh.capi()
    q = args[0]
    desc = C.paged_desc(*args, q_len, flags=flags)
    T, H, D = q.shape
    if suffix:
        out = torch.empty((T, H, D), dtype=q.dtype, device="cuda")
        lse = torch.empty((T * H,), dtype=torch.float32, device="cuda")
        n = C.suffix_workspace_size(desc)
    else:
        out = torch.empty((T, H, D), dtype=torch.float32, device="cuda")
        lse = torch.empty((T * H * 8,), dtype=torch.float32, device="cuda")
        n = C.stage1_workspace_size(desc)
    ws = torch.empty((max(n, 1),), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    (C.suffix_decode if suffix else C.fa_fp32_stage1)(desc, out, lse, ws)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return out, lse, C.device_error(), dt, C.plan(desc, q_len, suffix).kernel


CASES = {
    # per-item suffix decode (kernel 0): 16 requests x 8 kv heads, up to 1024 tokens
    "decode": (dict(seed=1, B=16, kv_max=1024, H=32, KVH=8), 1, True, 0),
    # planned suffix decode (kernel 2): 256 requests x 8 kv heads over a 4608-token table
    "planned": (dict(seed=2, B=256, kv_max=4608, H=8, KVH=8, kv_typ=400), 1, True, 2),
    # stage-1 on tcgen05 (kernel 1): 2 requests of 64 query tokens x 4 heads per kv head, 2048 tokens
    "stage1": (dict(seed=3, B=2, kv_max=2048, H=8, KVH=2, q_len=64, shared=True), 64, False, 1),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_stalled_wait_aborts_and_context_survives(name):
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    kw, q_len, suffix, kernel = CASES[name]
    args = _inputs(**kw)
    ref_out, ref_lse, err0, _, k = _call(args, q_len, suffix, 0)
    assert err0 == 0 and k == kernel
    _, _, err, dt, _ = _call(args, q_len, suffix, C.FLAG_DEBUG_STALL)
    assert err & 1, "the stalled wait did not run out"
    # every CTA gives up after ~1 ms (a wave of CTAs at a time) and drains in
    # microseconds: far below the 100 ms default limit of one wait per CTA
    assert dt < 5.0, dt
    out, lse, err2, _, _ = _call(args, q_len, suffix, 0)
    assert err2 == 0
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)


def test_block_id_check_mode_accepts_valid_tables():
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    kw, q_len, suffix, _ = CASES["decode"]
    args = _inputs(**kw)
    ref_out, _, _, _, _ = _call(args, q_len, suffix, 0)
    out, _, err, _, _ = _call(args, q_len, suffix, C.FLAG_CHECK_BLOCK_IDS)
    assert err == 0
    assert torch.equal(out, ref_out)
