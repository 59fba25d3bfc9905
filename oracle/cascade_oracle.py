"""CPU oracle for the cascade-decode operator set -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA path in ``vllm-hust-cascade-kernel_b200`` never calls into it, and the
product ops fail loudly when the CUDA extension is missing.

It restates, in numpy fp64, the golden arithmetic of the reference
(``Raing5Days/vllm-hust-cascade-kernel``), citing the lines it follows:

* paged stage-1 / suffix attention: ``fa_fp64_ref``
  (ascend-kernel/csrc/ops/fa_fp32_stage1/test/fa_fp32_ref.py:82-126), page
  gather ``_gather_kv`` (same file :68-79), tie-band bound
  ``fa_fp64_ref_tieband`` (same file :150-206, bf16 neighbours :129-147);
* LSE merge: ``fp64_ref`` (ascend-kernel/csrc/ops/lse_merge/test/lse_merge_cases.py:45-50);
* SwiGLU gate_up: the intended mode-1 chain of
  ascend-kernel/csrc/ops/f3_floor/design.md:107-109 (the reference never
  implemented it): fp32 ``silu(gate) * up`` then RNE to bf16.

Extensions over the reference golden, each a documented superset:

* ``chunk`` (online-softmax step) and ``split`` (independent KV partitions
  merged in LSE space) describe the kernel's own quantisation structure; the
  reference semantics are ``chunk=512, split=None``;
* ``p_dtype='fp16'`` quantises P to fp16 for fp16 inputs (the reference kernel
  is bf16-only, fa_fp32_stage1.cpp:188-190);
* kv length 0 yields O = 0 and LSE = -inf (the reference golden raises on an
  empty concatenate); ``lse_merge_ref`` gives a -inf side zero weight.

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference's own
``fa_fp32_ref.py`` / ``lse_merge_cases.py`` in the build container and commits
their outputs; ``tests/test_oracle_golden.py`` checks this module against them.
"""

from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


# ---------------------------------------------------------------------------
# rounding helpers (RNE), own implementation on the IEEE bit patterns
# ---------------------------------------------------------------------------

def round_bf16(x):
    """Round fp32 values to the bf16 grid with round-to-nearest-even.

    Follows the quantisation point ``bf16(ls)`` of fa_fp32_ref.py:25-27 / :118.
    Input is rounded to fp32 first (the kernel's exps are fp32 values).
    Returns fp64 values on the bf16 grid."""
    x32 = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x32.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).astype(np.float64)
    if nan.any():
        out = np.where(nan, np.nan, out)
    return out


def round_fp16(x):
    """Round to the IEEE half grid (numpy's float16 cast is RNE)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float64)


def quantize(x, dtype):
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "fp16":
        return round_fp16(x)
    if dtype == "fp32":
        return np.asarray(x, dtype=np.float32).astype(np.float64)
    raise ValueError(dtype)


def ulp(x, dtype):
    """Spacing of the ``dtype`` grid at |x| (bf16: 8 significant bits,
    fp16: 11, fp32: 24), floored at the smallest normal spacing."""
    mant = {"bf16": 8, "fp16": 11, "fp32": 24}[dtype]
    emin = {"bf16": -126, "fp16": -14, "fp32": -126}[dtype]
    ax = np.maximum(np.abs(np.asarray(x, dtype=np.float64)), 2.0 ** emin)
    return 2.0 ** (np.floor(np.log2(ax)) - (mant - 1))


def bf16_bits(x):
    """fp32 array -> uint16 bf16 bit patterns (RNE)."""
    x32 = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x32.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def bf16_bits_to_f64(bits):
    u = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return u.view(np.float32).astype(np.float64)


def _neighbours(ls, dtype):
    """Nearest grid value and the two grid neighbours around ``ls``.

    Restates _bf16_round_and_neighbors (fa_fp32_ref.py:129-147) and extends it
    to fp16 (ulp from numpy.spacing on the half grid)."""
    if dtype == "bf16":
        x32 = np.asarray(ls, dtype=np.float32)
        u = x32.view(np.uint32).astype(np.uint64)
        rne = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000)
        p = rne.astype(np.uint32).view(np.float32).astype(np.float64)
        up = (rne + (1 << 16)).astype(np.uint32).view(np.float32).astype(np.float64)
        dn = (rne - (1 << 16)).astype(np.uint32).view(np.float32).astype(np.float64)
    else:
        h = np.asarray(ls, dtype=np.float32).astype(np.float16)
        p = h.astype(np.float64)
        up = np.nextafter(h, np.float16(np.inf)).astype(np.float64)
        dn = np.nextafter(h, np.float16(-np.inf)).astype(np.float64)
    g_hi = np.where(p < ls, up, p)
    g_lo = np.where(p < ls, p, dn)
    return p, g_lo, g_hi


# ---------------------------------------------------------------------------
# seeded inputs of the reference's precision suite
# ---------------------------------------------------------------------------

def gen_paged_inputs(batch, kv_seqlens, num_heads, kv_heads, embed=128, seed=0, q_len=1, block_cols=None,
                     share_blocks=False):
    """The seeded paged-KV inputs of the reference's precision suite.

    Restates gen_inputs (fa_fp32_stage1/test/fa_fp32_ref.py:30-60): one
    numpy default_rng(seed) draws K then V ([num_blocks, 128, KVH, D]) then
    Q ([batch*q_len, H, D]) from the standard normal in float32; block size
    128; share_blocks gives every request block ids 0..n-1 (the cascade's
    shared prefix), otherwise requests get consecutive distinct blocks.
    Returns (q, k, v float32, block_table int32, q_seqlens int64,
    kv_seqlens int64, num_tokens)."""
    rng = np.random.default_rng(seed)
    kv_seqlens = list(kv_seqlens)
    bs = 128
    pages = [(kv + bs - 1) // bs for kv in kv_seqlens]
    if block_cols is None:
        block_cols = max(pages)
    num_blocks = max(pages) if share_blocks else sum(pages)
    k = rng.standard_normal((num_blocks, bs, kv_heads, embed)).astype(np.float32)
    v = rng.standard_normal((num_blocks, bs, kv_heads, embed)).astype(np.float32)
    q = rng.standard_normal((batch * q_len, num_heads, embed)).astype(np.float32)
    bt = np.zeros((batch, block_cols), dtype=np.int32)
    nxt = 0
    for b, nb in enumerate(pages):
        if share_blocks:
            bt[b, :nb] = np.arange(nb, dtype=np.int32)
        else:
            bt[b, :nb] = np.arange(nxt, nxt + nb, dtype=np.int32)
            nxt += nb
    qs = np.full(batch, q_len, dtype=np.int64)
    return q, k, v, bt, qs, np.asarray(kv_seqlens, dtype=np.int64), int(qs.sum())


# ---------------------------------------------------------------------------
# paged attention (stage-1 shared prefix, and per-request suffix decode)
# ---------------------------------------------------------------------------

def gather_pages(pool, bt_row, kv):
    """One request's logical KV rows from the paged pool -> [kv, KVH, D].

    Restates _gather_kv (fa_fp32_ref.py:68-79): logical token t lives in page
    ``bt_row[t // bs]`` at in-page row ``t % bs``; bs = pool.shape[1]."""
    bs = pool.shape[1]
    if kv == 0:
        return np.zeros((0,) + pool.shape[2:], dtype=pool.dtype)
    nblk = (kv + bs - 1) // bs
    ids = np.asarray(bt_row[:nblk], dtype=np.int64)
    rows = pool[ids].reshape((nblk * bs,) + pool.shape[2:])
    return rows[:kv]


def _contiguous_segments(kv, split, chunk):
    """[(segment = list of chunk index arrays)] for contiguous splits."""
    if split is None or split <= 0 or split >= kv:
        bounds = [(0, kv)]
    else:
        bounds = [(s, min(kv, s + split)) for s in range(0, kv, split)]
    return [[np.arange(c0, min(s1, c0 + chunk)) for c0 in range(s0, s1, chunk)]
            for (s0, s1) in bounds]


def decode_segments(kv, split=256, tile=64, warps=4):
    """Token structure of the decode kernel (csrc/paged_decode.cu): a CTA owns
    ``split`` kv tokens, streamed in ``tile``-token stages; warp w of the CTA
    takes the w-th ``tile/warps`` tokens of every stage and runs its own online
    softmax over them one stage at a time.  Returns segments as lists of chunk
    index arrays (empty segments dropped)."""
    sub = tile // warps
    segs = []
    for s0 in range(0, kv, split):
        s1 = min(kv, s0 + split)
        for w in range(warps):
            chunks = []
            for t0 in range(s0, s1, tile):
                a = t0 + w * sub
                b = min(s1, a + sub)
                if a < b:
                    chunks.append(np.arange(a, b))
            if chunks:
                segs.append(chunks)
    return segs


def paged_attention_ref(q, k, v, block_table, q_seqlens, kv_seqlens, *,
                        chunk=512, split=None, segments=None, p_dtype="bf16", scale=None,
                        with_tieband=False, tie_band_rel=2e-5, tieband_rule="reference"):
    """fp64 paged attention with the reference kernel's quantisation points.

    Restates fa_fp64_ref (fa_fp32_ref.py:82-126): S = (q.k)*scale; online
    softmax over ``chunk``-token steps with running max hm, dm = exp(m_old-m);
    P = round(exp(S - m)) to ``p_dtype`` feeds P@V while the row sum gl adds
    the UNquantised exps; O = acc/gl; LSE = ln(gl) + m.  No mask: every query
    row of a request sees all of that request's kv tokens (the shared-prefix
    stage, fa_fp32_stage1.cpp:265).

    ``split`` (tokens) partitions each request's kv into independent segments
    whose online softmax starts afresh; the segments are merged exactly in LSE
    space -- the structure of a split-KV kernel.  ``split=None`` is the
    reference's single pass.  ``segments`` (a function kv -> list of segments,
    each an ordered list of chunk index arrays, e.g. ``decode_segments``)
    overrides chunk/split with an arbitrary token-to-segment assignment.

    q: [T,H,D]; k,v: [numBlocks, bs, KVH, D] (values already on the input grid).
    ``tieband_rule``: "reference" accumulates the near-tie bound exactly as
    fa_fp32_ref.py:199-200 (amb += dm * new_term), which is exact for a single
    chunk but can under-count flips of an earlier chunk once later chunks
    raise the running max; "rescaled" carries the bound like the accumulator
    (amb = dm * amb + new_term), the right rule for many small chunks.

    Returns (O [T,H,D] f64, LSE [T,H] f64[, A [T,H,D] tie-band bound]).
    kv == 0 -> O = 0, LSE = -inf."""
    q64 = np.asarray(q, dtype=np.float64)
    k64 = np.asarray(k, dtype=np.float64)
    v64 = np.asarray(v, dtype=np.float64)
    T, H, D = q64.shape
    KVH = k64.shape[2]
    group = H // KVH
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    O = np.zeros((T, H, D))
    LSE = np.full((T, H), -np.inf)
    A = np.zeros((T, H, D)) if with_tieband else None
    head_map = np.arange(H) // group
    tok = 0
    for b in range(len(q_seqlens)):
        ql = int(q_seqlens[b])
        kv = int(kv_seqlens[b])
        if ql == 0:
            continue
        if kv == 0:
            tok += ql
            continue
        kb = gather_pages(k64, block_table[b], kv)[:, head_map, :]  # [kv,H,D]
        vb = gather_pages(v64, block_table[b], kv)[:, head_map, :]
        qb = q64[tok:tok + ql].transpose(1, 0, 2)                   # [H,ql,D]
        S = np.einsum("htd,khd->htk", qb, kb) * scale
        seg_o, seg_l, seg_a = [], [], []
        segs = segments(kv) if segments is not None else _contiguous_segments(kv, split, chunk)
        for seg in segs:
            m = np.full((H, ql), -np.inf)
            gl = np.zeros((H, ql))
            acc = np.zeros((H, ql, D))
            amb = np.zeros((H, ql, D)) if with_tieband else None
            for ci, idx in enumerate(seg):
                sc = S[:, :, idx]
                m_new = np.maximum(m, sc.max(axis=2))
                dm = np.where(ci == 0, 1.0, np.exp(m - m_new))
                ls = np.exp(sc - m_new[:, :, None])
                if with_tieband:
                    p, g_lo, g_hi = _neighbours(ls, p_dtype)
                    mid = 0.5 * (g_lo + g_hi)
                    ambiguous = np.abs(ls - mid) <= tie_band_rel * ls
                    term = np.einsum("htk,khd->htd", ambiguous * (g_hi - g_lo), np.abs(vb[idx]))
                    if tieband_rule == "reference":
                        # fa_fp32_ref.py:199-200: the step's dm scales the new term
                        amb = amb + dm[:, :, None] * term
                    else:
                        amb = dm[:, :, None] * amb + term
                else:
                    p = quantize(ls, p_dtype)
                gl = dm * gl + ls.sum(axis=2)
                acc = dm[:, :, None] * acc + np.einsum("htk,khd->htd", p, vb[idx])
                m = m_new
            seg_o.append(acc / gl[:, :, None])
            seg_l.append(np.log(gl) + m)
            if with_tieband:
                seg_a.append(amb / gl[:, :, None])
        if len(seg_o) == 1:
            o_b, l_b = seg_o[0], seg_l[0]
            a_b = seg_a[0] if with_tieband else None
        else:
            L = np.stack(seg_l)                       # [nseg,H,ql]
            mx = L.max(axis=0)
            w = np.exp(L - mx[None])
            tot = w.sum(axis=0)
            o_b = np.einsum("shq,shqd->hqd", w, np.stack(seg_o)) / tot[:, :, None]
            l_b = mx + np.log(tot)
            a_b = (np.einsum("shq,shqd->hqd", w, np.stack(seg_a)) / tot[:, :, None]
                   if with_tieband else None)
        O[tok:tok + ql] = o_b.transpose(1, 0, 2)
        LSE[tok:tok + ql] = l_b.T
        if with_tieband:
            A[tok:tok + ql] = a_b.transpose(1, 0, 2)
        tok += ql
    if with_tieband:
        return O, LSE, A
    return O, LSE


def expand_lse_padded(lse_th, stride=8):
    """[T,H] -> flat [T*H*stride] with every (t,h) value replicated ``stride``
    times: the 32-byte padded LSE rows written by the reference stage-1 kernel
    (row index token*H + head, block_epilogue_rescale_o_no_split_row.hpp:408-414)."""
    flat = np.asarray(lse_th, dtype=np.float32).reshape(-1, 1)
    return np.repeat(flat, stride, axis=1).reshape(-1)


# ---------------------------------------------------------------------------
# LSE merge
# ---------------------------------------------------------------------------

def lse_merge_ref(o1, o2, l1, l2):
    """fp64 row-wise merge of two attention partials in LSE space.

    Restates fp64_ref (lse_merge_cases.py:45-50) and the kernel formula of
    kernel_lse_merge.cpp:16-20: m = max(l1,l2); w = exp(l - m);
    out = (o1*w1 + o2*w2) / (w1 + w2).  Extension: a side whose LSE is -inf
    has weight 0 (its O is not read, so 0*NaN cannot leak); both -inf -> 0.
    o*: [..., D]; l*: [...] (compact)."""
    o1 = np.asarray(o1, dtype=np.float64)
    o2 = np.asarray(o2, dtype=np.float64)
    l1 = np.asarray(l1, dtype=np.float64)
    l2 = np.asarray(l2, dtype=np.float64)
    m = np.maximum(l1, l2)
    both = np.isneginf(m)
    msafe = np.where(both, 0.0, m)
    with np.errstate(invalid="ignore"):
        w1 = np.where(np.isneginf(l1), 0.0, np.exp(l1 - msafe))
        w2 = np.where(np.isneginf(l2), 0.0, np.exp(l2 - msafe))
    a = np.where((w1 > 0)[..., None], o1, 0.0) * w1[..., None]
    b = np.where((w2 > 0)[..., None], o2, 0.0) * w2[..., None]
    den = (w1 + w2)[..., None]
    out = np.where(both[..., None], 0.0, (a + b) / np.where(den == 0, 1.0, den))
    lse = np.where(both, -np.inf, msafe + np.log(np.where(both, 1.0, w1 + w2)))
    return out, lse


# ---------------------------------------------------------------------------
# gate_up GEMM + SwiGLU
# ---------------------------------------------------------------------------

def gateup_ref(x, w, mode=1):
    """Gate/up projection with the f3_gateup_epilogue conventions.

    x: [M,K] values on the bf16 grid; w: [2I,K] (nn.Linear layout, gate rows
    [0,I), up rows [I,2I); f3_floor.cpp:18-21).  Returns fp64 arrays:
    mode 1 -> silu(gate)*up computed in fp32 then RNE bf16
    (f3_floor/design.md:107-109); mode 2 -> C = x@w^T rounded to bf16
    (the plain GEMM into the workspace, kernel_f3_floor.cpp:171-199)."""
    x32 = np.asarray(x, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    c = x32.astype(np.float64) @ w32.astype(np.float64).T
    I = w32.shape[0] // 2
    if mode == 2:
        return round_bf16(c)
    gate = c[:, :I].astype(np.float32)
    up = c[:, I:].astype(np.float32)
    silu = gate / (np.float32(1.0) + np.exp(-gate, dtype=np.float32))
    return round_bf16(silu * up)


def gateup_ref_fp64(x, w):
    """Unrounded fp64 silu(gate)*up (for error budgeting)."""
    c = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    I = c.shape[1] // 2
    g, u = c[:, :I], c[:, I:]
    return g / (1.0 + np.exp(-g)) * u


# ---------------------------------------------------------------------------
# one cascade decode step (stage-1 prefix + suffix + merge), as the reference's
# consumer composes it (ascend-kernel/README.md:158-201)
# ---------------------------------------------------------------------------

def cascade_step_ref(q, k, v, prefix_bt, group_sizes, prefix_lens, suffix_bt, suffix_lens, *,
                     p_dtype="bf16", out_dtype="bf16", kv_heads_subset=None, round_suffix=True):
    """fp64 cascade step.  q [B,H,D]; k/v [NB,bs,KVH,D] (grid values);
    prefix_bt [G,cols]; suffix_bt [B,cols].  Stage-1 flattens each prefix
    group's requests into one request of q_len = group size (README.md:174-177);
    the suffix runs per request with q_len 1; the merge follows
    lse_merge_cases.py:45-50.  ``kv_heads_subset`` restricts the computation
    to those kv heads (and their query heads).  ``round_suffix=False`` keeps
    the suffix partial unrounded (the single-combine step does not round it
    to the query dtype before merging).  Returns (out [B,H',D] rounded to
    out_dtype, lse [B,H'])."""
    q = np.asarray(q, np.float64)
    B, H, D = q.shape
    KVH = k.shape[2]
    group = H // KVH
    if kv_heads_subset is not None:
        heads = np.concatenate([np.arange(g * group, (g + 1) * group) for g in kv_heads_subset])
        q = q[:, heads]
        k = k[:, :, list(kv_heads_subset)]
        v = v[:, :, list(kv_heads_subset)]
    o1, l1 = paged_attention_ref(q, k, v, prefix_bt, np.asarray(group_sizes), np.asarray(prefix_lens),
                                 p_dtype=p_dtype)
    o2, l2 = paged_attention_ref(q, k, v, suffix_bt, np.ones(B, np.int64), np.asarray(suffix_lens),
                                 p_dtype=p_dtype)
    if round_suffix:
        o2 = quantize(o2, p_dtype)      # the suffix output is in the input dtype
    out, lse = lse_merge_ref(o1, o2, l1, l2)
    return quantize(out, out_dtype), lse
