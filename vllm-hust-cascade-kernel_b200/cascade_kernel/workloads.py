"""Seeded synthetic cascade-decode workloads with the benchmark shapes.

The reference publishes no dataset for this path; these generators stand in
for it with the shapes and value distributions of the benchmark configs:
q/k/v ~ N(0,1) in bf16 (fp16 for the ragged and CPU-golden configs), block
tables that are random permutations of the physical pages, suffix lengths
drawn from the stated distributions with a fixed seed.

Every generator returns a ``Workload`` whose tensors live on ``device``.
"""
from dataclasses import dataclass, field

import numpy as np
import torch

from .cascade import CascadeTables


@dataclass
class Workload:
    name: str
    q: torch.Tensor                 # [B, H, 128]
    k_pool: torch.Tensor            # [NB, bs, KVH, 128]
    v_pool: torch.Tensor
    tables: CascadeTables
    group_sizes: list               # requests per prefix group
    prefix_lens: list               # prefix tokens per group
    suffix_lens: np.ndarray         # suffix tokens per request
    meta: dict = field(default_factory=dict)

    @property
    def batch(self):
        return self.q.shape[0]

    def kv_token_bytes(self):
        """K+V bytes of one token of one layer (all kv heads)."""
        return 2 * self.k_pool.shape[2] * self.k_pool.shape[3] * self.k_pool.element_size()

    def algorithmic_bytes(self, out_elem=2):
        """Bytes a cascade step must move at minimum: prefix KV once per group,
        suffix KV once, q read by both stages, the fp32 stage-1 partial and its
        padded LSE written+read, the suffix partial and LSE written+read, and
        the merged output written."""
        B, H, D = self.q.shape
        qb = self.q.numel() * self.q.element_size()
        kvb = self.kv_token_bytes()
        stage1 = qb + sum(self.prefix_lens) * kvb + B * H * D * 4 + B * H * 8 * 4
        suffix = qb + int(self.suffix_lens.sum()) * kvb + B * H * D * self.q.element_size() + B * H * 4
        merge = B * H * D * 4 + B * H * D * self.q.element_size() + B * H * 8 * 4 + B * H * 4 \
            + B * H * D * out_elem
        return {"stage1": stage1, "suffix": suffix, "merge": merge, "total": stage1 + suffix + merge}

    def flops(self):
        B, H, D = self.q.shape
        pre = sum(4 * g * (H) * p * D for g, p in zip(self.group_sizes, self.prefix_lens))
        suf = int(4 * H * D * self.suffix_lens.sum())
        return {"stage1": pre, "suffix": suf, "total": pre + suf}


def _pages(n, bs):
    return (n + bs - 1) // bs


def make_cascade(name, *, group_sizes, prefix_lens, suffix_lens, H, KVH, bs, dtype, seed,
                 device="cuda", extra_pages=0):
    """Build a cascade workload: prefix groups with shared pages, per-request
    suffix pages, all placed in one pool by a random permutation."""
    rng = np.random.default_rng(seed)
    G = len(group_sizes)
    B = int(sum(group_sizes))
    suffix_lens = np.asarray(suffix_lens, dtype=np.int64)
    assert suffix_lens.shape == (B,)
    pre_pages = [_pages(p, bs) for p in prefix_lens]
    suf_pages = [_pages(int(s), bs) for s in suffix_lens]
    n_pages = sum(pre_pages) + sum(suf_pages) + extra_pages
    perm = rng.permutation(n_pages).astype(np.int32)
    cursor = 0
    cols_p = max(1, max(pre_pages))
    bt_p = np.zeros((G, cols_p), np.int32)
    for g in range(G):
        bt_p[g, :pre_pages[g]] = perm[cursor:cursor + pre_pages[g]]
        cursor += pre_pages[g]
    cols_s = max(1, max(suf_pages))
    bt_s = np.zeros((B, cols_s), np.int32)
    for b in range(B):
        bt_s[b, :suf_pages[b]] = perm[cursor:cursor + suf_pages[b]]
        cursor += suf_pages[b]

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    D = 128
    k_pool = torch.randn((max(n_pages, 1), bs, KVH, D), generator=gen, device=device,
                         dtype=torch.float32).to(dtype)
    v_pool = torch.randn((max(n_pages, 1), bs, KVH, D), generator=gen, device=device,
                         dtype=torch.float32).to(dtype)
    q = torch.randn((B, H, D), generator=gen, device=device, dtype=torch.float32).to(dtype)
    uniform = group_sizes[0] if all(g == group_sizes[0] for g in group_sizes) else 0
    i64 = dict(dtype=torch.int64, device=device)
    tables = CascadeTables(
        prefix_block_table=torch.from_numpy(bt_p).to(device),
        prefix_q_seqlens=torch.tensor(list(group_sizes), **i64),
        prefix_kv_seqlens=torch.tensor(list(prefix_lens), **i64),
        suffix_block_table=torch.from_numpy(bt_s).to(device),
        suffix_q_seqlens=torch.ones(B, **i64),
        suffix_kv_seqlens=torch.from_numpy(suffix_lens).to(device),
        uniform_group=int(uniform),
    )
    return Workload(name, q, k_pool, v_pool, tables, list(group_sizes), list(prefix_lens), suffix_lens,
                    meta=dict(H=H, KVH=KVH, bs=bs, dtype=str(dtype).replace("torch.", ""), seed=seed,
                              pages=n_pages))


def c1_cpu_golden(device="cuda", seed=0):
    """4 requests sharing a 512-token prefix, suffix U[64,256], H=8/KVH=2, bs=128, fp16."""
    rng = np.random.default_rng(seed)
    suf = rng.integers(64, 257, size=4)
    return make_cascade("c1_cpu_golden", group_sizes=[4], prefix_lens=[512], suffix_lens=suf, H=8, KVH=2,
                        bs=128, dtype=torch.float16, seed=seed, device=device)


def c2_llama8b(device="cuda", seed=0, kv_heads=8, heads=32):
    """Llama-3-8B cascade decode: B=64, prefix 4096, suffix U[128,1024], H=32/KVH=8, bs=128, bf16."""
    rng = np.random.default_rng(seed)
    suf = rng.integers(128, 1025, size=64)
    return make_cascade("c2_llama3_8b_cascade", group_sizes=[64], prefix_lens=[4096], suffix_lens=suf,
                        H=heads, KVH=kv_heads, bs=128, dtype=torch.bfloat16, seed=seed, device=device)


def c4_llama70b(device="cuda", seed=0, kv_heads=8, heads=64):
    """Llama-3-70B attention: 4 groups x 64 requests, prefix 16384, suffix U[256,2048], H=64/KVH=8."""
    rng = np.random.default_rng(seed)
    suf = rng.integers(256, 2049, size=256)
    return make_cascade("c4_llama3_70b_cascade", group_sizes=[64] * 4, prefix_lens=[16384] * 4,
                        suffix_lens=suf, H=heads, KVH=kv_heads, bs=128, dtype=torch.bfloat16, seed=seed,
                        device=device)


def c5_ragged(device="cuda", seed=0):
    """Ragged: 32 groups (16 requests each), prefix lognormal(median 1024, sigma 1)
    clipped to [16, 32768]; suffix lognormal(median 200, sigma 1) with 5% zeros;
    H=40/KVH=8, bs=16, fp16."""
    rng = np.random.default_rng(seed)
    pre = np.clip(np.rint(rng.lognormal(np.log(1024), 1.0, size=32)), 16, 32768).astype(int)
    suf = np.clip(np.rint(rng.lognormal(np.log(200), 1.0, size=512)), 1, 32768).astype(np.int64)
    suf[rng.random(512) < 0.05] = 0
    return make_cascade("c5_ragged", group_sizes=[16] * 32, prefix_lens=list(pre), suffix_lens=suf, H=40,
                        KVH=8, bs=16, dtype=torch.float16, seed=seed, device=device)


CONFIGS = {"c1": c1_cpu_golden, "c2": c2_llama8b, "c4": c4_llama70b, "c5": c5_ragged}
