"""Host logic of the cascade step graph that needs no GPU: how
CascadeLayersGraph(overlap_io=True) groups the steps' host copies."""
import itertools

import pytest

from cascade_kernel.cascade import copy_groups


def test_copy_groups_bench_layout():
    # 20 steps over 8 layer buffers: 1, 2, then 4 steps, the last step alone
    assert copy_groups([i % 8 for i in range(20)], 4) == [[0], [1, 2], [3, 4, 5, 6], [7, 8, 9, 10],
                                                          [11, 12, 13, 14], [15, 16, 17, 18], [19]]


def test_copy_groups_small_cases():
    assert copy_groups([0], 4) == [[0]]
    assert copy_groups([], 4) == []
    assert copy_groups([0, 1, 0, 1], 4) == [[0], [1], [2], [3]]      # 2 buffers -> groups of 1
    assert copy_groups([0, 1, 2, 3, 0, 1, 2, 3, 0], 4) == [[0], [1, 2], [3, 4], [5, 6], [7], [8]]
    assert copy_groups([i % 8 for i in range(10)], 1) == [[i] for i in range(10)]


@pytest.mark.parametrize("n_buf,n_steps,io_group",
                         list(itertools.product([1, 2, 3, 5, 8, 16], [1, 2, 7, 20, 33], [1, 2, 4, 8])))
def test_copy_groups_invariants(n_buf, n_steps, io_group):
    """Every step exactly once and in order; no buffer twice in a group; no
    group above min(io_group, n_buf // 2) (but at least 1); the first and the
    last group hold one step."""
    bufs = [(7 * i) % n_buf for i in range(n_steps)]
    g = copy_groups(bufs, io_group)
    assert [i for grp in g for i in grp] == list(range(n_steps))
    limit = max(1, min(io_group, n_buf // 2))
    for grp in g:
        assert 1 <= len(grp) <= limit
        assert len({bufs[i] for i in grp}) == len(grp)
    assert len(g[0]) == 1 and len(g[-1]) == 1


def test_reference_arm_inputs_equal_the_workload():
    """bench.py's reference arm builds the C2 inputs without the repo's package
    (so none of our native libraries load there); its restated recipe must
    give the workload our arm times, value for value."""
    import torch
    import bench
    from cascade_kernel import workloads
    a = bench.reference_c2_inputs(seed=0, device="cpu")
    b = workloads.c2_llama8b(seed=0, device="cpu")
    for x, y in ((a.q, b.q), (a.k_pool, b.k_pool), (a.v_pool, b.v_pool),
                 (a.tables.prefix_block_table, b.tables.prefix_block_table),
                 (a.tables.suffix_block_table, b.tables.suffix_block_table)):
        assert torch.equal(x, y.cpu())
    assert (a.suffix_lens == b.suffix_lens).all()
    assert a.algorithmic_bytes()["total"] == b.algorithmic_bytes()["total"]
