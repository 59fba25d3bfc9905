"""Host-side checks of the paging contract (no CUDA calls).

A block table row r may only name pages in [0, num_blocks) for the
ceil(kv_r / block_size) pages request r reads; entries past that are never
read and may hold anything. The reference guards the contract statically
(ascend-kernel/csrc/ops/fa_fp32_stage1/op_kernel/kernel_fa_fp32_stage1.cpp:107-112).
Here ``cascade_check_block_table`` checks a host copy and names the first bad
entry; the kernels themselves replace a bad id by a zero-filled page and set a
device error bit, but no test launches a kernel with bad ids: these cases run
on the CPU against the host checker only.
"""
import numpy as np
import pytest


def _capi():
    from cascade_kernel import capi
    capi.load()
    return capi


def _table(seed=0, rows=6, bs=16, num_blocks=200):
    rng = np.random.default_rng(seed)
    kv = rng.integers(0, 300, size=rows).astype(np.int64)
    kv[0] = 0
    cols = int(max(1, ((kv + bs - 1) // bs).max()))
    bt = np.full((rows, cols), -7, np.int32)           # unread entries hold garbage on purpose
    perm = rng.permutation(num_blocks).astype(np.int32)
    c = 0
    for r in range(rows):
        n = (int(kv[r]) + bs - 1) // bs
        bt[r, :n] = perm[c:c + n]
        c += n
    return bt, kv, bs, num_blocks


def test_valid_table_passes_and_unread_entries_are_ignored():
    C = _capi()
    bt, kv, bs, nb = _table()
    C.check_block_table(bt, kv, bs, nb)               # -7 past each row's pages is never read


@pytest.mark.parametrize("bad", [-1, 200, 2 ** 31 - 1])
def test_out_of_range_id_is_named(bad):
    C = _capi()
    bt, kv, bs, nb = _table()
    r = int(np.argmax(kv))
    col = int((kv[r] - 1) // bs)                       # the row's last page
    bt[r, col] = bad
    with pytest.raises(C.CascadeError, match=r"outside \[0, num_blocks=200\)") as e:
        C.check_block_table(bt, kv, bs, nb)
    assert e.value.bad == (r, col)
    assert e.value.code == C.ERR_INVALID


def test_first_bad_entry_in_row_order():
    C = _capi()
    bt, kv, bs, nb = _table(seed=3)
    rows = [r for r in range(len(kv)) if kv[r] > 0]
    bt[rows[-1], 0] = nb
    bt[rows[1], 0] = -5
    with pytest.raises(C.CascadeError) as e:
        C.check_block_table(bt, kv, bs, nb)
    assert e.value.bad == (rows[1], 0)


def test_kv_longer_than_table_is_rejected():
    C = _capi()
    bt, kv, bs, nb = _table()
    kv = kv.copy()
    kv[2] = bt.shape[1] * bs + 1
    with pytest.raises(C.CascadeError, match="columns") as e:
        C.check_block_table(bt, kv, bs, nb)
    assert e.value.bad == (2, bt.shape[1])


def test_zero_length_rows_read_nothing():
    C = _capi()
    bt = np.full((3, 2), 10 ** 6, np.int32)
    C.check_block_table(bt, np.zeros(3, np.int64), 128, 4)
