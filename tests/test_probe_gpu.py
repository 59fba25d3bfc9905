"""The HBM read-roof probe (cascade_probe_hbm_read) reads what it claims:
every probe folds the words it loads into its sink with XOR, so the XOR of
the sink is a checksum of exactly the bytes read. Mode 0 loads every word of
the buffer; mode 1 (bulk copies of 32 KB chunks) folds one word per KB of
every chunk; modes 2 and 3 (the decode's paged TMA pattern, row-major and
kv-head-major item order) sample the same words in a different order."""
import numpy as np
import pytest

import helpers as Hh

pytestmark = pytest.mark.gpu


def _sink_xor(sink):
    return int(np.bitwise_xor.reduce(sink.cpu().numpy().view(np.uint32)))


def test_probe_reads_every_byte_once():
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    g = torch.Generator(device="cuda").manual_seed(5)
    buf = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, device="cuda", generator=g)
    words = buf.view(torch.int32).cpu().numpy().view(np.uint32)
    res = {}
    for mode in range(4):
        sink = torch.zeros(2048, dtype=torch.int32, device="cuda")
        C.probe_hbm_read(buf, mode, 2048, sink)
        torch.cuda.synchronize()
        res[mode] = _sink_xor(sink)
    assert C.device_error() == 0
    # mode 0: every 32-bit word of the buffer
    assert res[0] == int(np.bitwise_xor.reduce(words))
    # mode 1: word lane * 256 of every 32 KB chunk (8192 words), lanes 0..31
    per_chunk = words.reshape(-1, 8192)[:, ::256]
    assert res[1] == int(np.bitwise_xor.reduce(per_chunk.reshape(-1)))
    # modes 2 and 3: the same items in another order
    assert res[2] == res[3] and res[2] != 0


def test_probe_rejects_bad_arguments():
    import torch
    Hh.need_cuda()
    C = Hh.capi()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(C.CascadeError, match="row_bytes"):
        C.probe_hbm_read(buf, 2, 300)
    with pytest.raises(C.CascadeError, match="mode must be"):
        C.probe_hbm_read(buf, 7)
    with pytest.raises(C.CascadeError, match="sink needs"):
        C.probe_hbm_read(buf, 0, 0, torch.zeros(16, dtype=torch.int32, device="cuda"))
