"""GPU parity of the gate_up GEMM + SwiGLU epilogue (f3_gateup_epilogue modes
and the fused cascade_gateup_swiglu op) against the CPU oracle (small shapes)
and a torch fp32 reference (benchmark shapes).

Tolerance: the kernel accumulates in fp32 (tensor cores) and rounds the
SwiGLU result once to bf16, so every output must lie within one bf16 ulp of
the oracle's fp32-epilogue value (plus 1e-6 absolute for values near zero);
that also satisfies the BASELINE bound atol = rtol = 2e-2.
"""
import numpy as np
import pytest

import helpers as Hh
from oracle import cascade_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(M, K, I, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return x, w


def _within_one_ulp(d, ref):
    bound = O.ulp(ref, "bf16") + 1e-6
    err = np.abs(d - ref)
    assert (err <= bound).all(), f"max excess {(err - bound).max():.3e} at {np.unravel_index(np.argmax(err - bound), err.shape)}"


@pytest.mark.parametrize("M", [1, 16, 30, 37, 128, 130, 256])
def test_swiglu_small_vs_oracle(M):
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    K, I = 320, 384
    x, w = _inputs(M, K, I, seed=M)
    d = npu.cascade_gateup_swiglu(x, w)
    torch.cuda.synchronize()
    ref = O.gateup_ref(Hh.dev_to_f64(x), Hh.dev_to_f64(w), mode=1)
    _within_one_ulp(Hh.dev_to_f64(d), ref)
    exact = O.gateup_ref_fp64(Hh.dev_to_f64(x), Hh.dev_to_f64(w))
    np.testing.assert_allclose(Hh.dev_to_f64(d), exact, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("mode", [0, 2, 4])
def test_f3_modes_write_c_and_windows(mode):
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    M, K, I = 64, 256, 256
    x, w = _inputs(M, K, I, seed=10 + mode)
    d, ws = npu.f3_gateup_epilogue(x, w, None, None, mode)
    torch.cuda.synchronize()
    cref = O.gateup_ref(Hh.dev_to_f64(x), Hh.dev_to_f64(w), mode=2)
    _within_one_ulp(Hh.dev_to_f64(ws), cref)
    if mode == 0:
        assert torch.equal(d, ws[:, :I])
    if mode == 4:
        assert torch.equal(d, ws[:, I:])


def test_f3_mode1_inplace_gate_half():
    """f3_floor/design.md:102: D written in place over the gate half of the
    workspace (row stride 2I)."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    M, K, I = 32, 128, 128
    x, w = _inputs(M, K, I, seed=3)
    ws = torch.zeros(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    d, ws2 = npu.f3_gateup_epilogue(x, w, ws, ws[:, :I], 1)
    torch.cuda.synchronize()
    assert d.stride(0) == 2 * I and ws2.data_ptr() == ws.data_ptr()
    ref = O.gateup_ref(Hh.dev_to_f64(x), Hh.dev_to_f64(w), mode=1)
    _within_one_ulp(Hh.dev_to_f64(ws[:, :I]), ref)
    assert torch.count_nonzero(ws[:, I:]) == 0


@pytest.mark.parametrize("mode", [3, 5, 7, 8])
def test_f3_window_modes(mode):
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    M, K, I = 32, 64, 256
    x, w = _inputs(M, K, I, seed=4)
    ws = torch.randn(M, 2 * I, device="cuda").to(torch.bfloat16)
    d0 = torch.full((M, I), 7.0, device="cuda", dtype=torch.bfloat16)
    d, ws2 = npu.f3_gateup_epilogue(x, w, ws, d0, mode)
    torch.cuda.synchronize()
    if mode in (3, 5):
        assert torch.equal(d, ws[:, :I])
    elif mode == 8:
        assert torch.count_nonzero(d) == 0
    else:
        assert torch.all(d == 7.0)


def test_f3_reference_checks():
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    x, w = _inputs(15, 64, 128, seed=5)
    with pytest.raises(RuntimeError, match="f3_gateup_epilogue: M must be a multiple of 16"):
        npu.f3_gateup_epilogue(x, w, None, None, 1)
    x, w = _inputs(16, 64, 100, seed=5)
    with pytest.raises(RuntimeError, match="I must be a multiple of the N tile"):
        npu.f3_gateup_epilogue(x, w, None, None, 1)
    x, w = _inputs(16, 64, 128, seed=5)
    with pytest.raises(RuntimeError, match="mode must be 0..5, 7 or 8"):
        npu.f3_gateup_epilogue(x, w, None, None, 6)


@pytest.mark.parametrize("M", [1, 16, 64, 256, 4096])
def test_swiglu_llama8b_shapes_vs_torch_fp32(M):
    """BASELINE shapes (K=4096, I=14336): against torch fp32 GEMM + fp32
    SwiGLU on the same bf16 inputs, within one bf16 ulp (+ fp32 GEMM order
    noise), and the capi path equals the op."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    C = Hh.capi()
    K, I = 4096, 14336
    x, w = _inputs(M, K, I, seed=100 + M)
    d = npu.cascade_gateup_swiglu(x, w)
    c = x.float() @ w.float().t()
    g, u = c[:, :I], c[:, I:]
    ref = (g / (1 + torch.exp(-g)) * u)
    err = (d.float() - ref).abs()
    bound = torch.maximum(ref.abs(), d.float().abs()) * 2.0 ** -7 + 1e-4
    assert bool((err <= bound).all()), float((err - bound).max())
    d2 = torch.empty_like(d)
    C.gateup(x, w, None, d2, I, M, K, I, 1)
    torch.cuda.synchronize()
    assert torch.equal(d, d2)


@pytest.mark.parametrize("M,K,I", [(200, 4096, 14336), (256, 8192, 3584), (129, 1024, 640), (256, 64, 128),
                                   (256, 256, 20480), (136, 208, 20480), (256, 128, 17024), (256, 8192, 7168),
                                   (136, 1040, 512), (200, 512, 1792)])
def test_swiglu_256_row_forms(M, K, I):
    """129..256 rows (the CTA-pair 256 x 256 or 256 x 224 tile, the one-CTA
    256-row tile with a shared W tile, or the 128-row forms the launcher picks
    by tile count; 80 / 76 pair tiles for more tiles than pairs; the split-K
    cluster of pairs for narrow shards: 4 splits at I = 3584 and 512 -- the
    latter with a ragged last K block and 17 K blocks split 4/4/4/5 -- and 2
    at I = 7168 and 1792), K from one block to 8192 and a ragged last K block:
    within one bf16 ulp of torch fp32 (+ GEMM order noise), bit-identical on
    a second call, no device error, and the C ABI equal to the op."""
    import torch
    Hh.need_cuda()
    npu = Hh.ops()
    C = Hh.capi()
    x, w = _inputs(M, K, I, seed=M + K + I)
    d = npu.cascade_gateup_swiglu(x, w)
    d_again = npu.cascade_gateup_swiglu(x, w)
    c = x.float() @ w.float().t()
    g, u = c[:, :I], c[:, I:]
    ref = (g / (1 + torch.exp(-g)) * u)
    err = (d.float() - ref).abs()
    bound = torch.maximum(ref.abs(), d.float().abs()) * 2.0 ** -7 + 1e-4
    assert bool((err <= bound).all()), float((err - bound).max())
    assert torch.equal(d, d_again)
    d2 = torch.empty_like(d)
    C.gateup(x, w, None, d2, I, M, K, I, 1)
    torch.cuda.synchronize()
    assert torch.equal(d, d2)
    assert C.device_error() == 0
