"""Tensor-core block-scaled MMA self-test (tcgen05 kind::mxf4) against the CPU oracle's MXFP4 decode.

Pins the conventions every tensor-core kernel here relies on: 128-byte swizzled K-major operands loaded by TMA and by
bulk copy, shared-memory and instruction descriptors, scale-factor chunks placed in TMEM by tcgen05.cp (sf_id per
MMA), and accumulator readback. Scales vary per row and per block, so a misplaced scale changes the result.
Tolerance: max-abs <= 1e-5 * max|ref| and rel-L2 <= 1e-6 (fp32 accumulation of exact products).
"""
import numpy as np
import pytest
import torch

from gptoss_b200 import capi
from oracle import mxfp4

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = capi.ptr


@pytest.mark.parametrize("N,K,swz", [(8, 64, 128), (8, 576, 128), (16, 1024, 128), (64, 512, 128), (128, 256, 128),
                                     (256, 256, 128), (24, 320, 128), (192, 512, 128), (8, 64, 64), (8, 128, 64),
                                     (8, 576, 64), (16, 1024, 64), (256, 320, 64)])
def test_mxf4_gemm_selftest(N, K, swz):
    """swz: A loaded with the 128-byte swizzle (128-byte boxes of K) or the 64-byte one (64-byte boxes)."""
    lib = capi.load()
    g = torch.Generator().manual_seed(N * 1000 + K)
    a_b = torch.randint(0, 256, (128, K // 32, 16), generator=g, dtype=torch.uint8)
    a_s = torch.randint(110, 140, (128, K // 32), generator=g, dtype=torch.uint8)
    b_b = torch.randint(0, 256, (N, K // 32, 16), generator=g, dtype=torch.uint8)
    b_s = torch.randint(110, 140, (N, K // 32), generator=g, dtype=torch.uint8)
    d = [t.to(DEV).contiguous() for t in (a_b, a_s, b_b, b_s)]
    out = torch.full((128, N), float("nan"), device=DEV)
    rc = lib.gptoss_selftest_mxf4_gemm_swizzle(*(P(t) for t in d), P(out), N, K, swz)
    assert rc == 0, lib.gptoss_last_error().decode()
    A = mxfp4.dequant(a_b.numpy(), a_s.numpy()).astype(np.float64)
    B = mxfp4.dequant(b_b.numpy(), b_s.numpy()).astype(np.float64)
    want = A @ B.T
    got = out.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - want)
    assert err.max() <= 1e-5 * np.abs(want).max(), err.max() / np.abs(want).max()
    assert np.linalg.norm(got - want) <= 1e-6 * np.linalg.norm(want)


@pytest.mark.parametrize("which", [0, 1, 2, 3, 4])
def test_activation_terms_roundtrip(which):
    """x -> 16 e2m1 residual terms -> decoded sum: within 2^-22 of each 32-block's maximum (fp32 rounding of the sum
    included), and the first term equals the reference quantizer's rounding of x (oracle/mxfp4.quantize: the same
    power-of-two scale), except at exact midpoints between e2m1 values, which round to even here and to the lower
    value there."""
    lib = capi.load()
    g = torch.Generator().manual_seed(9 + which)
    n = 3072
    x = torch.randn(n, generator=g) * torch.exp(torch.randn(n, generator=g))    # widely varying magnitudes
    x[:32] = 0.0
    x[32:64] = torch.tensor([6.0, -6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25] + [1e-3] * 22)
    dx = x.to(DEV)
    out = torch.empty_like(dx)
    per = torch.empty(2, n, device=DEV)
    assert lib.gptoss_selftest_terms(P(dx), n, P(out), P(per), which) == 0, lib.gptoss_last_error().decode()
    xb = x.view(-1, 32).double()
    err = (out.cpu().double().view(-1, 32) - xb).abs().max(dim=1).values
    amax = xb.abs().max(dim=1).values
    assert (err <= amax * 2.0 ** -22).all(), (err / amax.clamp_min(1e-30)).max()
    qb, qs = mxfp4.quantize(x.numpy().reshape(-1, 32)[None])
    first = mxfp4.dequant(qb, qs).reshape(-1)
    scale = np.repeat(mxfp4.e8m0_to_float(qs.reshape(-1)), 32)
    y = np.abs(x.numpy()) / scale
    tie = np.isin(y, np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32))
    got = per[0].cpu().numpy()
    assert tie.sum() >= 6
    assert np.array_equal(got[~tie], first[~tie])
    even = {0.25: 0.0, 0.75: 1.0, 1.25: 1.0, 1.75: 2.0, 2.5: 2.0, 3.5: 4.0, 5.0: 4.0}
    want_tie = np.sign(x.numpy()[tie]) * np.array([even[float(v)] for v in y[tie]]) * scale[tie]
    assert np.array_equal(got[tie], want_tie.astype(np.float32))


def test_mxf4_peak_is_plausible():
    """The measured dense kind::mxf4 rate (the batched path's roofline denominator) lies between a quarter of and
    just above NVIDIA's nominal dense FP4 figure for B200 (9 PFLOP/s)."""
    import ctypes
    from gptoss_b200 import capi
    lib = capi.load()
    tf = ctypes.c_double()
    assert lib.gptoss_selftest_mxf4_peak(ctypes.byref(tf)) == 0, lib.gptoss_last_error().decode()
    assert 2250.0 < tf.value < 10000.0, tf.value


def test_mxf4_mma_cost_by_n():
    """Time per M = 128, K = 64 kind::mxf4 MMA for N = 8 .. 256 (printed with pytest -s): positive, at most the N = 256
    time plus a little for every N, and the N = 256 figure consistent with the measured peak."""
    import ctypes
    lib = capi.load()
    ns = {}
    for n in (8, 16, 32, 64, 128, 256):
        v = ctypes.c_double()
        assert lib.gptoss_selftest_mxf4_mma_ns(n, ctypes.byref(v)) == 0, lib.gptoss_last_error().decode()
        ns[n] = v.value
    print("ns per MMA by N:", {n: round(t, 2) for n, t in ns.items()})
    assert all(t > 0 for t in ns.values())
    assert all(ns[n] <= 1.1 * ns[256] for n in ns)
    assert lib.gptoss_selftest_mxf4_mma_ns(12, ctypes.byref(ctypes.c_double())) != 0
