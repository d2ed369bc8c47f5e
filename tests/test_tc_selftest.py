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


@pytest.mark.parametrize("N,K", [(8, 64), (8, 576), (16, 1024), (64, 512), (128, 256), (256, 256), (24, 320)])
def test_mxf4_gemm_selftest(N, K):
    lib = capi.load()
    g = torch.Generator().manual_seed(N * 1000 + K)
    a_b = torch.randint(0, 256, (128, K // 32, 16), generator=g, dtype=torch.uint8)
    a_s = torch.randint(110, 140, (128, K // 32), generator=g, dtype=torch.uint8)
    b_b = torch.randint(0, 256, (N, K // 32, 16), generator=g, dtype=torch.uint8)
    b_s = torch.randint(110, 140, (N, K // 32), generator=g, dtype=torch.uint8)
    d = [t.to(DEV).contiguous() for t in (a_b, a_s, b_b, b_s)]
    out = torch.full((128, N), float("nan"), device=DEV)
    rc = lib.gptoss_selftest_mxf4_gemm(*(P(t) for t in d), P(out), N, K)
    assert rc == 0, lib.gptoss_last_error().decode()
    A = mxfp4.dequant(a_b.numpy(), a_s.numpy()).astype(np.float64)
    B = mxfp4.dequant(b_b.numpy(), b_s.numpy()).astype(np.float64)
    want = A @ B.T
    got = out.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - want)
    assert err.max() <= 1e-5 * np.abs(want).max(), err.max() / np.abs(want).max()
    assert np.linalg.norm(got - want) <= 1e-6 * np.linalg.norm(want)
