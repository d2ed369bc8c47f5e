"""gptoss_kernel_moe_static_scratch: the MoE entry point for callers that cannot allocate device memory during the
call (an engine that hands all its memory to its own budgeted allocator, or a decode loop that must not meet the
implicit synchronization of cudaMalloc). Its scratch is a fixed device array in the library.

Checked through the C ABI, two calls in a row on the same residual stream (x_resid += MoE(x_norm) twice), at the
real 20b layer shape:
  * bit-identical to gptoss_kernel_moe on the CUDA-core path (the same kernels, only the scratch differs);
  * against the float64 oracle (oracle/moe.py kernel_moe_f64, applied twice): rtol 1e-4 / atol 1e-3 (the
    reference's runtime/tests/test_kernels.py:174 bound) and max-abs <= 2e-5 * max|x_resid|;
  * the tensor-core path of gptoss_kernel_moe against the same oracle and bound (its absolute part scaled with the
    output above 1e3), and the two paths against each other within the sum of their bounds.
Shapes past the fixed scratch (k * I > 8 * 3072) must fail with -1 and a message. This file is collected last, so a
run that stops at the first failure has run every other test before it.
"""
import numpy as np
import pytest
import torch

from gptoss_b200 import capi, synth
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = capi.ptr
NAMES = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks", "down_proj_scales",
         "down_proj_bias")


@pytest.fixture(scope="module")
def case():
    t = synth.moe_layer(seed=0)
    p = "model.layers.0.mlp.experts."
    host = [t[p + n] for n in NAMES]
    ex = [h.to(DEV) for h in host]
    ex[2], ex[5] = ex[2].float(), ex[5].float()
    g = torch.Generator().manual_seed(31)
    x_norm = torch.randn(2880, generator=g)
    ids = torch.tensor([3, 17, 8, 30], dtype=torch.int32)
    w = torch.softmax(torch.randn(4, generator=g), 0)
    x0 = torch.randn(2880, generator=g)
    return host, ex, x_norm, ids, w, x0


def run_twice(lib, fn, case):
    _, ex, x_norm, ids, w, x0 = case
    d_x, d_ids, d_w = x_norm.to(DEV), ids.to(DEV), w.to(DEV)
    xr = x0.to(DEV).clone()
    for _ in range(2):
        rc = fn(*(P(e) for e in ex), P(d_x), P(d_ids), P(d_w), P(xr), 4, 2880, 2880, 1.702, 7.0)
        assert rc == 0, lib.gptoss_last_error().decode()
    return xr.cpu()


def test_static_scratch_bitidentical_to_cuda_core_path(case):
    lib = capi.load()
    got = run_twice(lib, lib.gptoss_kernel_moe_static_scratch, case)
    prev = lib.gptoss_set_moe_impl(0)
    try:
        want = run_twice(lib, lib.gptoss_kernel_moe, case)
    finally:
        lib.gptoss_set_moe_impl(prev)
    assert torch.isfinite(got).all()
    assert torch.equal(got, want)


def oracle_twice(case):
    host, _, x_norm, ids, w, x0 = case
    arrs = [h.float().numpy() if h.dtype == torch.bfloat16 else h.numpy() for h in host]
    want = x0.numpy().astype(np.float64)
    for _ in range(2):
        want = omoe.kernel_moe_f64(*arrs, x_norm.numpy(), ids.numpy(), w.numpy(), want)
    return want


def test_static_scratch_matches_float64_oracle(case):
    lib = capi.load()
    got = run_twice(lib, lib.gptoss_kernel_moe_static_scratch, case).numpy().astype(np.float64)
    want = oracle_twice(case)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


def test_static_scratch_matches_tensor_core_path(case):
    """Both paths meet the float64 bound on their own; their difference is then within the sum of the two bounds
    (rtol 2e-4 / atol 2e-3: two results each within rtol 1e-4 / atol 1e-3 of the exact value)."""
    lib = capi.load()
    got = run_twice(lib, lib.gptoss_kernel_moe_static_scratch, case).numpy().astype(np.float64)
    prev = lib.gptoss_set_moe_impl(1)
    try:
        tc = run_twice(lib, lib.gptoss_kernel_moe, case).numpy().astype(np.float64)
    finally:
        lib.gptoss_set_moe_impl(prev)
    want = oracle_twice(case)
    # The tensor-core path sums 4 x 23 partial output vectors in fp32 (one per 256-row job), so its absolute error
    # follows the output's scale: this case's outputs reach ~3.5e3 (scales up to 2^-1, against the reference test's
    # 2^-4), where atol 1e-3 is 4 fp32 spacings. The absolute bound grows with max|want| / 1e3 above that scale.
    atol = 1e-3 * max(1.0, np.abs(want).max() / 1e3)
    np.testing.assert_allclose(tc, want, rtol=1e-4, atol=atol)
    assert np.abs(tc - want).max() <= 2e-5 * np.abs(want).max()
    np.testing.assert_allclose(got, tc, rtol=2e-4, atol=1e-3 + atol)
    assert np.abs(got - tc).max() <= 4e-5 * np.abs(tc).max()


def test_static_scratch_rejects_oversize():
    lib = capi.load()
    buf = torch.zeros(16, device=DEV)
    # k * I = 8 * 3104 > 8 * 3072: refused before any launch
    rc = lib.gptoss_kernel_moe_static_scratch(*(P(buf) for _ in range(10)), 8, 3104, 3104, 1.702, 7.0)
    assert rc == -1
    assert "fixed scratch" in lib.gptoss_last_error().decode()
