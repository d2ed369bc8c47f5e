"""gptoss_kernel_moe_static_scratch (no device allocation during the call) against gptoss_kernel_moe.

Two calls in a row on the same residual stream (x_resid += MoE(x_norm) twice) through each entry point, at the
real 20b layer shape, must agree within the MoE tolerance of this suite: allclose rtol 1e-4 / atol 1e-3 and
max-abs <= 2e-5 * max|x_resid|. Shapes past the fixed scratch (k * I > 8 * 3072) must fail with -1 and a message.
"""
import numpy as np
import pytest
import torch

from gptoss_b200 import capi, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = capi.ptr


def _layer():
    t = synth.moe_layer(seed=0)
    p = "model.layers.0.mlp.experts."
    return [t[p + "gate_up_proj_blocks"].to(DEV), t[p + "gate_up_proj_scales"].to(DEV),
            t[p + "gate_up_proj_bias"].float().to(DEV), t[p + "down_proj_blocks"].to(DEV),
            t[p + "down_proj_scales"].to(DEV), t[p + "down_proj_bias"].float().to(DEV)]


def test_static_scratch_matches_kernel_moe():
    lib = capi.load()
    ex = _layer()
    g = torch.Generator().manual_seed(31)
    x_norm = torch.randn(2880, generator=g).to(DEV)
    ids = torch.tensor([3, 17, 8, 30], dtype=torch.int32, device=DEV)
    w = torch.softmax(torch.randn(4, generator=g), 0).to(DEV)
    x0 = torch.randn(2880, generator=g).to(DEV)
    outs = []
    for fn in (lib.gptoss_kernel_moe_static_scratch, lib.gptoss_kernel_moe):
        xr = x0.clone()
        for _ in range(2):
            rc = fn(*(P(e) for e in ex), P(x_norm), P(ids), P(w), P(xr), 4, 2880, 2880, 1.702, 7.0)
            assert rc == 0, lib.gptoss_last_error().decode()
        outs.append(xr.cpu().numpy().astype(np.float64))
    got, want = outs
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


def test_static_scratch_rejects_oversize():
    lib = capi.load()
    buf = torch.zeros(16, device=DEV)
    # k * I = 8 * 3104 > 8 * 3072: refused before any launch
    rc = lib.gptoss_kernel_moe_static_scratch(*(P(buf) for _ in range(10)), 8, 3104, 3104, 1.702, 7.0)
    assert rc == -1
    assert "fixed scratch" in lib.gptoss_last_error().decode()
