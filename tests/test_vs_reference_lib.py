"""Our C ABI against openvang/gptoss-infer's own runtime built for sm_100a (oracle/_ref/libgptoss_ref.so, made by
oracle/Makefile where the reference sources exist): same entry points, same device inputs. Checker only.

Ids must be identical. MoE outputs must agree within the fp32 accumulation-order bound used elsewhere
(max-abs <= 2e-5 * max|ref|, rel-L2 <= 2e-5), both libraries also being checked against float64.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gptoss_b200 import capi, synth
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libgptoss_ref.so"
DEV = "cuda"
P = capi.ptr


@pytest.fixture(scope="module")
def libs():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libgptoss_ref.so not built (reference sources absent when building)")
    return capi.load(), capi.load(REF_LIB)


def rel(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return np.abs(got - want).max() / np.abs(want).max(), np.linalg.norm(got - want) / np.linalg.norm(want)


def test_router_and_moe_agree_with_reference_runtime(libs):
    ours, ref = libs
    t = synth.moe_layer(seed=31)
    p = "model.layers.0.mlp."
    W, b = t[p + "router.weight"].to(DEV), t[p + "router.bias"].float().to(DEV)
    ex = [t[p + "experts." + n].to(DEV) for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                                                  "down_proj_blocks", "down_proj_scales", "down_proj_bias")]
    ex[2], ex[5] = ex[2].float(), ex[5].float()
    X = synth.tokens(16, seed=32)
    for r in range(X.shape[0]):
        x = X[r].to(DEV)
        outs = []
        for lib in (ours, ref):
            ids = torch.empty(4, device=DEV, dtype=torch.int32)
            w = torch.empty(4, device=DEV)
            assert lib.gptoss_kernel_router(P(W), P(b), P(x), 32, 2880, 4, P(ids), P(w)) == 0
            y = torch.zeros(2880, device=DEV)
            assert lib.gptoss_kernel_moe(*(P(e) for e in ex), P(x), P(ids), P(w), P(y), 4, 2880, 2880, 1.702,
                                         7.0) == 0
            outs.append((ids.cpu().numpy(), w.cpu().numpy(), y.cpu().numpy()))
        (i0, w0, y0), (i1, w1, y1) = outs
        assert i0.tolist() == i1.tolist()
        np.testing.assert_allclose(w0, w1, rtol=1e-5, atol=1e-6)
        mx, l2 = rel(y0, y1)
        assert mx <= 2e-5 and l2 <= 2e-5, (r, mx, l2)


def test_kernel_time_against_reference_runtime(libs):
    """Times both libraries' gptoss_kernel_moe on the same config-0 inputs (informational; prints the ratio)."""
    ours, ref = libs
    t = synth.moe_layer(seed=33)
    p = "model.layers.0.mlp."
    ex = [t[p + "experts." + n].to(DEV) for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                                                  "down_proj_blocks", "down_proj_scales", "down_proj_bias")]
    ex[2], ex[5] = ex[2].float(), ex[5].float()
    x = synth.tokens(1, seed=34)[0].to(DEV)
    ids = torch.tensor([3, 17, 30, 8], dtype=torch.int32, device=DEV)
    w = torch.full((4,), 0.25, device=DEV)
    y = torch.zeros(2880, device=DEV)
    res = {}
    for name, lib in (("ours", ours), ("reference", ref)):
        for _ in range(5):
            assert lib.gptoss_kernel_moe(*(P(e) for e in ex), P(x), P(ids), P(w), P(y), 4, 2880, 2880, 1.702, 7.0) == 0
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(50):
            lib.gptoss_kernel_moe(*(P(e_) for e_ in ex), P(x), P(ids), P(w), P(y), 4, 2880, 2880, 1.702, 7.0)
        e.record()
        torch.cuda.synchronize()
        res[name] = s.elapsed_time(e) / 50 * 1e3
    print(f"\ngptoss_kernel_moe us/call (incl. sync): ours {res['ours']:.1f}  reference {res['reference']:.1f}")
    assert res["ours"] > 0 and res["reference"] > 0
