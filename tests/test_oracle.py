"""Pins the CPU oracle: the reference's own MXFP4 known-answer tests, restated, plus golden vectors that the
reference itself produced (tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest
import torch

from conftest import load_golden, tiny_tensors
from oracle import moe as omoe
from oracle import mxfp4


def naive_dequant(blocks, scales):
    """Element by element from the spec (reference/tests/test_mxfp4.py:7-14)."""
    out = []
    for row_b, row_s in zip(blocks.reshape(-1, 16).tolist(), scales.reshape(-1).tolist()):
        for byte in row_b:
            for code in (byte & 0x0F, byte >> 4):
                out.append(mxfp4.FP4_VALUES[code] * 2.0 ** (row_s - 127))
    return np.array(out, dtype=np.float32).reshape(*scales.shape[:-1], scales.shape[-1] * 32)


def test_matches_naive_decoding():
    g = load_golden("mxfp4_kat.npz")
    b, s = g["rand_blocks"], g["rand_scales"]
    assert np.array_equal(mxfp4.dequant(b, s), naive_dequant(b, s))


def test_matches_reference_golden_bitwise():
    g = load_golden("mxfp4_kat.npz")
    got = mxfp4.dequant(g["rand_blocks"], g["rand_scales"])
    assert np.array_equal(got.view(np.uint32), g["rand_out"].view(np.uint32))


def test_every_code_and_nibble_order():
    g = load_golden("mxfp4_kat.npz")
    b = np.zeros((1, 16), np.uint8)
    b[0, 0] = 0x21
    out = mxfp4.dequant(b, np.array([127], np.uint8))
    assert out[0] == 0.5 and out[1] == 1.0
    assert np.array_equal(out.view(np.uint32), g["nibble_out"].view(np.uint32))
    out = mxfp4.dequant(g["codes_blocks"], np.array([128], np.uint8))
    assert out[:16].tolist() == [2 * v for v in mxfp4.FP4_VALUES]
    assert np.array_equal(out.view(np.uint32), g["codes_out"].view(np.uint32))   # -0.0 keeps its sign bit


def test_scale_extremes_are_exact():
    g = load_golden("mxfp4_kat.npz")
    b = np.full((1, 16), 0x77, np.uint8)
    lo = mxfp4.dequant(b, np.array([1], np.uint8))
    assert lo[0] == 6.0 * 2.0 ** -126
    hi = mxfp4.dequant(b, np.array([254], np.uint8))
    assert hi[0] == np.float32(np.inf)           # 6 * 2**127 overflows fp32, as in the reference
    assert np.array_equal(lo.view(np.uint32), g["ext_lo_out"].view(np.uint32))
    assert np.array_equal(hi.view(np.uint32), g["ext_hi_out"].view(np.uint32))


def test_every_valid_scale_is_an_exact_power_of_two():
    g = load_golden("mxfp4_kat.npz")
    b = np.full((255, 1, 16), 0x22, np.uint8)
    s = np.arange(255, dtype=np.uint8).reshape(255, 1)
    out = mxfp4.dequant(b, s)
    want = np.array([2.0 ** (v - 127) for v in range(255)], dtype=np.float64).astype(np.float32)
    assert np.array_equal(out[:, 0], want) and np.array_equal(out[:, 31], want)
    assert np.array_equal(out.view(np.uint32), g["allscale_out"].view(np.uint32))


def test_nan_scale_rejected():
    with pytest.raises(ValueError):
        mxfp4.dequant(np.zeros((1, 16), np.uint8), np.array([255], np.uint8))


def test_quantize_matches_reference():
    g = load_golden("mxfp4_kat.npz")
    qb, qs = mxfp4.quantize(g["rt_w"])
    assert np.array_equal(qb, g["rt_blocks"]) and np.array_equal(qs, g["rt_scales"])
    assert np.array_equal(mxfp4.dequant(qb, qs), g["rt_w"])
    qb, qs = mxfp4.quantize(g["gq_w"])
    assert np.array_equal(qb, g["gq_blocks"]) and np.array_equal(qs, g["gq_scales"])


def test_tiny_moe_matches_reference():
    g = load_golden("tiny_moe.npz")
    t = tiny_tensors(g)
    p = "model.layers.0."
    h = omoe.rms_norm(g["x"], t[p + "post_attention_layernorm.weight"])
    np.testing.assert_allclose(h, g["h"], rtol=1e-6, atol=1e-6)
    out, ids, gate, logits = omoe.moe(t, p, g["h"], k=4, return_routing=True)
    assert np.array_equal(ids, g["top_idx"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)


def test_config0_moe_matches_reference():
    from gptoss_b200 import synth
    g = load_golden("config0_moe.npz")
    t = synth.moe_layer(seed=0)
    assert synth.digest(t) == str(g["weights_sha256"]), "synthetic weights drifted from the golden's"
    x = synth.tokens(4, seed=1).numpy()
    assert np.array_equal(x, g["x"])
    tn = synth.to_numpy(t)
    p = "model.layers.0."
    h = omoe.rms_norm(x, tn[p + "post_attention_layernorm.weight"])
    np.testing.assert_allclose(h, g["h"], rtol=1e-6, atol=1e-6)
    out, ids, gate, logits = omoe.moe(tn, p, g["h"], k=4, return_routing=True)
    assert not omoe.near_tie_rows(logits, 4).any()
    assert np.array_equal(ids, g["top_idx"])
    err = np.abs(out - g["out"])
    assert err.max() <= 1e-5 * np.abs(g["out"]).max()                             # max-abs, scaled
    assert np.linalg.norm(out - g["out"]) <= 1e-5 * np.linalg.norm(g["out"])       # rel-L2


def test_router_sort_rule_with_engineered_tie():
    """runtime/tests/test_kernels.py:264-279: expert E-1 duplicates expert 1, which leads; the lower id wins."""
    for E, k in ((32, 4), (32, 8), (6, 4)):
        g = torch.Generator().manual_seed(3)
        W = (torch.randn(E, 2880, generator=g) * 0.05).to(torch.bfloat16).float().numpy()
        b = (torch.randn(E, generator=g) * 0.1).numpy()
        x = torch.randn(2880, generator=g).numpy()
        b[1] += 10
        W[E - 1], b[E - 1] = W[1], b[1]
        logits, ids, w = omoe.router_f64(W, b, x, k)
        want = sorted(range(E), key=lambda e: (-logits[e], e))[:k]
        assert ids.tolist() == want and ids[0] == 1 and ids[1] == E - 1


def test_kernel_and_batched_semantics_agree():
    g = load_golden("tiny_moe.npz")
    t = tiny_tensors(g)
    p = "model.layers.0.mlp."
    args = [t[p + "experts." + n] for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                                           "down_proj_blocks", "down_proj_scales", "down_proj_bias")]
    h = g["h"]
    _, ids, gate = omoe.router(h, t[p + "router.weight"], t[p + "router.bias"], 4)
    resid = np.zeros_like(h)
    batched = omoe.moe_batched_f64(*args, h, ids, gate, resid)
    for r in range(h.shape[0]):
        single = omoe.kernel_moe_f64(*args, h[r], ids[r], gate[r], resid[r])
        np.testing.assert_allclose(batched[r], single, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(batched, g["out"], rtol=1e-5, atol=1e-6)
