"""GPU parity tests through the C ABI (ctypes, device pointers), against the CPU oracle and the reference-made golden
vectors. Mirrors openvang/gptoss-infer runtime/tests/test_kernels.py:129-174 (router, real-shape MoE) and adds the
bit-exact MXFP4 decode, the config-0 block, and the tensor-core path.

Tolerances (stated here, used below):
  * MXFP4 decode, expert ids: bit-exact.
  * router weights: rtol 1e-5, atol 1e-6 vs float64 (the reference test's bound).
  * gptoss_kernel_moe vs float64: rtol 1e-4, atol 1e-3 (runtime/tests/test_kernels.py:174), and additionally
    max-abs <= 2e-5 * max|ref| and rel-L2 <= 2e-5 (fp32 accumulation-order noise only).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, tiny_tensors
from gptoss_b200 import capi, synth
from oracle import moe as omoe
from oracle import mxfp4

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = capi.ptr


@pytest.fixture(scope="module")
def lib():
    return capi.load()


def ok(lib, rc):
    assert rc == 0, lib.gptoss_last_error().decode()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rel_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30), \
        np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)


# ---------------------------------------------------------------------------------------------------- dequant
def test_mxfp4_dequant_bitexact(lib):
    g = torch.Generator().manual_seed(5)
    n = 4096
    blocks = torch.randint(0, 256, (n, 16), generator=g, dtype=torch.uint8).numpy()
    scales = torch.randint(0, 255, (n,), generator=g, dtype=torch.uint8).numpy()
    scales[:255] = np.arange(255, dtype=np.uint8)                     # every valid scale, 0 and 254 included
    blocks[:16] = (np.arange(256, dtype=np.uint8).reshape(16, 16))    # every byte value
    db, ds = dev(blocks), dev(scales)
    out = torch.empty(n * 32, device=DEV)
    ok(lib, lib.gptoss_kernel_mxfp4_dequant(P(db), P(ds), P(out), n))
    want = mxfp4.dequant(blocks.reshape(n, 1, 16), scales.reshape(n, 1)).reshape(-1)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_mxfp4_dequant_golden_and_nan_rejection(lib):
    g = load_golden("mxfp4_kat.npz")
    b, s = g["rand_blocks"].reshape(-1, 16), g["rand_scales"].reshape(-1)
    out = torch.empty(b.shape[0] * 32, device=DEV)
    db, ds = dev(b), dev(s)          # keep the device tensors alive for the duration of the call
    ok(lib, lib.gptoss_kernel_mxfp4_dequant(P(db), P(ds), P(out), b.shape[0]))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), g["rand_out"].reshape(-1).view(np.uint32))
    bad = dev(np.array([127, 255], np.uint8))
    assert lib.gptoss_kernel_mxfp4_dequant(P(db), P(bad), P(out), 2) == -1
    assert b"0xFF" in lib.gptoss_last_error()


# ---------------------------------------------------------------------------------------------------- rmsnorm
def test_rmsnorm(lib):
    gen = torch.Generator(device=DEV).manual_seed(1)
    x, w = torch.randn(2880, device=DEV, generator=gen) * 3, torch.randn(2880, device=DEV, generator=gen)
    y = torch.empty_like(x)
    ok(lib, lib.gptoss_kernel_rmsnorm(P(x), P(w), P(y), 2880, 1e-5))
    xd = x.double()
    torch.testing.assert_close(y.double(), xd * torch.rsqrt(xd.pow(2).mean() + 1e-5) * w.double(), rtol=1e-5,
                               atol=1e-6)


# ---------------------------------------------------------------------------------------------------- router
@pytest.mark.parametrize("E,k", [(32, 4), (32, 8), (6, 4), (1, 1), (17, 3)])
def test_router(lib, E, k):
    """runtime/tests/test_kernels.py:263-279, with the engineered tie: experts 1 and E-1 tie, the lower id wins."""
    gen = torch.Generator(device=DEV).manual_seed(3)
    W = (torch.randn(E, 2880, device=DEV, generator=gen) * 0.05).to(torch.bfloat16)
    b, x = torch.randn(E, device=DEV, generator=gen) * 0.1, torch.randn(2880, device=DEV, generator=gen)
    if E > 2:
        b[1] += 10
        W[E - 1], b[E - 1] = W[1], b[1]
    ids = torch.empty(k, device=DEV, dtype=torch.int32)
    w = torch.empty(k, device=DEV)
    ok(lib, lib.gptoss_kernel_router(P(W), P(b), P(x), E, 2880, k, P(ids), P(w)))
    logits = (W.double() @ x.double() + b.double()).tolist()
    want = sorted(range(E), key=lambda e: (-logits[e], e))[:k]
    assert ids.tolist() == want
    v = torch.tensor([logits[e] for e in want], dtype=torch.float64)
    torch.testing.assert_close(w.double().cpu(), torch.softmax(v, 0), rtol=1e-5, atol=1e-6)
    assert lib.gptoss_kernel_router(P(W), P(b), P(x), E, 2880, E + 1, P(ids), P(w)) != 0   # k > E is rejected


def test_router_many_tokens_exact_ids(lib):
    """512 random tokens at config-0 router statistics: ids equal the float64 ranking on every token."""
    t = synth.moe_layer(seed=21, E=32)
    Wt = t["model.layers.0.mlp.router.weight"]
    bt = t["model.layers.0.mlp.router.bias"].float()
    W, b = Wt.to(DEV), bt.to(DEV)
    X = synth.tokens(512, seed=22)
    ids = torch.empty(4, device=DEV, dtype=torch.int32)
    w = torch.empty(4, device=DEV)
    got = []
    for r in range(X.shape[0]):
        x = X[r].to(DEV)
        ok(lib, lib.gptoss_kernel_router(P(W), P(b), P(x), 32, 2880, 4, P(ids), P(w)))
        got.append(ids.cpu().numpy().copy())
    logits = X.double().numpy() @ Wt.double().numpy().T + bt.double().numpy()
    want = omoe.topk_ids(logits, 4)
    assert np.array_equal(np.stack(got), want)


# ---------------------------------------------------------------------------------------------------- moe
def real_shape_case(E=6, seed=4):
    """runtime/tests/test_kernels.py:282-294: real H = I = 2880, E experts, ids [5, 0, 3, 2]."""
    g = torch.Generator().manual_seed(seed)
    H = I = 2880
    k = 4
    gu_b = torch.randint(0, 256, (E, 2 * I, H // 32, 16), generator=g, dtype=torch.uint8)
    gu_s = torch.randint(118, 124, (E, 2 * I, H // 32), generator=g, dtype=torch.uint8)
    dn_b = torch.randint(0, 256, (E, H, I // 32, 16), generator=g, dtype=torch.uint8)
    dn_s = torch.randint(118, 124, (E, H, I // 32), generator=g, dtype=torch.uint8)
    gu_bias, dn_bias = torch.randn(E, 2 * I, generator=g) * 0.1, torch.randn(E, H, generator=g) * 0.1
    x = torch.randn(H, generator=g)
    resid = torch.randn(H, generator=g)
    ids = torch.tensor([5, 0, 3, 2], dtype=torch.int32)
    weights = torch.softmax(torch.randn(k, generator=g), 0)
    return [gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias, x, ids, weights], resid, H, I, k


def small_shape_case(seed=9):
    """A second tensor-core shape (k = 2, H = 512, I = 256, 4 experts) for the shape-switch test."""
    g = torch.Generator().manual_seed(seed)
    E, H, I, k = 4, 512, 256, 2
    gu_b = torch.randint(0, 256, (E, 2 * I, H // 32, 16), generator=g, dtype=torch.uint8)
    gu_s = torch.randint(118, 124, (E, 2 * I, H // 32), generator=g, dtype=torch.uint8)
    dn_b = torch.randint(0, 256, (E, H, I // 32, 16), generator=g, dtype=torch.uint8)
    dn_s = torch.randint(118, 124, (E, H, I // 32), generator=g, dtype=torch.uint8)
    gu_bias, dn_bias = torch.randn(E, 2 * I, generator=g) * 0.1, torch.randn(E, H, generator=g) * 0.1
    x = torch.randn(H, generator=g)
    resid = torch.randn(H, generator=g)
    ids = torch.tensor([3, 1], dtype=torch.int32)
    weights = torch.softmax(torch.randn(k, generator=g), 0)
    return [gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias, x, ids, weights], resid, H, I, k


@pytest.mark.parametrize("impl", [1, 2])
def test_moe_tensor_cores_alternating_shapes(lib, impl):
    """Two shapes alternating on one thread share its decode workspace, whose launch-to-launch state (barrier words,
    launch epoch, epoch-tagged partial sums) sits at shape-dependent offsets: every call must give the result the
    shape gives alone (bit-identical), and the small shape must meet the float64 bound. impl 1: the row-job kernel
    (where the shape allows it), 2: the stream-K kernel."""
    cases = [real_shape_case(), small_shape_case()]
    dev_cases = [([t.to(DEV).contiguous() for t in args], resid.to(DEV), H, I, k) for args, resid, H, I, k in cases]

    def run(i):
        d, resid, H, I, k = dev_cases[i]
        out = resid.clone()
        ok(lib, lib.gptoss_kernel_moe(*(P(t) for t in d), P(out), k, H, I, 1.702, 7.0))
        return out.cpu()

    prev = lib.gptoss_set_moe_impl(impl)
    try:
        alone = [run(0), run(0), run(1), run(1)]
        assert torch.equal(alone[0], alone[1]) and torch.equal(alone[2], alone[3])
        for i in (0, 1, 0, 1, 1, 0):
            assert torch.equal(run(i), alone[2 * i]), i
    finally:
        lib.gptoss_set_moe_impl(prev)
    args, resid, H, I, k = cases[1]
    want = omoe.kernel_moe_f64(*[a.numpy() for a in args[:6]], args[6].numpy(), args[7].numpy(), args[8].numpy(),
                               resid.numpy())
    got = alone[2].double().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("impl", [0, 1, 2])
def test_moe_real_shape(lib, impl):
    args, resid, H, I, k = real_shape_case()
    want = omoe.kernel_moe_f64(*[a.numpy() for a in args[:6]], args[6].numpy(), args[7].numpy(), args[8].numpy(),
                               resid.numpy())
    d = [t.to(DEV).contiguous() for t in args]
    out = resid.to(DEV).clone()
    prev = lib.gptoss_set_moe_impl(impl)
    try:
        ok(lib, lib.gptoss_kernel_moe(*(P(t) for t in d), P(out), k, H, I, 1.702, 7.0))
    finally:
        lib.gptoss_set_moe_impl(prev)
    got = out.cpu().double().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)
    mx, l2 = rel_err(got - resid.double().numpy(), want - resid.double().numpy())
    assert mx <= 2e-5 and l2 <= 2e-5, (mx, l2)


def test_moe_tiny_golden(lib):
    """Reference.moe on the tiny layer (H=64, I=32, 8 experts), one token at a time through the two ABI calls."""
    g = load_golden("tiny_moe.npz")
    t = tiny_tensors(g)
    p = "model.layers.0.mlp."
    W = torch.from_numpy(t[p + "router.weight"]).to(torch.bfloat16).to(DEV)
    b = dev(t[p + "router.bias"])
    ex = [dev(t[p + "experts." + n]) for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                                               "down_proj_blocks", "down_proj_scales", "down_proj_bias")]
    ids = torch.empty(4, device=DEV, dtype=torch.int32)
    w = torch.empty(4, device=DEV)
    for r in range(g["h"].shape[0]):
        h = dev(g["h"][r])
        ok(lib, lib.gptoss_kernel_router(P(W), P(b), P(h), 8, 64, 4, P(ids), P(w)))
        assert ids.cpu().numpy().tolist() == g["top_idx"][r].tolist()
        out = torch.zeros(64, device=DEV)
        ok(lib, lib.gptoss_kernel_moe(*(P(e) for e in ex), P(h), P(ids), P(w), P(out), 4, 64, 32, 1.702, 7.0))
        mx, l2 = rel_err(out.cpu().numpy(), g["out"][r])
        assert mx <= 2e-5 and l2 <= 2e-5, (r, mx, l2)


@pytest.fixture(scope="module")
def config0():
    t = synth.moe_layer(seed=0)
    g = load_golden("config0_moe.npz")
    assert synth.digest(t) == str(g["weights_sha256"])
    p = "model.layers.0."
    d = {
        "ln": t[p + "post_attention_layernorm.weight"].float().to(DEV),
        "W": t[p + "mlp.router.weight"].to(DEV), "b": t[p + "mlp.router.bias"].float().to(DEV),
        "ex": [t[p + "mlp.experts." + n].to(DEV).float() if n.endswith("bias") else t[p + "mlp.experts." + n].to(DEV)
               for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                         "down_proj_blocks", "down_proj_scales", "down_proj_bias")],
    }
    return d, g


@pytest.mark.parametrize("impl", [0, 1, 2])
def test_config0_block_vs_reference_golden(lib, config0, impl):
    """RMSNorm -> router -> MoE for each of the 4 golden tokens, against Reference.moe's own output."""
    d, g = config0
    ids = torch.empty(4, device=DEV, dtype=torch.int32)
    w = torch.empty(4, device=DEV)
    prev = lib.gptoss_set_moe_impl(impl)
    try:
        for r in range(g["x"].shape[0]):
            x = dev(g["x"][r])
            h = torch.empty_like(x)
            ok(lib, lib.gptoss_kernel_rmsnorm(P(x), P(d["ln"]), P(h), 2880, 1e-5))
            np.testing.assert_allclose(h.cpu().numpy(), g["h"][r], rtol=1e-5, atol=1e-6)
            hg = dev(g["h"][r])                              # feed the golden h so routing sees the same input
            ok(lib, lib.gptoss_kernel_router(P(d["W"]), P(d["b"]), P(hg), 32, 2880, 4, P(ids), P(w)))
            assert ids.cpu().numpy().tolist() == g["top_idx"][r].tolist()
            out = torch.zeros(2880, device=DEV)
            ok(lib, lib.gptoss_kernel_moe(*(P(e) for e in d["ex"]), P(hg), P(ids), P(w), P(out), 4, 2880, 2880,
                                          1.702, 7.0))
            mx, l2 = rel_err(out.cpu().numpy(), g["out"][r])
            assert mx <= 2e-5 and l2 <= 2e-5, (r, mx, l2)
    finally:
        lib.gptoss_set_moe_impl(prev)


@pytest.fixture(params=[1, 2], ids=["rows", "streamk"])
def tc_impl(lib, request):
    """The tensor-core decode kernel a prepared layer runs: 1 = the row-job kernel, 2 = the stream-K kernel."""
    prev = lib.gptoss_set_moe_impl(request.param)
    yield request.param
    lib.gptoss_set_moe_impl(prev)


def make_layer(lib, d, E=32, k=4):
    L = lib.gptoss_moe_layer_create(P(d["ln"]), 1e-5, P(d["W"]), P(d["b"]), *(P(e) for e in d["ex"]), E, k, 2880, 2880,
                                    1.702, 7.0)
    assert L, lib.gptoss_last_error().decode()
    return L


def test_layer_forward_config0_vs_reference_golden(lib, config0, tc_impl):
    """Prepared layer (fused RMSNorm + router + tensor-core GEMVs) on the 4 golden tokens: x + Reference.moe(h)."""
    d, g = config0
    L = make_layer(lib, d)
    try:
        for r in range(g["x"].shape[0]):
            x = dev(g["x"][r])
            out = x.clone()
            ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(out), None, None))
            torch.cuda.synchronize()
            mx, l2 = rel_err((out - x).cpu().numpy(), g["out"][r])
            assert mx <= 2e-5 and l2 <= 2e-5, (r, mx, l2)
    finally:
        lib.gptoss_moe_layer_destroy(L)


def test_layer_forward_is_deterministic_and_in_place(lib, config0, tc_impl):
    d, g = config0
    L = make_layer(lib, d)
    try:
        x = dev(g["x"][1])
        a, b = x.clone(), x.clone()
        ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(a), None, None))
        ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(b), None, None))
        c = x.clone()
        ok(lib, lib.gptoss_moe_layer_forward(L, P(c), P(c), None, None))     # x_resid aliases x
        torch.cuda.synchronize()
        assert torch.equal(a, b) and torch.equal(a, c)
    finally:
        lib.gptoss_moe_layer_destroy(L)


def test_traced_kernel_matches_untraced(lib, config0, tc_impl):
    """gptoss_trace_enable switches to the traced instantiation of the decode kernel (clock64 stamps compiled in):
    its results are bit-identical to the untraced kernel's, and it writes its stamps (slot 0 = start, slot 82 = end,
    per CTA)."""
    d, g = config0
    L = make_layer(lib, d)
    tr = torch.zeros(160 * 160, dtype=torch.int64, device=DEV)
    try:
        x = dev(g["x"][2])
        plain, traced = x.clone(), x.clone()
        ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(plain), None, None))
        ok(lib, lib.gptoss_trace_enable(P(tr), tr.numel() * 8))
        try:
            ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(traced), None, None))
        finally:
            ok(lib, lib.gptoss_trace_enable(None, 0))
        torch.cuda.synchronize()
        assert torch.equal(plain, traced)
        t = tr.view(160, 160).cpu()
        ctas = int((t[:, 0] != 0).sum())
        assert ctas > 0 and bool(((t[:ctas, 82] - t[:ctas, 0]) > 0).all())
    finally:
        lib.gptoss_moe_layer_destroy(L)


def test_layer_create_rejects_bad_shapes(lib, config0):
    d, _ = config0
    L = lib.gptoss_moe_layer_create(P(d["ln"]), 1e-5, P(d["W"]), P(d["b"]), *(P(e) for e in d["ex"]), 32, 9, 2880,
                                    2880, 1.702, 7.0)
    assert not L and b"k <= 8" in lib.gptoss_last_error()


def test_layer_forward_epoch_wraps_past_zero(lib, config0, tc_impl):
    """The decode kernel tags split-tile partial sums with a launch epoch kept in the workspace; epoch 0 is the tag of
    a zero-filled word and must never be current. With the epoch word seeded just below the wrap, the launches run at
    epochs 0xFFFFFFFF, 1 and 2, each bit-identical to an ordinary launch."""
    import ctypes
    d, g = config0
    L = make_layer(lib, d)
    try:
        x = dev(g["x"][0])
        want = x.clone()
        ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(want), None, None))
        torch.cuda.synchronize()
        prev = ctypes.c_uint()
        ok(lib, lib.gptoss_test_decode_epoch(4, 2880, 2880, 0xFFFFFFFE, ctypes.byref(prev)))
        assert prev.value != 0
        for _ in range(3):
            out = x.clone()
            ok(lib, lib.gptoss_moe_layer_forward(L, P(x), P(out), None, None))
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        ok(lib, lib.gptoss_test_decode_epoch(4, 2880, 2880, 5, ctypes.byref(prev)))
        assert prev.value == 2
    finally:
        lib.gptoss_moe_layer_destroy(L)


@pytest.mark.parametrize("which", ["gate_up", "down"])
def test_nan_scale_rejected(lib, config0, which):
    """An E8M0 scale byte 0xFF (NaN) is refused wherever scales enter the tensor-core paths, as the reference's
    loader refuses it (runtime/src/engine.cu:119-122): layer creation, the raw-weights decode entry point (for a
    selected expert) and the batched entry point."""
    d, _ = config0
    ex = list(d["ex"])
    i = 1 if which == "gate_up" else 4
    bad = ex[i].clone()
    bad[17, 123, 45] = 0xFF                               # expert 17
    ex[i] = bad
    L = lib.gptoss_moe_layer_create(P(d["ln"]), 1e-5, P(d["W"]), P(d["b"]), *(P(e) for e in ex), 32, 4, 2880, 2880,
                                    1.702, 7.0)
    assert not L and b"0xFF" in lib.gptoss_last_error()
    x = torch.randn(2880, device=DEV)
    out = torch.zeros(2880, device=DEV)
    w = torch.full((4,), 0.25, device=DEV)
    prev = lib.gptoss_set_moe_impl(1)
    try:
        ids_bad = torch.tensor([2, 17, 5, 9], dtype=torch.int32, device=DEV)
        assert lib.gptoss_kernel_moe(*(P(e) for e in ex), P(x), P(ids_bad), P(w), P(out), 4, 2880, 2880,
                                     1.702, 7.0) != 0
        assert b"0xFF" in lib.gptoss_last_error()
        ids_ok = torch.tensor([2, 16, 5, 9], dtype=torch.int32, device=DEV)   # expert 17 not selected: accepted
        ok(lib, lib.gptoss_kernel_moe(*(P(e) for e in ex), P(x), P(ids_ok), P(w), P(out), 4, 2880, 2880, 1.702, 7.0))
    finally:
        lib.gptoss_set_moe_impl(prev)
    xs = torch.randn(3, 2880, device=DEV)
    ys = torch.zeros_like(xs)
    ids3 = torch.tensor([[2, 17, 5, 9], [0, 1, 2, 3], [4, 5, 6, 7]], dtype=torch.int32, device=DEV)
    w3 = torch.full((3, 4), 0.25, device=DEV)
    assert lib.gptoss_kernel_moe_batched(*(P(e) for e in ex), P(xs), P(ids3), P(w3), P(ys), 3, 4, 2880, 2880, 1.702,
                                         7.0) != 0
    assert b"0xFF" in lib.gptoss_last_error()
