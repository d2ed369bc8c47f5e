"""Batched (prefill) MoE path on tensor cores against the CPU oracle.

The batched form of the reference's MoE (gptoss_ref/model.py:100-104): every expert applied to the rows that
selected it, results weighted and added in slot order. Tolerances as the decode tests (the reference's own
test_kernels.py:148-174 bound): allclose rtol 1e-4 / atol 1e-3 against float64, plus max-abs <= 2e-5 * max|ref|.
Router ids must equal the float64 ranking on every token without a near-tie (rel 1e-5). The MoE tests run both
tile plans (stacked: 128 tokens a tile, one MMA per activation term; packed: a token's 8 terms as 8 rows, 16 tokens a
tile), forced through gptoss_set_prefill_packing.

Reduced activation terms (gptoss_set_prefill_terms): with nt terms each 32-value block is the nearest nt-term e2m1
sum, a rounding step of 2^(3 - 3 nt) of the block's scale (nt >= 2), so the output error falls by about 8x per term.
On configs[2]'s input the rel-L2 error against float64 must lie within [0.1, 2] x 8^(1 - nt) (nt = 1: [0.05, 0.5]),
which also shows that each count really runs with that many terms. Only 8 terms meet rtol 1e-4 / atol 1e-3 on
configs[2] (outputs of magnitude ~1e3, so atol 1e-3 is a relative 1e-6); on the input distribution of the
reference's own test_moe_real_shape (runtime/tests/test_kernels.py:148-174, batched here) 7 terms are the fewest
that meet it.
"""
import numpy as np
import pytest
import torch

from gptoss_b200 import capi, synth
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = capi.ptr
PX = "model.layers.0."
EX = PX + "mlp.experts."


def _experts(t):
    return [t[EX + "gate_up_proj_blocks"], t[EX + "gate_up_proj_scales"], t[EX + "gate_up_proj_bias"].float(),
            t[EX + "down_proj_blocks"], t[EX + "down_proj_scales"], t[EX + "down_proj_bias"].float()]


def _ok(lib, rc):
    assert rc == 0, lib.gptoss_last_error().decode()


def _check(got, want):
    got = np.asarray(got, np.float64)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


@pytest.fixture(params=[0, 1], ids=["stacked", "packed"])
def packing(request):
    lib = capi.load()
    prev = lib.gptoss_set_prefill_packing(request.param)
    assert prev >= -1
    yield request.param
    lib.gptoss_set_prefill_packing(prev)


class _Terms:
    """Sets the batched MoE's activation term count for a with-block, restoring it afterwards."""

    def __init__(self, lib, nt):
        self.lib, self.nt = lib, nt

    def __enter__(self):
        self.prev = self.lib.gptoss_set_prefill_terms(self.nt)
        assert self.prev >= 1, self.lib.gptoss_last_error().decode()

    def __exit__(self, *a):
        self.lib.gptoss_set_prefill_terms(self.prev)


def _run_batched(lib, ex_cpu, x, ids, w, resid):
    ex = [e.to(DEV) for e in ex_cpu]
    dx, did, dw, dr = (torch.as_tensor(a).to(DEV).contiguous() for a in (x, ids, w, resid))
    T, k = ids.shape
    _ok(lib, lib.gptoss_kernel_moe_batched(*(P(e) for e in ex), P(dx), P(did), P(dw), P(dr), T, k, 2880, 2880,
                                           1.702, 7.0))
    return dr.cpu().numpy()


def _oracle(ex_cpu, x, ids, w, resid):
    n = [e.numpy() for e in ex_cpu]
    return omoe.moe_batched_f64(*n, x, ids, w, resid)


def _random_routing(T, E, k, seed):
    g = np.random.default_rng(seed)
    ids = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = torch.softmax(torch.from_numpy(g.standard_normal((T, k)).astype(np.float32)), -1).numpy()
    return ids, w


def test_router_batched_exact_ids():
    lib = capi.load()
    t = synth.moe_layer(seed=0)
    W = t[PX + "mlp.router.weight"]
    b = t[PX + "mlp.router.bias"].float()
    x = synth.tokens(512, seed=5).numpy()
    h = omoe.rms_norm(x, t[PX + "post_attention_layernorm.weight"].float().numpy())
    ids = torch.empty(512, 4, dtype=torch.int32, device=DEV)
    w = torch.empty(512, 4, device=DEV)
    dW, db, dh = W.to(DEV), b.to(DEV), torch.from_numpy(h).to(DEV)      # kept alive across the call
    _ok(lib, lib.gptoss_kernel_router_batched(P(dW), P(db), P(dh), 32, 2880, 4, 512, P(ids), P(w)))
    logits = h.astype(np.float64) @ W.float().numpy().astype(np.float64).T + b.numpy().astype(np.float64)
    want = omoe.topk_ids(logits, 4)
    ties = omoe.near_tie_rows(logits, 4)
    got = ids.cpu().numpy()
    assert np.array_equal(got[~ties], want[~ties])
    sel = np.take_along_axis(logits, want, 1)
    ww = np.exp(sel - sel[:, :1])
    ww /= ww.sum(1, keepdims=True)
    np.testing.assert_allclose(w.cpu().numpy()[~ties], ww[~ties], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T", [1, 37])
def test_moe_batched_random_routing(T, packing):
    lib = capi.load()
    t = synth.moe_layer(seed=3, E=8)
    ex = _experts(t)
    g = np.random.default_rng(T)
    x = g.standard_normal((T, 2880)).astype(np.float32)
    resid = g.standard_normal((T, 2880)).astype(np.float32)
    ids, w = _random_routing(T, 8, 4, T + 1)
    _check(_run_batched(lib, ex, x, ids, w, resid), _oracle(ex, x, ids, w, resid))


def test_moe_batched_skewed(packing):
    """Every token picks experts 0..3 (in varying order): 50 rows per expert, several M tiles, a partial last tile."""
    lib = capi.load()
    t = synth.moe_layer(seed=4, E=4)
    ex = _experts(t)
    g = np.random.default_rng(2)
    T = 50
    x = g.standard_normal((T, 2880)).astype(np.float32)
    resid = np.zeros((T, 2880), np.float32)
    ids = np.stack([g.permutation(4) for _ in range(T)]).astype(np.int32)
    w = np.full((T, 4), 0.25, np.float32)
    _check(_run_batched(lib, ex, x, ids, w, resid), _oracle(ex, x, ids, w, resid))


def test_layer_forward_batched_matches_decode_and_oracle(packing):
    """Prepared layer, 20 tokens: the batched forward (RMSNorm + router + MoE) agrees with the float64 oracle on the
    oracle's routing, with the per-token decode kernel, and is deterministic."""
    lib = capi.load()
    t = synth.moe_layer(seed=0)
    d = {k_: v.to(DEV) for k_, v in t.items()}
    ln = d[PX + "post_attention_layernorm.weight"].float()
    W, b = d[PX + "mlp.router.weight"], d[PX + "mlp.router.bias"].float()
    ex = [e.to(DEV) for e in _experts(t)]
    L = lib.gptoss_moe_layer_create(P(ln), 1e-5, P(W), P(b), *(P(e) for e in ex), 32, 4, 2880, 2880, 1.702, 7.0)
    assert L, lib.gptoss_last_error().decode()
    try:
        T = 20
        x = synth.tokens(T, seed=8)
        xb = x.to(DEV).contiguous()
        outs = []
        for _ in range(2):
            y = xb.clone()
            _ok(lib, lib.gptoss_moe_layer_forward_batched(L, P(xb), P(y), T, None, None))
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy())
        assert np.array_equal(outs[0], outs[1])
        dec = []
        for i in range(T):
            y = xb[i].clone()
            _ok(lib, lib.gptoss_moe_layer_forward(L, P(xb[i]), P(y), None, None))
            dec.append(y)
        torch.cuda.synchronize()
        dec = torch.stack(dec).cpu().numpy()
        # oracle on its own float64 routing
        xn = x.numpy()
        h = omoe.rms_norm(xn, t[PX + "post_attention_layernorm.weight"].float().numpy())
        logits = h.astype(np.float64) @ t[PX + "mlp.router.weight"].float().numpy().astype(np.float64).T + \
            t[PX + "mlp.router.bias"].float().numpy().astype(np.float64)
        ids = omoe.topk_ids(logits, 4)
        assert not omoe.near_tie_rows(logits, 4).any()
        sel = np.take_along_axis(logits, ids, 1)
        w = np.exp(sel - sel[:, :1])
        w = (w / w.sum(1, keepdims=True)).astype(np.float32)
        want = _oracle(_experts(t), h, ids.astype(np.int32), w, xn)
        _check(outs[0], want)
        _check(dec, want)
    finally:
        lib.gptoss_moe_layer_destroy(L)


def test_layer_forward_batched_config2_2048_zipf():
    """configs[2] at full size: 2048 bf16 N(0,1) tokens, router bias skewed towards Zipf s=1.1 (per-expert row counts
    from a few tens to the 2048 cap, so every M-tile shape occurs). The whole batch runs through the prepared layer,
    in both tile plans; the expert ids of every token equal the float64 ranking (except near-ties), 48 sampled rows
    (the most and least loaded experts' tokens included) meet the float64 oracle's bound in both plans, and two runs
    of a plan are bit-identical."""
    lib = capi.load()
    T = 2048
    t, x, L, W, b = _config2_layer(lib, T)
    try:
        xb = x.to(DEV).contiguous()
        plans = {}
        for pack in (0, 1):
            prev = lib.gptoss_set_prefill_packing(pack)
            try:
                outs = [_forward(lib, L, xb, T) for _ in range(2)]
            finally:
                lib.gptoss_set_prefill_packing(prev)
            assert np.array_equal(outs[0], outs[1])
            plans[pack] = outs[0]
    finally:
        lib.gptoss_moe_layer_destroy(L)
    rows, ids, ties, want, scale = _config2_reference(lib, t, x, W, b, T)
    for pack, out in plans.items():
        got = np.asarray(out[rows], np.float64)
        # The skewed routing gives rows of magnitude ~1e3; fp32 accumulation error scales with the terms, so the
        # absolute part of the element-wise bound is taken relative to the largest output (1e-6 of it; 1e-3 at 1e3).
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6 * scale, err_msg=f"pack={pack}")
        assert np.abs(got - want).max() <= 2e-5 * scale
        assert np.linalg.norm(got - want) <= 2e-5 * np.linalg.norm(want)


def _config2_layer(lib, T):
    t = synth.moe_layer(seed=0)
    synth.zipf_router_bias(t, s=1.1, beta=1.0, seed=7)
    x = torch.randn(T, 2880, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).float()
    d = {k_: v.to(DEV) for k_, v in t.items()}
    ln = d[PX + "post_attention_layernorm.weight"].float()
    W, b = d[PX + "mlp.router.weight"], d[PX + "mlp.router.bias"].float()
    ex = [e.to(DEV) for e in _experts(t)]
    L = lib.gptoss_moe_layer_create(P(ln), 1e-5, P(W), P(b), *(P(e) for e in ex), 32, 4, 2880, 2880, 1.702, 7.0)
    assert L, lib.gptoss_last_error().decode()
    _config2_layer.keep = (d, ex)                    # device tensors stay referenced while the layer lives
    return t, x, L, W, b


def _forward(lib, L, xb, T):
    y = xb.clone()
    _ok(lib, lib.gptoss_moe_layer_forward_batched(L, P(xb), P(y), T, None, None))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _config2_reference(lib, t, x, W, b, T):
    """Sampled rows of configs[2] and their float64 oracle outputs (plus the library's ids checked on the batch)."""
    xn = x.numpy()
    h = omoe.rms_norm(xn, t[PX + "post_attention_layernorm.weight"].float().numpy())
    logits = h.astype(np.float64) @ t[PX + "mlp.router.weight"].float().numpy().astype(np.float64).T + \
        t[PX + "mlp.router.bias"].float().numpy().astype(np.float64)
    ids = omoe.topk_ids(logits, 4)
    ties = omoe.near_tie_rows(logits, 4)
    counts = np.bincount(ids.reshape(-1), minlength=32)
    assert counts.max() > 8 * max(1, counts.min()), counts          # the routing is skewed
    # the library's own ids for the whole batch
    dh = torch.from_numpy(h).to(DEV).contiguous()
    gid = torch.empty(T, 4, dtype=torch.int32, device=DEV)
    gw = torch.empty(T, 4, device=DEV)
    _ok(lib, lib.gptoss_kernel_router_batched(P(W), P(b), P(dh), 32, 2880, 4, T, P(gid), P(gw)))
    assert np.array_equal(gid.cpu().numpy()[~ties], ids[~ties])
    hot, cold = int(np.argmax(counts)), int(np.argmin(np.where(counts > 0, counts, T * 4)))
    rows = set(np.random.default_rng(3).choice(T, 40, replace=False).tolist())
    rows |= set(np.nonzero((ids == cold).any(1))[0][:4].tolist()) | set(np.nonzero((ids == hot).any(1))[0][:4].tolist())
    rows = np.array(sorted(r for r in rows if not ties[r]))
    sel = np.take_along_axis(logits[rows], ids[rows], 1)
    w = np.exp(sel - sel[:, :1])
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    want = _oracle(_experts(t), h[rows], ids[rows].astype(np.int32), w, xn[rows])
    return rows, ids, ties, want, np.abs(want).max()


def test_prefill_term_variants_config2():
    """configs[2] with 1 .. 8 activation terms (stacked plan, and the packed plan at 4 and 8): the rel-L2 error of the
    sampled rows against float64 lies within [0.1, 2] x 8^(1 - nt) ([0.05, 0.5] for nt = 1); the measured errors are
    printed (pytest -s) for the record."""
    lib = capi.load()
    T = 2048
    t, x, L, W, b = _config2_layer(lib, T)
    outs = {}
    try:
        xb = x.to(DEV).contiguous()
        for nt, pack in [(n, 0) for n in range(1, 9)] + [(4, 1), (8, 1)]:
            prev = lib.gptoss_set_prefill_packing(pack)
            try:
                with _Terms(lib, nt):
                    outs[(nt, pack)] = _forward(lib, L, xb, T)
            finally:
                lib.gptoss_set_prefill_packing(prev)
    finally:
        lib.gptoss_moe_layer_destroy(L)
    rows, ids, ties, want, scale = _config2_reference(lib, t, x, W, b, T)
    for (nt, pack), out in outs.items():
        got = np.asarray(out[rows], np.float64)
        assert np.isfinite(got).all()
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        mx = np.abs(got - want).max() / scale
        print(f"terms {nt} pack {pack}: rel-L2 {rel:.3e}  max-abs/max {mx:.3e}")
        lo, hi = (0.05, 0.5) if nt == 1 else (0.1 * 8.0 ** (1 - nt), 2 * 8.0 ** (1 - nt))
        if nt == 8:
            lo = 0.0                                   # exact up to fp32 accumulation
        assert lo <= rel <= hi, (nt, pack, rel)


def test_prefill_fewest_terms_reference_bound():
    """The input distribution of the reference's test_moe_real_shape (E = 6, scale bytes 118..123, biases N(0, 0.1),
    x and the residual N(0, 1)), 64 tokens with random routing: 7 terms meet rtol 1e-4 / atol 1e-3 against float64,
    6 do not (so 7 is the fewest terms that meet the reference's bound), and 8 (the default) meets it."""
    lib = capi.load()
    g = torch.Generator().manual_seed(4)
    E, H, I, k, T = 6, 2880, 2880, 4, 64
    gu_b = torch.randint(0, 256, (E, 2 * I, H // 32, 16), generator=g, dtype=torch.uint8)
    gu_s = torch.randint(118, 124, (E, 2 * I, H // 32), generator=g, dtype=torch.uint8)
    dn_b = torch.randint(0, 256, (E, H, I // 32, 16), generator=g, dtype=torch.uint8)
    dn_s = torch.randint(118, 124, (E, H, I // 32), generator=g, dtype=torch.uint8)
    gu_bias, dn_bias = torch.randn(E, 2 * I, generator=g) * 0.1, torch.randn(E, H, generator=g) * 0.1
    x = torch.randn(T, H, generator=g).numpy()
    resid = torch.randn(T, H, generator=g).numpy()
    ids, w = _random_routing(T, E, k, 5)
    ex = [gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias]
    want = _oracle(ex, x, ids, w, resid)
    for nt in (6, 7, 8):
        with _Terms(lib, nt):
            got = np.asarray(_run_batched(lib, ex, x, ids, w, resid), np.float64)
        viol = np.mean(np.abs(got - want) > 1e-3 + 1e-4 * np.abs(want))
        print(f"terms {nt}: max-abs {np.abs(got - want).max():.3e}, share outside the bound {viol:.4f}")
        if nt == 6:
            assert viol > 0, "6 terms unexpectedly meet the bound"
        else:
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)
