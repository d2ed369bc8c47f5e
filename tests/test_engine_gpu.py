"""The decode engine (gptoss_create / gptoss_step / gptoss_logits / gptoss_score / gptoss_prefill) end to end, on a
small random gpt-oss checkpoint written here in the Hugging Face safetensors layout (64 query heads, 8 key/value
heads, head dim 64; hidden 256, intermediate 128, 8 experts, top-4; 3 layers alternating a 4-key sliding window and
full attention; vocabulary 512).

The reference for the next-token logits is openvang/gptoss-infer's own fp32 forward, Reference.logits of gptoss_ref
(reference/gptoss_ref/model.py:107-134) reading the same checkpoint, with its fp16 KV rounding (kv_dtype), as the
reference runtime's cache holds it. Tolerances, per position: top-1 agreement, KL(reference || engine) <= 1e-5,
max |logit difference| <= 2e-3 * max |reference logit|. The engine's own paths are compared with each other bit for
bit (graph and eager steps, prefill and steps, greedy decoding and the argmax of the logits).
"""
import ctypes
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from gptoss_b200 import capi

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
STAGED = ROOT / "baseline" / "_ref" / "reference"
H, I, E, K, V, LAYERS, WINDOW = 256, 128, 8, 4, 512, 3, 4


def write_checkpoint(d, seed=0):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    n = lambda *s, std=1.0: (torch.randn(*s, generator=g) * std).to(torch.bfloat16)
    t = {"model.embed_tokens.weight": n(V, H), "lm_head.weight": n(V, H, std=0.05),
         "model.norm.weight": (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)}
    for l in range(LAYERS):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
        t[p + "post_attention_layernorm.weight"] = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
        t[p + "self_attn.q_proj.weight"] = n(4096, H, std=0.05)
        t[p + "self_attn.q_proj.bias"] = n(4096, std=0.02)
        t[p + "self_attn.k_proj.weight"] = n(512, H, std=0.05)
        t[p + "self_attn.k_proj.bias"] = n(512, std=0.02)
        t[p + "self_attn.v_proj.weight"] = n(512, H, std=0.05)
        t[p + "self_attn.v_proj.bias"] = n(512, std=0.02)
        t[p + "self_attn.o_proj.weight"] = n(H, 4096, std=0.02)
        t[p + "self_attn.o_proj.bias"] = n(H, std=0.02)
        t[p + "self_attn.sinks"] = n(64)
        t[p + "mlp.router.weight"] = n(E, H, std=0.05)
        t[p + "mlp.router.bias"] = n(E, std=0.02)
        for name, rows, kk in (("gate_up_proj", 2 * I, H), ("down_proj", H, I)):
            q = p + "mlp.experts." + name
            t[q + "_blocks"] = torch.randint(0, 256, (E, rows, kk // 32, 16), generator=g, dtype=torch.uint8)
            t[q + "_scales"] = torch.randint(118, 124, (E, rows, kk // 32), generator=g, dtype=torch.uint8)
            t[q + "_bias"] = n(E, rows, std=0.02)
    save_file(t, str(d / "model.safetensors"))
    cfg = {"num_hidden_layers": LAYERS, "hidden_size": H, "intermediate_size": I, "vocab_size": V,
           "num_local_experts": E, "num_experts_per_tok": K, "sliding_window": WINDOW, "num_attention_heads": 64,
           "num_key_value_heads": 8, "head_dim": 64, "max_position_embeddings": 131072, "rms_norm_eps": 1e-5,
           "swiglu_limit": 7.0, "rope_theta": 150000,
           "layer_types": ["sliding_attention" if l % 2 == 0 else "full_attention" for l in range(LAYERS)],
           "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                            "truncate": False, "original_max_position_embeddings": 4096}}
    (d / "config.json").write_text(json.dumps(cfg))
    (d / "generation_config.json").write_text(json.dumps({"eos_token_id": [1, 2]}))
    return cfg


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    cfg = write_checkpoint(d)
    return d, cfg


@pytest.fixture(scope="module")
def lib():
    return capi.load()


def create(lib, d, max_ctx=64):
    e = lib.gptoss_create(str(d).encode(), max_ctx, 0)
    assert e, lib.gptoss_last_error().decode()
    return e


def engine_logits(lib, e, tokens):
    out = []
    buf = np.empty(V, np.float32)
    for t in tokens:
        assert lib.gptoss_step(e, int(t)) == 0, lib.gptoss_last_error().decode()
        assert lib.gptoss_logits(e, buf.ctypes.data) == 0
        out.append(buf.copy())
    return np.stack(out)


TOKENS = [5, 17, 300, 42, 42, 7, 511, 0, 99, 250, 3, 128]


def test_engine_matches_reference_forward(lib, ckpt):
    if not (STAGED / "gptoss_ref" / "model.py").exists():
        pytest.skip("gptoss_ref is not staged (python oracle/stage_reference.py)")
    d, cfg = ckpt
    e = create(lib, d)
    try:
        assert lib.gptoss_vocab(e) == V
        got = engine_logits(lib, e, TOKENS)
        assert lib.gptoss_position(e) == len(TOKENS)
    finally:
        lib.gptoss_destroy(e)
    if str(STAGED) not in sys.path:
        sys.path.insert(0, str(STAGED))
    from gptoss_ref.config import GptOssConfig
    from gptoss_ref.model import Reference
    from gptoss_ref.weights import SafetensorsWeights
    ref = Reference(GptOssConfig.from_dict(cfg), SafetensorsWeights(d), kv_dtype=torch.float16)
    want = ref.logits(torch.tensor(TOKENS)).numpy().astype(np.float64)
    got = got.astype(np.float64)
    assert np.isfinite(got).all()
    for p in range(len(TOKENS)):
        assert int(np.argmax(got[p])) == int(np.argmax(want[p])), p
        lw = want[p] - np.logaddexp.reduce(want[p])
        lg = got[p] - np.logaddexp.reduce(got[p])
        kl = float(np.sum(np.exp(lw) * (lw - lg)))
        assert kl <= 1e-5, (p, kl)
        assert np.abs(got[p] - want[p]).max() <= 2e-3 * np.abs(want[p]).max(), p


def test_engine_graph_eager_prefill_greedy_and_score(lib, ckpt):
    d, _ = ckpt
    e = create(lib, d)
    try:
        graph = engine_logits(lib, e, TOKENS)
        assert lib.gptoss_reset(e) == 0 and lib.gptoss_use_graph(e, 0) == 0
        eager = engine_logits(lib, e, TOKENS)
        assert np.array_equal(graph, eager)
        assert lib.gptoss_use_graph(e, 1) == 0
        # batched prefill with scoring: the same distributions as the steps (the engine's tolerance for two paths)
        assert lib.gptoss_reset(e) == 0
        n, k = len(TOKENS), 3
        ids = np.array([[1, 2, 3]] * (n - 1), np.int32)
        lp = np.zeros((n - 1, k), np.float32)
        am = np.zeros(n - 1, np.int32)
        tlp = np.zeros(n - 1, np.float32)
        tok = np.array(TOKENS, np.int32)
        assert lib.gptoss_prefill(e, tok.ctypes.data, n, ids.ctypes.data, k, lp.ctypes.data, am.ctypes.data,
                                  tlp.ctypes.data) == 0, lib.gptoss_last_error().decode()
        assert lib.gptoss_position(e) == n
        for p in range(n - 1):
            ls = graph[p].astype(np.float64) - np.logaddexp.reduce(graph[p].astype(np.float64))
            assert am[p] == int(np.argmax(graph[p]))
            np.testing.assert_allclose(lp[p], ls[[1, 2, 3]], rtol=1e-3, atol=2e-3)
            np.testing.assert_allclose(tlp[p], ls[TOKENS[p + 1]], rtol=1e-3, atol=2e-3)
        buf = np.empty(V, np.float32)
        assert lib.gptoss_logits(e, buf.ctypes.data) == 0
        close_logits(buf, graph[-1])
        # score of the current logits
        one = np.array([7, 8], np.int32)
        lp2 = np.zeros(2, np.float32)
        a2, t2, lse = ctypes.c_int(), ctypes.c_float(), ctypes.c_float()
        assert lib.gptoss_score(e, one.ctypes.data, 2, 5, lp2.ctypes.data, ctypes.byref(a2), ctypes.byref(t2),
                                ctypes.byref(lse)) == 0
        l64 = buf.astype(np.float64)
        assert abs(lse.value - np.logaddexp.reduce(l64)) <= 1e-4 * max(1.0, abs(lse.value))
        assert a2.value == int(np.argmax(buf))
        # greedy: each generated token is the argmax of the previous step's logits
        assert lib.gptoss_reset(e) == 0
        out = np.zeros(6, np.int32)
        assert lib.gptoss_generate_greedy(e, TOKENS[0], 6, out.ctypes.data) == 0, lib.gptoss_last_error().decode()
        assert lib.gptoss_reset(e) == 0
        chain = [TOKENS[0]]
        for i in range(6):
            lg = engine_logits(lib, e, [chain[-1]])[0]
            chain.append(int(np.argmax(lg)))
        assert out.tolist() == chain[1:]
        # errors: out-of-range token, full context
        assert lib.gptoss_step(e, V) != 0 and b"token" in lib.gptoss_last_error()
    finally:
        lib.gptoss_destroy(e)


def close_logits(got, want):
    """Two paths of the engine: top-1 agreement, KL(want || got) <= 1e-5, max |difference| <= 2e-3 max |want|."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert int(np.argmax(got)) == int(np.argmax(want))
    lw, lg = want - np.logaddexp.reduce(want), got - np.logaddexp.reduce(got)
    assert float(np.sum(np.exp(lw) * (lw - lg))) <= 1e-5
    assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()


def test_engine_batched_prefill_then_decode(lib, ckpt):
    """A batched prefill longer than the sliding window (12 positions, window 4: the batch's own keys are attended
    before it is appended to the window cache), after two single steps, then three decode steps: every logits vector
    matches the all-steps path, and the reference's n-step loop semantics (positions, cache) carry over."""
    d, _ = ckpt
    e = create(lib, d)
    try:
        want = engine_logits(lib, e, TOKENS + [9, 10, 11])
        assert lib.gptoss_reset(e) == 0
        got = list(engine_logits(lib, e, TOKENS[:2]))
        tok = np.array(TOKENS[2:], np.int32)
        assert lib.gptoss_prefill(e, tok.ctypes.data, len(tok), None, 0, None, None, None) == 0, \
            lib.gptoss_last_error().decode()
        buf = np.empty(V, np.float32)
        assert lib.gptoss_logits(e, buf.ctypes.data) == 0
        got.append(buf.copy())
        got.extend(engine_logits(lib, e, [9, 10, 11]))
        idx = [0, 1, len(TOKENS) - 1, len(TOKENS), len(TOKENS) + 1, len(TOKENS) + 2]
        for g_, i in zip(got, idx):
            close_logits(g_, want[i])
    finally:
        lib.gptoss_destroy(e)


def test_engine_attention_block_impls_agree(lib, ckpt):
    """The decode step's attention block as three launches per layer (default) and as one cooperative launch: the same
    logits to the engine's tolerance for two paths, on the first positions and after a 5000-position random context
    (more keys per range than one pass of the fused kernel stages, window layers wrapped many times)."""
    d, _ = ckpt
    runs = {}
    prev = lib.gptoss_set_attention_impl(0)
    assert prev in (0, 1)
    try:
        for impl in (0, 1):
            assert lib.gptoss_set_attention_impl(impl) in (0, 1)
            e = create(lib, d, max_ctx=5100)
            try:
                first = engine_logits(lib, e, TOKENS[:4])
                assert lib.gptoss_kv_fill_random(e, 5000, 7) == 0, lib.gptoss_last_error().decode()
                late = engine_logits(lib, e, TOKENS[4:8])
                assert lib.gptoss_position(e) == 5004
            finally:
                lib.gptoss_destroy(e)
            runs[impl] = np.concatenate([first, late])
    finally:
        lib.gptoss_set_attention_impl(prev)
    assert np.isfinite(runs[1]).all()
    for a, b in zip(runs[1], runs[0]):
        close_logits(a, b)


def test_engine_budget_and_bad_dir(lib, ckpt, tmp_path):
    d, _ = ckpt
    assert not lib.gptoss_create(str(d).encode(), 64, 1 << 20)
    assert b"budget" in lib.gptoss_last_error()
    assert not lib.gptoss_create(str(tmp_path).encode(), 64, 0)
