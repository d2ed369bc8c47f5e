"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

There is no checkpoint or dataset on the GPU box, so every weight is random-init with gpt-oss-20b's shapes and the
checkpoint's Hugging Face tensor names (the names runtime/src/engine.cu:155-162 of openvang/gptoss-infer loads):

  mlp.router.weight                 bf16 [E, H]            N(0, 0.02)
  mlp.router.bias                   bf16 [E]               N(0, 0.01)
  mlp.experts.gate_up_proj_blocks   uint8 [E, 2I, H/32, 16] uniform 0..255 (every e2m1 code equally likely)
  mlp.experts.gate_up_proj_scales   uint8 [E, 2I, H/32]    uniform 120..126 (E8M0, bias 127)
  mlp.experts.gate_up_proj_bias     bf16 [E, 2I]           N(0, 0.01)
  mlp.experts.down_proj_blocks      uint8 [E, H, I/32, 16] uniform 0..255
  mlp.experts.down_proj_scales      uint8 [E, H, I/32]     uniform 120..126
  mlp.experts.down_proj_bias        bf16 [E, H]            N(0, 0.01)
  post_attention_layernorm.weight   bf16 [H]               1 + N(0, 0.02)

The generator is torch's CPU generator (mt19937) seeded per call, so the same seed gives the same bytes on every
machine with this torch version; tests/golden records hashes of the generated tensors to detect drift.
"""
import hashlib

import numpy as np
import torch

H, I, E, K_TOP = 2880, 2880, 32, 4
ALPHA, LIMIT, EPS = 1.702, 7.0, 1e-5


def moe_layer(seed=0, H=H, I=I, E=E, prefix="model.layers.0.", scale_lo=120, scale_hi=126):
    """One MoE layer's tensors (HF names) plus its RMSNorm weight, generated in a fixed order from `seed`."""
    g = torch.Generator().manual_seed(seed)
    n = lambda *s, std: (torch.randn(*s, generator=g) * std)
    t = {}
    t[prefix + "post_attention_layernorm.weight"] = (1 + n(H, std=0.02)).to(torch.bfloat16)
    t[prefix + "mlp.router.weight"] = n(E, H, std=0.02).to(torch.bfloat16)
    t[prefix + "mlp.router.bias"] = n(E, std=0.01).to(torch.bfloat16)
    p = prefix + "mlp.experts."
    for name, rows, k in (("gate_up_proj", 2 * I, H), ("down_proj", H, I)):
        t[p + name + "_blocks"] = torch.randint(0, 256, (E, rows, k // 32, 16), generator=g, dtype=torch.uint8)
        t[p + name + "_scales"] = torch.randint(scale_lo, scale_hi + 1, (E, rows, k // 32), generator=g,
                                                dtype=torch.uint8)
        t[p + name + "_bias"] = n(E, rows, std=0.01).to(torch.bfloat16)
    return t


def tokens(T, seed=1, H=H):
    """Residual-stream input x fp32 [T, H] ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, H, generator=g)


def zipf_router_bias(t, prefix="model.layers.0.", s=1.1, beta=1.0, seed=7):
    """Skews routing: router bias += beta * log p_e with p_e ~ rank^-s over a seeded permutation of the experts.

    Returns the permutation (hottest expert first). The realised per-expert counts are measured, not assumed."""
    w = t[prefix + "mlp.router.bias"]
    n_exp = w.shape[0]
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_exp, generator=g)
    p = torch.arange(1, n_exp + 1, dtype=torch.float64) ** (-s)
    p = p / p.sum()
    shift = torch.empty(n_exp, dtype=torch.float64)
    shift[perm] = beta * torch.log(p)
    t[prefix + "mlp.router.bias"] = (w.double() + shift).to(torch.bfloat16)
    return perm


def to_numpy(t):
    """HF tensors -> numpy (bf16 upcast to fp32 exactly; uint8 kept)."""
    out = {}
    for k, v in t.items():
        out[k] = v.numpy() if v.dtype == torch.uint8 else v.to(torch.float32).numpy()
    return out


def digest(t):
    """sha256 over the tensors' names, dtypes, shapes and raw bytes, in sorted name order."""
    h = hashlib.sha256()
    for k in sorted(t):
        v = t[k].contiguous()
        h.update(k.encode())
        h.update(str(v.dtype).encode())
        h.update(str(tuple(v.shape)).encode())
        raw = v.view(torch.uint8) if v.dtype != torch.uint8 else v
        h.update(np.ascontiguousarray(raw.numpy()).tobytes())
    return h.hexdigest()


def ep_router(layer, H=H, E=E, zipf_s=1.2, beta=1.0):
    """The RMSNorm weight and router of layer `layer` of the expert-parallel benchmark model (CPU generator, seed
    10_000 + layer, the moe_layer distributions), with the router bias skewed towards Zipf `zipf_s` over a seeded
    expert order (seed 20_000 + layer). Identical on every rank. Returns (ln fp32, W bf16, b fp32)."""
    g = torch.Generator().manual_seed(10_000 + layer)
    ln = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16).float()
    W = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(E, generator=g) * 0.01).to(torch.bfloat16)
    t = {"r.mlp.router.bias": b}
    zipf_router_bias(t, prefix="r.", s=zipf_s, beta=beta, seed=20_000 + layer)
    return ln, W, t["r.mlp.router.bias"].float()


def ep_experts(layer, e0, e1, device, H=H, I=I, scale_lo=120, scale_hi=126):
    """Experts e0..e1-1 of layer `layer` of the expert-parallel benchmark model, drawn on `device` expert by expert
    from a generator seeded by (layer, expert), so every split of the experts over ranks holds the same weights.
    Returns [gu_blocks, gu_scales, gu_bias fp32, dn_blocks, dn_scales, dn_bias fp32], experts stacked on dim 0."""
    return ep_experts_of(layer, range(e0, e1), device, H, I, scale_lo, scale_hi)


def ep_experts_of(layer, experts, device, H=H, I=I, scale_lo=120, scale_hi=126):
    """ep_experts for any list of expert ids (stacked in the list's order): a rank's experts under a placement."""
    parts = [[] for _ in range(6)]
    for e in experts:
        g = torch.Generator(device=device).manual_seed(1_000_003 * (layer + 1) + 7_919 * e)
        for j, (rows, k) in enumerate(((2 * I, H), (H, I))):
            parts[3 * j].append(torch.randint(0, 256, (rows, k // 32, 16), generator=g, device=device,
                                              dtype=torch.uint8))
            parts[3 * j + 1].append(torch.randint(scale_lo, scale_hi + 1, (rows, k // 32), generator=g,
                                                  device=device, dtype=torch.uint8))
            parts[3 * j + 2].append((torch.randn(rows, generator=g, device=device) * 0.01).to(torch.bfloat16).float())
    return [torch.stack(p).contiguous() for p in parts]
