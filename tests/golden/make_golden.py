"""Generates the golden fixtures in this folder by running openvang/gptoss-infer's own fp32 reference.

Run here, where the reference is importable (it does not exist on the GPU box, so the outputs are committed):

    GPTOSS_REF_ROOT=/path/to/gptoss-infer python tests/golden/make_golden.py

(GPTOSS_REF_ROOT defaults to a sibling checkout named `reference` next to this repository.)

Fixtures (numpy .npz, small enough to commit):
  mxfp4_kat.npz     outputs of gptoss_ref.mxfp4.dequant / quantize on the inputs of the reference's own
                    known-answer tests (reference/tests/test_mxfp4.py:17-62): random blocks, every code and
                    nibble order, scale extremes, all 255 valid scales, quantize round trip.
  tiny_moe.npz      Reference.moe (reference/gptoss_ref/model.py:92-105) on a tiny gpt-oss MoE layer (H=64, I=32,
                    8 experts, top-4, the shapes of reference/tests/conftest.py:29-37) for 9 tokens: all inputs and
                    the output, with the selected expert ids.
  config0_moe.npz   Reference.moe at the real shape (H=I=2880, 32 experts, top-4) on 4 tokens of the seeded
                    config-0 layer from gptoss_b200.synth (seed 0, tokens seed 1). The 423 MB of weights are not
                    stored: the fixture keeps their sha256 so a test can regenerate them and prove they are the
                    same bytes, plus the normed input, the output and the expert ids.
"""
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "gptoss-infer_b200"))
sys.path.insert(0, str(Path(os.environ.get("GPTOSS_REF_ROOT", ROOT.parent / "reference")) / "reference"))

from gptoss_ref import model as ref_model  # noqa: E402
from gptoss_ref import mxfp4 as ref_mxfp4  # noqa: E402
from gptoss_ref.config import GptOssConfig  # noqa: E402
from gptoss_ref.weights import DictWeights  # noqa: E402

from gptoss_b200 import synth  # noqa: E402


def cfg_for(H, I, E, k):
    return GptOssConfig.from_dict({
        "vocab_size": 97, "hidden_size": H, "intermediate_size": I, "num_hidden_layers": 1,
        "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 16, "num_local_experts": E,
        "num_experts_per_tok": k, "sliding_window": 6, "layer_types": ["sliding_attention"],
        "rms_norm_eps": 1e-5, "rope_theta": 150000.0, "swiglu_limit": 7.0,
        "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                         "truncate": False, "original_max_position_embeddings": 4096}})


def mxfp4_kat():
    out = {}
    g = torch.Generator().manual_seed(1)
    b = torch.randint(0, 256, (3, 5, 4, 16), generator=g, dtype=torch.uint8)
    s = torch.randint(100, 150, (3, 5, 4), generator=g, dtype=torch.uint8)
    out |= {"rand_blocks": b.numpy(), "rand_scales": s.numpy(), "rand_out": ref_mxfp4.dequant(b, s).numpy()}
    b = torch.zeros(1, 16, dtype=torch.uint8)
    b[0, 0] = 0x21
    out["nibble_out"] = ref_mxfp4.dequant(b, torch.tensor([127], dtype=torch.uint8)).numpy()
    codes = torch.arange(16, dtype=torch.uint8)
    b = (codes[0::2] | (codes[1::2] << 4)).reshape(1, 8).repeat(1, 2)
    out["codes_blocks"] = b.numpy()
    out["codes_out"] = ref_mxfp4.dequant(b, torch.tensor([128], dtype=torch.uint8)).numpy()
    b = torch.full((1, 16), 0x77, dtype=torch.uint8)
    out["ext_lo_out"] = ref_mxfp4.dequant(b, torch.tensor([1], dtype=torch.uint8)).numpy()
    out["ext_hi_out"] = ref_mxfp4.dequant(b, torch.tensor([254], dtype=torch.uint8)).numpy()
    b = torch.full((255, 1, 16), 0x22, dtype=torch.uint8)
    s = torch.arange(255, dtype=torch.uint8).reshape(255, 1)
    out["allscale_out"] = ref_mxfp4.dequant(b, s).numpy()
    g = torch.Generator().manual_seed(2)
    b = torch.randint(0, 256, (4, 3, 16), generator=g, dtype=torch.uint8)
    s = torch.randint(110, 130, (4, 3), generator=g, dtype=torch.uint8)
    w = ref_mxfp4.dequant(b, s)
    qb, qs = ref_mxfp4.quantize(w)
    out |= {"rt_w": w.numpy(), "rt_blocks": qb.numpy(), "rt_scales": qs.numpy()}
    # Gaussian weights through quantize: exercises the rounding rule, not only exact grid points.
    g = torch.Generator().manual_seed(3)
    w = torch.randn(6, 64, generator=g) * 0.3
    qb, qs = ref_mxfp4.quantize(w)
    out |= {"gq_w": w.numpy(), "gq_blocks": qb.numpy(), "gq_scales": qs.numpy()}
    np.savez_compressed(HERE / "mxfp4_kat.npz", **out)


def run_moe(t, x, H, I, E, k, prefix="model.layers.0."):
    cfg = cfg_for(H, I, E, k)
    ref = ref_model.Reference(cfg, DictWeights(t))
    w = t[prefix + "post_attention_layernorm.weight"].to(torch.float32)
    h = ref_model.rms_norm(x, w, cfg.rms_norm_eps)
    with torch.inference_mode():
        out, top_idx = ref.moe(0, h, return_routing=True)
    return h, out, top_idx


def tiny_moe():
    H, I, E, k, T = 64, 32, 8, 4, 9
    t = synth.moe_layer(seed=11, H=H, I=I, E=E, scale_lo=120, scale_hi=123)
    x = synth.tokens(T, seed=12, H=H)
    h, out, top_idx = run_moe(t, x, H, I, E, k)
    arrays = {k_.replace(".", "__"): v for k_, v in synth.to_numpy(t).items()}
    np.savez_compressed(HERE / "tiny_moe.npz", x=x.numpy(), h=h.numpy(), out=out.numpy(),
                        top_idx=top_idx.numpy().astype(np.int32), **arrays)


def config0_moe():
    T = 4
    t = synth.moe_layer(seed=0)
    x = synth.tokens(T, seed=1)
    h, out, top_idx = run_moe(t, x, synth.H, synth.I, synth.E, synth.K_TOP)
    np.savez_compressed(HERE / "config0_moe.npz", weights_sha256=np.array(synth.digest(t)),
                        x=x.numpy(), h=h.numpy(), out=out.numpy(), top_idx=top_idx.numpy().astype(np.int32))


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count())
    mxfp4_kat()
    tiny_moe()
    config0_moe()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
