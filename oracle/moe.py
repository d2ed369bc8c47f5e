"""CPU oracle (test infrastructure only): the gpt-oss MoE block restated in numpy.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this module; it is the checker,
never the thing measured as the product or shipped.

Restates openvang/gptoss-infer:
  * rms_norm          reference/gptoss_ref/model.py:21-22
  * swiglu            reference/gptoss_ref/model.py:25-30  (even rows glu clamped above at `limit`, odd rows
                      linear clamped to [-limit, limit]; glu * sigmoid(alpha * glu) * (lin + 1))
  * router            reference/gptoss_ref/model.py:95-98  (logits = h W^T + b in fp32; top-k sorted by logit,
                      ties to the lower expert id as runtime/src/kernels.cu:307-324 specifies, NaN never wins;
                      softmax over the k selected logits)
  * moe               reference/gptoss_ref/model.py:92-105 (Reference.moe: loop over the unique selected experts
                      in ascending id, dequantize each expert per call, index_add of gate-weighted outputs)
  * kernel_moe_f64    runtime/include/gptoss/gptoss.h:54-58 semantics of gptoss_kernel_moe, in float64, the
                      way runtime/tests/test_kernels.py:300-307 states it
  * router_f64        runtime/tests/test_kernels.py:274-278 (float64 logits, sorted by (-logit, id))
Weights use the checkpoint's Hugging Face names (runtime/src/engine.cu:155-162).
"""
import numpy as np

from . import mxfp4


def rms_norm(x, weight, eps=1e-5):
    x = np.asarray(x, dtype=np.float32)
    r = np.float32(1.0) / np.sqrt((x * x).mean(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
    return (x * r * np.asarray(weight, dtype=np.float32)).astype(np.float32)


def swiglu(t, alpha=1.702, limit=7.0):
    glu, lin = t[..., 0::2], t[..., 1::2]
    dt = t.dtype
    glu = np.minimum(glu, dt.type(limit))
    lin = np.clip(lin, dt.type(-limit), dt.type(limit))
    with np.errstate(over="ignore"):                   # exp overflow -> sigmoid 0, as torch.sigmoid saturates
        return glu * (dt.type(1) / (dt.type(1) + np.exp(-dt.type(alpha) * glu))) * (lin + dt.type(1))


def topk_ids(logits, k):
    """Top-k expert ids per row, sorted by logit descending, ties to the lower id, NaN never selected first."""
    lg = np.asarray(logits, dtype=np.float64)
    lg = np.where(np.isnan(lg), -np.inf, lg)
    E = lg.shape[-1]
    ids = np.broadcast_to(np.arange(E), lg.shape)
    order = np.lexsort((ids, -lg), axis=-1)                    # primary key -logit, secondary key id
    return order[..., :k].astype(np.int32)


def softmax(v, axis=-1):
    m = v.max(axis=axis, keepdims=True)
    e = np.exp(v - m)
    return e / e.sum(axis=axis, keepdims=True)


def router(h, router_w, router_b, k):
    """fp32 router as Reference.moe computes it: returns (logits [T,E], ids [T,k] int32, gate [T,k] fp32)."""
    h = np.asarray(h, dtype=np.float32)
    logits = h @ np.asarray(router_w, dtype=np.float32).T + np.asarray(router_b, dtype=np.float32)
    ids = topk_ids(logits, k)
    top = np.take_along_axis(logits, ids, axis=-1)
    return logits, ids, softmax(top).astype(np.float32)


def expert(t, prefix, e):
    """(w1 [2I,H], b1 [2I], w2 [H,I], b2 [H]) in fp32 for expert e, dequantized per call (weights.py:35-47)."""
    p = prefix + "mlp.experts."
    w1 = mxfp4.dequant(t[p + "gate_up_proj_blocks"][e], t[p + "gate_up_proj_scales"][e])
    w2 = mxfp4.dequant(t[p + "down_proj_blocks"][e], t[p + "down_proj_scales"][e])
    b1 = np.asarray(t[p + "gate_up_proj_bias"][e], dtype=np.float32)
    b2 = np.asarray(t[p + "down_proj_bias"][e], dtype=np.float32)
    return w1, b1, w2, b2


def moe(t, prefix, h, k=4, alpha=1.702, limit=7.0, return_routing=False):
    """Reference.moe on normed tokens h [T,H] (model.py:92-105), fp32 throughout."""
    h = np.asarray(h, dtype=np.float32)
    logits, ids, gate = router(h, t[prefix + "mlp.router.weight"], t[prefix + "mlp.router.bias"], k)
    out = np.zeros_like(h)
    for e in np.unique(ids).tolist():
        rows, slot = np.nonzero(ids == e)
        w1, b1, w2, b2 = expert(t, prefix, e)
        y = swiglu(h[rows] @ w1.T + b1, alpha, limit) @ w2.T + b2
        np.add.at(out, rows, y * gate[rows, slot][:, None])
    return (out, ids, gate, logits) if return_routing else out


def router_f64(W, b, x, k):
    """Float64 logits and the (-logit, id) sort rule of runtime/tests/test_kernels.py:274-278."""
    logits = np.asarray(W, dtype=np.float64) @ np.asarray(x, dtype=np.float64) + np.asarray(b, dtype=np.float64)
    ids = topk_ids(logits, k)
    return logits, ids, softmax(logits[ids])


def kernel_moe_f64(gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias, x, ids, weights, resid, alpha=1.702, limit=7.0):
    """x_resid + sum_slot w[slot] (W2[e] swiglu(W1[e] x + b1[e]) + b2[e]) in float64 (gptoss.h:54-58)."""
    out = np.asarray(resid, dtype=np.float64).copy()
    x = np.asarray(x, dtype=np.float64)
    for slot, e in enumerate(np.asarray(ids).tolist()):
        w1 = mxfp4.dequant(gu_b[e], gu_s[e]).astype(np.float64)
        w2 = mxfp4.dequant(dn_b[e], dn_s[e]).astype(np.float64)
        a = swiglu(w1 @ x + np.asarray(gu_bias[e], dtype=np.float64), alpha, limit)
        out += float(weights[slot]) * (w2 @ a + np.asarray(dn_bias[e], dtype=np.float64))
    return out


def moe_batched_f64(gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias, x, ids, weights, resid, alpha=1.702, limit=7.0):
    """Batched form: resid[t] + sum_slot w[t,slot] (W2[e] swiglu(W1[e] x[t] + b1[e]) + b2[e]), float64.

    Experts are decoded once each and applied to the rows that selected them, as Reference.moe does."""
    x = np.asarray(x, dtype=np.float64)
    ids = np.asarray(ids)
    w = np.asarray(weights, dtype=np.float64)
    out = np.asarray(resid, dtype=np.float64).copy()
    for e in np.unique(ids).tolist():
        rows, slot = np.nonzero(ids == e)
        w1 = mxfp4.dequant(gu_b[e], gu_s[e]).astype(np.float64)
        w2 = mxfp4.dequant(dn_b[e], dn_s[e]).astype(np.float64)
        a = swiglu(x[rows] @ w1.T + np.asarray(gu_bias[e], dtype=np.float64), alpha, limit)
        y = a @ w2.T + np.asarray(dn_bias[e], dtype=np.float64)
        np.add.at(out, rows, y * w[rows, slot][:, None])
    return out


def near_tie_rows(logits, k, rel=1e-5):
    """Rows whose k-th and (k+1)-th largest logits are closer than rel * |k-th logit| (routing near-ties)."""
    lg = np.sort(np.asarray(logits, dtype=np.float64), axis=-1)[..., ::-1]
    if lg.shape[-1] <= k:
        return np.zeros(lg.shape[:-1], dtype=bool)
    gap = lg[..., k - 1] - lg[..., k]
    return gap <= rel * np.abs(lg[..., k - 1])
