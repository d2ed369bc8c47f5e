"""Expert-parallel dispatch/combine (gptoss_b200/ep.py) on CPU: two gloo ranks, a small MoE layer, routing and
expert compute from the float64 oracle; the sharded result must equal the single-process float64 batched MoE
(reference gptoss_ref/model.py:100-104 semantics) to 1e-12 relative, including a step where one rank receives no
rows at all."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, I, E, K = 64, 32, 4, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "gptoss-infer_b200")]
    from gptoss_b200 import synth
    return synth.to_numpy(synth.moe_layer(seed=21, H=H, I=I, E=E))


def _oracle_parts(t):
    from oracle import moe as omoe
    p = "model.layers.0."
    ex = p + "mlp.experts."
    n = [t[ex + "gate_up_proj_blocks"], t[ex + "gate_up_proj_scales"], t[ex + "gate_up_proj_bias"],
         t[ex + "down_proj_blocks"], t[ex + "down_proj_scales"], t[ex + "down_proj_bias"]]
    W, b, g = t[p + "mlp.router.weight"], t[p + "mlp.router.bias"], t[p + "post_attention_layernorm.weight"]
    return omoe, n, W, b, g


def _worker(rank, world, port, x_all, force_rank0, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = _layer()
        from gptoss_b200 import ep
        omoe, n, W, b, g = _oracle_parts(t)
        El = E // world

        def route(x):
            h = omoe.rms_norm(x.numpy().astype(np.float32), g).astype(np.float64)   # fp32 norm, as the reference
            logits = h @ np.asarray(W, np.float64).T + np.asarray(b, np.float64)
            if force_rank0:
                logits[:, El:] -= 1e3                       # everything goes to rank 0's experts
            ids = omoe.topk_ids(logits, K)
            sel = np.take_along_axis(logits, ids, 1)
            w = np.exp(sel - sel[:, :1])
            w /= w.sum(1, keepdims=True)
            return torch.from_numpy(h), torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w)

        def compute(h_rows, lids, w):
            ids_g = lids.numpy().astype(np.int64)[:, None] + rank * El
            zero = np.zeros(h_rows.shape, np.float64)
            y = omoe.moe_batched_f64(*n, h_rows.numpy(), ids_g, w.numpy()[:, None], zero)
            return torch.from_numpy(y)

        layer = ep.ExpertParallelMoE(route, compute, rank, world, E, K, H)
        shard = torch.from_numpy(x_all[rank::world].astype(np.float64)).clone()
        out = layer.forward(shard)
        out_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def _reference(x_all, force_rank0, world):
    t = _layer()
    omoe, n, W, b, g = _oracle_parts(t)
    h = omoe.rms_norm(x_all, g).astype(np.float64)
    logits = h @ np.asarray(W, np.float64).T + np.asarray(b, np.float64)
    if force_rank0:
        logits[:, E // world:] -= 1e3
    ids = omoe.topk_ids(logits, K)
    sel = np.take_along_axis(logits, ids, 1)
    w = np.exp(sel - sel[:, :1])
    w /= w.sum(1, keepdims=True)
    return omoe.moe_batched_f64(*n, h, ids, w, x_all.astype(np.float64))


@pytest.mark.parametrize("force_rank0", [False, True])
def test_ep_two_ranks_matches_single_process(force_rank0):
    world = 2
    x_all = np.random.default_rng(5).standard_normal((12, H)).astype(np.float32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, x_all, force_rank0, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out = np.empty((12, H), np.float64)
    for r in range(world):
        out[r::world] = got[r]
    want = _reference(x_all, force_rank0, world)
    np.testing.assert_allclose(out, want, rtol=1e-12, atol=1e-12)


def test_balanced_placement_properties():
    """Expert placement by expected load: every expert placed once, E / world per rank, each rank's list ascending,
    and on the benchmark's Zipf-skewed loads the busiest rank carries no more than the contiguous placement's."""
    from gptoss_b200 import ep
    g = torch.Generator().manual_seed(3)
    for world in (1, 2, 4, 8):
        loads = (torch.rand(32, generator=g) ** 4 * 1000).tolist()
        perm = ep.balanced_placement(loads, world)
        assert sorted(perm) == list(range(32))
        El = 32 // world
        ranks = [perm[r * El:(r + 1) * El] for r in range(world)]
        assert all(r == sorted(r) for r in ranks)
        busiest = max(sum(loads[e] for e in r) for r in ranks)
        contiguous = max(sum(loads[r * El:(r + 1) * El]) for r in range(world))
        assert busiest <= contiguous + 1e-9
        # LPT bound: the busiest rank exceeds the mean by at most the largest single load
        assert busiest <= sum(loads) / world + max(loads) + 1e-9
    assert ep.balanced_placement([5, 1, 1, 5, 3, 3, 2, 2], 2) == [0, 1, 4, 6, 2, 3, 5, 7]


def test_placement_relabelling_keeps_the_moe_output():
    """Relabelling the experts (router rows and expert weights permuted together) leaves the batched MoE unchanged:
    the float64 oracle on a relabelled tiny model equals the original's."""
    import numpy as np
    from gptoss_b200 import ep, synth
    from oracle import moe as omoe
    t = synth.moe_layer(seed=5, H=64, I=32, E=8)
    p = "model.layers.0."
    x = synth.tokens(12, seed=6, H=64).numpy()
    perm = ep.balanced_placement([7, 1, 3, 3, 9, 2, 2, 5], 2)
    W, b = ep.apply_placement(perm, t[p + "mlp.router.weight"], t[p + "mlp.router.bias"])
    t2 = dict(t)
    t2[p + "mlp.router.weight"], t2[p + "mlp.router.bias"] = W, b
    for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
              "down_proj_scales", "down_proj_bias"):
        t2[p + "mlp.experts." + n] = t[p + "mlp.experts." + n][perm]
    tn, tn2 = synth.to_numpy(t), synth.to_numpy(t2)
    h = omoe.rms_norm(x, tn[p + "post_attention_layernorm.weight"])
    a = omoe.moe(tn, p, h)
    b2 = omoe.moe(tn2, p, h)
    np.testing.assert_allclose(b2, a, rtol=1e-6, atol=1e-7)
