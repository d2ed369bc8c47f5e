"""Expert-parallel batched MoE (gptoss_b200/ep.py) on the GPU: routing by the library's batched router, dispatch and
combine by all-to-all, the local experts by the batched tensor-core path with k = 1.

Every row's expert computation and the slot-ordered combine are the operations of the single-GPU batched forward
(gptoss_moe_layer_forward_batched, the batched form of gptoss_ref/model.py:100-104), so the expert-parallel result
must be bit-identical to it: on one GPU (no collective), and over two GPUs with NCCL (skipped with fewer GPUs),
including a step where one rank receives no rows. The expert-parallel kernels use the stacked tile plan (a token's
activation terms as successive MMAs on one accumulator row); the packed plan adds the same terms in another order
(equal within the float64 bound, not bit for bit), so every test here runs the batched path in the stacked plan.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from gptoss_b200 import capi, ep, synth

pytestmark = pytest.mark.gpu
PX = "model.layers.0."


@pytest.fixture(autouse=True)
def stacked_plan():
    lib = capi.load()
    prev = lib.gptoss_set_prefill_packing(0)
    yield
    lib.gptoss_set_prefill_packing(prev)
EX = PX + "mlp.experts."
E8 = 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(skew_to_first_half):
    t = synth.moe_layer(seed=3, E=E8)
    if skew_to_first_half:                    # every token picks experts 0..3 only
        b = t[PX + "mlp.router.bias"].float()
        b[E8 // 2:] -= 100.0
        t[PX + "mlp.router.bias"] = b.to(torch.bfloat16)
    return t


def _router(t, dev):
    return (t[PX + "post_attention_layernorm.weight"].float().to(dev), t[PX + "mlp.router.weight"].to(dev),
            t[PX + "mlp.router.bias"].float().to(dev))


def _experts(t, dev, e0, e1):
    names = ["gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
             "down_proj_scales", "down_proj_bias"]
    out = []
    for n in names:
        v = t[EX + n][e0:e1]
        out.append((v.float() if v.dtype == torch.bfloat16 else v).contiguous().to(dev))
    return out


def _layer(lib, ln, W, b, ex, E, k):
    P = capi.ptr
    L = lib.gptoss_moe_layer_create(P(ln), 1e-5, P(W), P(b), *(P(e) for e in ex), E, k, 2880, 2880, 1.702, 7.0)
    assert L, lib.gptoss_last_error().decode()
    return L


def _single_gpu_reference(t, x, dev):
    """The single-GPU batched forward over all tokens (all experts on one device)."""
    lib = capi.load()
    ln, W, b = _router(t, dev)
    ex = _experts(t, dev, 0, E8)
    L = _layer(lib, ln, W, b, ex, E8, 4)
    try:
        xd = x.to(dev).contiguous()
        y = xd.clone()
        assert lib.gptoss_moe_layer_forward_batched(L, capi.ptr(xd), capi.ptr(y), x.shape[0], None, None) == 0, \
            lib.gptoss_last_error().decode()
        torch.cuda.synchronize()
        return y.cpu()
    finally:
        lib.gptoss_moe_layer_destroy(L)


def _ep_forward(lib, t, x_shard, rank, world, dev, group=None):
    El = E8 // world
    ln, W, b = _router(t, dev)
    ex = _experts(t, dev, rank * El, (rank + 1) * El)
    L = _layer(lib, ln, W, b, ex, El, min(4, El))
    try:
        m = ep.ExpertParallelMoE(ep.gpu_route(lib, ln, W, b, E8, 4), ep.gpu_compute(lib, L), rank, world, E8, 4,
                                 2880, group)
        y = m.forward(x_shard.to(dev).contiguous())
        torch.cuda.synchronize()
        return y.cpu()
    finally:
        lib.gptoss_moe_layer_destroy(L)


@pytest.mark.parametrize("skew", [False, True])
def test_ep_one_gpu_bit_identical_to_batched_forward(skew):
    lib = capi.load()
    t = _model(skew)
    x = synth.tokens(40, seed=11)
    want = _single_gpu_reference(t, x, "cuda")
    got = _ep_forward(lib, t, x, 0, 1, "cuda")
    assert torch.equal(got, want)


def _worker(rank, world, port, skew, x, q):
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        lib = capi.load()
        lib.gptoss_set_prefill_packing(0)              # a fresh process: the stacked plan, as the parent's reference
        t = _model(skew)
        y = _ep_forward(lib, t, x[rank::world], rank, world, dev)
        q.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("skew", [False, True])
def test_ep_two_gpus_bit_identical_to_batched_forward(skew):
    import torch.multiprocessing as mp
    world = 2
    x = synth.tokens(40, seed=12)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    os.environ.update(env)
    procs = [ctx.Process(target=_worker, args=(r, world, port, skew, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = torch.empty(40, 2880)
    for r in range(world):
        out[r::world] = torch.from_numpy(got[r])
    want = _single_gpu_reference(_model(skew), x, "cuda:0")
    assert torch.equal(out, want)


# ---------------------------------------------------------------- dispatch and combine over peer memory (one kernel
# sequence per layer, gptoss_ep_layer_forward)
def _peer_forward(lib, t, x_shard, rank, world, dev, T_max, calls=2):
    El = E8 // world
    ln, W, b = _router(t, dev)
    ex = _experts(t, dev, rank * El, (rank + 1) * El)
    L = _layer(lib, ln, W, b, ex, El, 4)
    g = ep.EpGroup(lib, E8, 4, 2880, 2880, rank, world, T_max)
    try:
        m = ep.PeerExpertParallelMoE(g, L, W, b, ln)
        outs = []
        for _ in range(calls):                       # several layer calls: epochs advance, regions are reused
            y = m.forward(x_shard.to(dev).contiguous().clone())
            torch.cuda.synchronize()
            outs.append(y.cpu())
        assert g.status() == 0
        return outs
    finally:
        g.close()
        lib.gptoss_moe_layer_destroy(L)


@pytest.mark.parametrize("skew", [False, True])
def test_peer_ep_one_gpu_bit_identical_to_batched_forward(skew):
    lib = capi.load()
    t = _model(skew)
    x = synth.tokens(40, seed=13)
    want = _single_gpu_reference(t, x, "cuda")
    for got in _peer_forward(lib, t, x, 0, 1, "cuda", T_max=64):
        assert torch.equal(got, want)


def _peer_worker(rank, world, port, skew, x, split, q):
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        lib = capi.load()
        lib.gptoss_set_prefill_packing(0)
        t = _model(skew)
        lo, hi = split[rank], split[rank + 1]
        outs = _peer_forward(lib, t, x[lo:hi], rank, world, dev, T_max=40)
        q.put((rank, [o.numpy() for o in outs]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("skew,split", [(False, (0, 20, 40)), (True, (0, 13, 40)), (False, (0, 40, 40))])
def test_peer_ep_two_gpus_bit_identical_to_batched_forward(skew, split):
    """Two GPUs; uneven token splits, one rank with no tokens, and (skew) one rank that receives no rows."""
    import torch.multiprocessing as mp
    world = 2
    x = synth.tokens(40, seed=14)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, skew, x, split, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = _single_gpu_reference(_model(skew), x, "cuda:0")
    for c in range(2):
        out = torch.cat([torch.from_numpy(got[r][c]) for r in range(world)])
        assert torch.equal(out, want)


def test_peer_ep_bounded_wait_runs_out_and_next_call_is_clean():
    """A cross-rank wait that nothing ends, on one GPU and without any fault: rank 0 of a world of 2 whose second
    region is a second local allocation that no rank ever signals. Every expert-parallel barrier gives up after its
    bound (about a second), gptoss_ep_status reports 60-62, all memory touched is valid, and the next normal call
    (world 1, fresh regions) is bit-identical to the single-GPU batched forward."""
    import ctypes
    import time
    lib = capi.load()
    P = capi.ptr
    t = _model(False)
    x = synth.tokens(40, seed=15)
    world, T_max, El = 2, 40, E8 // 2
    ln, W, b = _router(t, "cuda")
    L = _layer(lib, ln, W, b, _experts(t, "cuda", 0, El), El, 4)
    nbytes = ctypes.c_longlong()
    regions = []
    try:
        assert lib.gptoss_ep_region_bytes(E8, 4, 2880, 2880, world, T_max, ctypes.byref(nbytes)) == 0
        for _ in range(world):
            r = ctypes.c_void_p()
            assert lib.gptoss_ep_region_alloc(nbytes, ctypes.byref(r)) == 0, lib.gptoss_last_error().decode()
            regions.append(r.value)
        peers = (ctypes.c_void_p * world)(*regions)
        w64 = torch.empty(2880 * 32, dtype=torch.float64, device="cuda")
        assert lib.gptoss_router_w64(P(W), E8, 2880, P(w64), None) == 0
        xd = x.to("cuda").contiguous()
        y = xd.clone()
        t0 = time.time()
        rc = lib.gptoss_ep_layer_forward(L, P(w64), P(b), P(ln), 1e-5, E8, 0, world, P(xd), P(y), 40, T_max, peers,
                                         1, None)
        assert rc == 0, lib.gptoss_last_error().decode()
        code = ctypes.c_int()
        assert lib.gptoss_ep_status(E8, 4, 2880, 2880, world, T_max, ctypes.byref(code)) == 0
        waited = time.time() - t0
        assert 60 <= code.value <= 62, code.value
        assert waited < 60.0, waited
    finally:
        torch.cuda.synchronize()
        for r in regions:
            lib.gptoss_ep_region_free(r)
        lib.gptoss_moe_layer_destroy(L)
    want = _single_gpu_reference(t, x, "cuda")
    for got in _peer_forward(lib, t, x, 0, 1, "cuda", T_max=64):
        assert torch.equal(got, want)


def test_placement_relabelling_bit_identical_on_gpu():
    """Expert placement by load relabels the experts (router rows and expert weights permuted together). The batched
    forward adds each token's slots in logit order, which the relabelling keeps, so the result is bit-identical."""
    t = _model(False)
    perm = ep.balanced_placement([9, 1, 4, 4, 7, 2, 2, 5], 2)
    W, b = ep.apply_placement(perm, t[PX + "mlp.router.weight"], t[PX + "mlp.router.bias"])
    t2 = dict(t)
    t2[PX + "mlp.router.weight"], t2[PX + "mlp.router.bias"] = W, b
    for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
              "down_proj_scales", "down_proj_bias"):
        t2[EX + n] = t[EX + n][perm].contiguous()
    x = synth.tokens(40, seed=16)
    assert torch.equal(_single_gpu_reference(t2, x, "cuda"), _single_gpu_reference(t, x, "cuda"))
