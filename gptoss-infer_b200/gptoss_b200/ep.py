"""Expert parallelism for the batched MoE path: experts sharded contiguously over the G ranks of a process group
(E / G per rank), tokens data-parallel (each rank routes its own shard).

One layer call on every rank (all ranks take the same collective steps in the same order):
  1. route the rank's tokens (RMSNorm, router, top k, softmax) with the library's batched router;
  2. dispatch: each (token, slot) pair goes to the rank owning its expert. The per-destination counts are exchanged
     with one all-to-all, then the normalized token rows (fp32) and their (local expert id, gate weight) with one
     all-to-all each, packed in destination order (token, then slot, ascending within a destination);
  3. the received rows run through the rank's local experts (the library's batched tensor-core MoE with k = 1, so
     each row comes back as w * (W2 swiglu(W1 h + b1) + b2));
  4. combine: the results return with the reverse all-to-all and are added to the residual stream in slot order.

Because every row's expert computation and the slot-ordered combine are the same operations as in the single-GPU
batched path, the result is bit-identical to it for any G. Collectives are torch.distributed all_to_all_single (NCCL
over NVLink between GPUs, gloo for the CPU tests). The routing and local expert steps are injectable so the
dispatch/combine logic runs on CPU with a reference compute.
"""
import torch
import torch.distributed as dist

from . import capi


def _a2a(out, inp, out_splits, in_splits, group, world):
    if world == 1:
        out.copy_(inp)
    else:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


class ExpertParallelMoE:
    """x <- x + MoE(RMSNorm(x)) for a rank's token shard, experts [rank * El, (rank + 1) * El) held locally.

    route(x) -> (h [T, H] fp32, ids [T, k] int32 (global expert ids), w [T, k] fp32)
    compute(h_rows [n, H], local_ids [n] int32, w [n] fp32) -> y [n, H] fp32 (w already applied)
    """

    def __init__(self, route, compute, rank, world, E, k, H, group=None):
        if E % world:
            raise ValueError(f"{E} experts do not split evenly over {world} ranks")
        self.route, self.compute = route, compute
        self.rank, self.world, self.E, self.k, self.H = rank, world, E, k, H
        self.El = E // world
        self.group = group

    def forward(self, x):
        T, H = x.shape
        k, G = self.k, self.world
        h, ids, w = self.route(x)
        dest = ids.long() // self.El                                   # [T, k]
        flat = dest.reshape(-1)
        order = torch.argsort(flat, stable=True)                       # (token, slot) grouped by destination
        send = torch.bincount(flat, minlength=G)
        recv = torch.empty_like(send)
        _a2a(recv, send, None, None, self.group, G)
        sc, rc = send.tolist(), recv.tolist()
        n_send, n_recv = sum(sc), sum(rc)
        h_send = h[order // k].contiguous()
        meta_send = torch.stack([(ids.reshape(-1)[order].long() - flat[order] * self.El).to(w.dtype),
                                 w.reshape(-1)[order]], 1).contiguous()   # local ids are exact in w's type
        h_recv = torch.empty(n_recv, H, dtype=h.dtype, device=h.device)
        meta_recv = torch.empty(n_recv, 2, dtype=w.dtype, device=h.device)
        _a2a(h_recv, h_send, rc, sc, self.group, G)
        _a2a(meta_recv, meta_send, rc, sc, self.group, G)
        if n_recv:
            y_recv = self.compute(h_recv, meta_recv[:, 0].to(torch.int32).contiguous(), meta_recv[:, 1].contiguous())
        else:
            y_recv = torch.empty(0, H, dtype=h.dtype, device=h.device)
        y_back = torch.empty(n_send, H, dtype=h.dtype, device=h.device)
        _a2a(y_back, y_recv.contiguous(), sc, rc, self.group, G)
        y_ts = torch.empty(T * k, H, dtype=h.dtype, device=h.device)
        y_ts[order] = y_back
        y_ts = y_ts.view(T, k, H)
        for s in range(k):                                             # slot order, as the single-GPU combine
            x += y_ts[:, s]
        return x


def gpu_route(lib, norm_w, router_w, router_b, E, k, eps=1e-5):
    """The library's batched router (RMSNorm, fp64 logits, top k, softmax) on the current stream."""
    P = capi.ptr

    def route(x):
        T, H = x.shape
        h = torch.empty_like(x)
        ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, k, dtype=torch.float32, device=x.device)
        rc = lib.gptoss_moe_route_batched(P(router_w), P(router_b), P(x), P(norm_w), eps, E, H, k, T, P(h), P(ids),
                                          P(w), torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
        return h, ids, w

    return route


def gpu_compute(lib, layer):
    """The local experts of a prepared layer (gptoss_moe_layer_create with this rank's experts) on given rows."""
    P = capi.ptr

    def compute(h_rows, lids, w):
        n, H = h_rows.shape
        y = torch.zeros_like(h_rows)
        rc = lib.gptoss_moe_layer_experts_batched(layer, P(h_rows), P(lids), P(w), P(y), n, 1,
                                                  torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
        return y

    return compute


class EpGroup:
    """The shared state of the library's peer-memory expert parallelism for one process group: every rank's region
    (allocated zeroed here, exported with a CUDA IPC handle, the handles exchanged with all_gather_object and the
    peers' regions mapped into this process) and the layer-call epoch, which all ranks advance together. One group
    serves every layer of a model; its calls must be issued in the same order on every rank."""

    def __init__(self, lib, E, k, H, I, rank, world, T_max, group=None):
        import ctypes
        self.lib, self.E, self.k, self.H, self.I = lib, E, k, H, I
        self.rank, self.world, self.T_max = rank, world, T_max
        nbytes = ctypes.c_longlong()
        _ok(lib, lib.gptoss_ep_region_bytes(E, k, H, I, world, T_max, ctypes.byref(nbytes)))
        region = ctypes.c_void_p()
        _ok(lib, lib.gptoss_ep_region_alloc(nbytes, ctypes.byref(region)))
        self.region = region.value
        handle = ctypes.create_string_buffer(64)
        _ok(lib, lib.gptoss_ipc_handle(self.region, handle))
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, handle.raw, group=group)
        else:
            handles = [handle.raw]
        self._opened = []
        peers = []
        for r, hb in enumerate(handles):
            if r == rank:
                peers.append(self.region)
                continue
            p = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(hb, 64)
            _ok(lib, lib.gptoss_ipc_open(buf, ctypes.byref(p)))
            peers.append(p.value)
            self._opened.append(p.value)
        self.peers = (ctypes.c_void_p * world)(*peers)
        self.epoch = 0
        self.group = group

    def status(self):
        import ctypes
        code = ctypes.c_int()
        _ok(self.lib, self.lib.gptoss_ep_status(self.E, self.k, self.H, self.I, self.world, self.T_max,
                                                ctypes.byref(code)))
        return code.value

    def close(self):
        """Every rank calls this after its last layer call; the barrier keeps a region alive until no peer can
        still write into it."""
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            self.lib.gptoss_ipc_close(p)
        self._opened = []
        if self.region:
            self.lib.gptoss_ep_region_free(self.region)
            self.region = None


class PeerExpertParallelMoE:
    """x <- x + MoE(RMSNorm(x)) for this rank's token shard, experts [rank E/world, (rank + 1) E/world) in `layer`
    (gptoss_moe_layer_create with those experts and the full k), dispatch and combine inside the library's kernels
    over NVLink peer memory (gptoss_ep_layer_forward); bit-identical to the single-GPU batched forward."""

    def __init__(self, ep_group, layer, router_w, router_b, norm_w, eps=1e-5):
        g = ep_group
        self.g, self.layer, self.eps = g, layer, eps
        self.router_b, self.norm_w = router_b, norm_w
        self.w64 = torch.empty(g.H * 32, dtype=torch.float64, device=router_w.device)
        _ok(g.lib, g.lib.gptoss_router_w64(capi.ptr(router_w), g.E, g.H, capi.ptr(self.w64),
                                           torch.cuda.current_stream().cuda_stream))

    def forward(self, x):
        g = self.g
        T = x.shape[0]
        if T > g.T_max:
            raise ValueError(f"{T} tokens > T_max {g.T_max}")
        g.epoch += 1
        P = capi.ptr
        _ok(g.lib, g.lib.gptoss_ep_layer_forward(self.layer, P(self.w64), P(self.router_b), P(self.norm_w), self.eps,
                                                 g.E, g.rank, g.world, P(x), P(x), T, g.T_max, g.peers, g.epoch,
                                                 torch.cuda.current_stream().cuda_stream))
        return x


def balanced_placement(loads, world):
    """Expert placement by expected load: which expert each rank holds, E / world experts per rank.

    loads[e] is expert e's expected row count (from routing statistics, e.g. a calibration batch). Greedy
    longest-processing-time: experts in decreasing load, each to the rank with the fewest rows that still has room
    (ties to the lower rank, equal loads to the lower expert id). Returns perm, a list of E expert ids: rank r holds
    experts perm[r * El : (r + 1) * El], each rank's in ascending id order. Relabelling the model by perm (router rows
    and expert weights; apply_placement) makes the contiguous ownership of the kernels balanced; the MoE output is
    unchanged (the combine adds each token's slots in logit order, which a relabelling does not change; only exact
    logit ties, which go to the lower id, could pick differently)."""
    E = len(loads)
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    El = E // world
    order = sorted(range(E), key=lambda e: (-float(loads[e]), e))
    held = [[] for _ in range(world)]
    rows = [0.0] * world
    for e in order:
        r = min((r for r in range(world) if len(held[r]) < El), key=lambda r: (rows[r], r))
        held[r].append(e)
        rows[r] += float(loads[e])
    return [e for r in range(world) for e in sorted(held[r])]


def apply_placement(perm, router_w, router_b):
    """The router of the relabelled model: expert j of the new labelling is expert perm[j] of the old one."""
    idx = torch.as_tensor(perm, dtype=torch.long, device=router_w.device)
    return router_w[idx].contiguous(), router_b[idx].contiguous()


def _ok(lib, rc):
    if rc != 0:
        raise RuntimeError(lib.gptoss_last_error().decode())
