"""Benchmark of the gpt-oss-20b MXFP4 MoE path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload moe-decode|prefill|ep] [--impl ours|reference]

Default workload "moe-decode" (BASELINE configs[0] stacked as in configs[1]): bs=1 decode through the 24 MoE layers
of a 20b-shaped random-init model: per step, one token x goes x <- x + MoE(RMSNorm(x)) through 24 distinct layers
(router 2880->32, top-4, MXFP4 gate/up + clamped SwiGLU, MXFP4 down, weighted combine). 24 x 423 MB of expert
weights are resident, far above the 126 MB L2, and each step reads 24 x 53,130,240 algorithmic bytes.
Timed region: W untimed steps, then exactly K steps between a barrier + synchronize on both sides, CUDA events on
the launching stream, max over ranks. With N > 1 every rank runs an independent replica (bs=1 decode does not
shard): value = N * K * bytes / max time ("replicas only", scaling "weak").

The same line carries, measured in the same run:
  "ep"       configs[3] at the run's N: 8192 tokens (over all ranks) x 24 MoE layers per step, experts sharded over
             the N ranks (placed by expected load), dispatch and combine inside the kernels over NVLink peer memory;
             max over ranks (strong scaling). At N = 1 it is the one-GPU baseline of the same workload.
  "prefill"  (N = 1) configs[2]: 2048 tokens x 1 MoE layer per step through the batched tensor-core path.
  "ref_gpu"  (N = 1) the reference's own CUDA kernels (openvang/gptoss-infer runtime, built for sm_100a from its
             sources into oracle/_ref/) against this library's, same ABI entry points, same inputs, same box.

Workloads "prefill" and "ep" alone print their own line (metric of that workload).

--impl reference times the reference's own CPU implementation of this path: Reference.moe of gptoss_ref
(openvang/gptoss-infer reference/gptoss_ref/model.py:92-105, fp32 torch, dequantizing each selected expert per call),
staged into baseline/_ref/ by oracle/stage_reference.py, with torch using every host core; one token through one
MoE layer per step, same metric, unit and config as this arm. Where the package is not staged it falls back to the
numpy restatement in oracle/moe.py and says so ("kind": "port").
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "gptoss-infer_b200")]

H, I, E, K_TOP, LAYERS = 2880, 2880, 32, 4, 24
EXPERT_BYTES = 8_294_400 + 518_400 + 4_147_200 + 259_200            # blocks + scales, gate/up and down
LAYER_BYTES = K_TOP * EXPERT_BYTES + 184_320 + K_TOP * (5760 + 2880) * 2   # + router + bf16 biases = 53,130,240
GATEUP_BYTES = K_TOP * (8_294_400 + 518_400 + 5760 * 4) + H * 4 + K_TOP * I * 4   # per launch, fp32 bias/in/out
METRIC = "bs=1 decode MoE-layer HBM GB/s (20b-shaped, 24 layers)"
UNIT = "GB/s"
PREFILL_METRIC = "prefill tok/s (2048 tokens x 1 MoE layer, Zipf s=1.1 routing)"
EP_METRIC = "expert-parallel prefill tok/s (8192 tokens x 24 MoE layers, Zipf s=1.2 routing)"
REF_BUDGET_S = 60.0                  # timed seconds at most for a CPU reference arm
REF_STAGED = ROOT / "baseline" / "_ref" / "reference"
REF_LIB = ROOT / "oracle" / "_ref" / "libgptoss_ref.so"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="moe-decode", choices=["moe-decode", "prefill", "ep", "decode"])
    ap.add_argument("--tokens", type=int, default=None,
                    help="prefill: tokens per step (config 2: 2048); ep: tokens per step over all ranks (config 3: 8192)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ep-impl", default="peer", choices=["peer", "nccl"],
                    help="ep: dispatch/combine inside the kernels over peer memory, or NCCL all-to-all around them")
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "contiguous"],
                    help="ep: experts placed on ranks by expected load (calibration batch) or in id order")
    ap.add_argument("--moe-impl", type=int, default=None, help="0 = SIMT, 1 = tensor cores (default: library's)")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="moe-decode: skip the ep / prefill / ref_gpu objects")
    ap.add_argument("--decode-tokens", type=int, default=128, help="decode: greedy tokens per timed run (configs[1]: 128)")
    ap.add_argument("--decode-reps", type=int, default=7, help="decode: timed runs (median reported)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()                          # the first sample is taken before the timed region starts
            while not self.rows and time.time() - t0 < 5.0:
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            n, t0 = len(self.rows), time.time()       # and one more right after it ends (short regions)
            while len(self.rows) == n and time.time() - t0 < 1.0:
                time.sleep(0.02)
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.t.join(timeout=5)

    def summary(self):
        import statistics
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) >= 9:
                for n, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------------- setup
class Ctx:
    """One process per GPU: world size, rank, local rank, device, and the max-over-ranks helpers."""

    def __init__(self):
        import torch
        self.ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.ws > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
        else:
            torch.cuda.set_device(0)
        self.dev = torch.device("cuda", torch.cuda.current_device())

    def barrier(self):
        import torch
        if self.ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max(self, v):
        import torch
        if self.ws == 1:
            return v
        t = torch.tensor([float(v)], device=self.dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum_list(self, v):
        import torch
        t = torch.tensor(v, dtype=torch.float64, device=self.dev)
        if self.ws > 1:
            torch.distributed.all_reduce(t)
        return t.tolist()

    def close(self):
        if self.ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def peaks():
    pk = ROOT / "MEASURED_PEAKS.json"
    return json.loads(pk.read_text()) if pk.exists() else {}


def fp4_peak(lib, sustained):
    """Dense FP4 (kind::mxf4) tensor peak of this GPU in TFLOP/s: measured live by the library's back-to-back MMA
    microbenchmark when it has one, else 4 x the measured bf16 cuBLAS peak (dense FP4 runs at 4x the bf16 rate)."""
    import ctypes
    if hasattr(lib, "gptoss_selftest_mxf4_peak"):
        tf = ctypes.c_double()
        if lib.gptoss_selftest_mxf4_peak(ctypes.byref(tf)) == 0 and tf.value > 0:
            return tf.value, "measured: back-to-back tcgen05.mma kind::mxf4 M=128 N=256 K=64 on every SM"
    bf16 = peaks().get("bf16_tflops_sustained" if sustained else "bf16_tflops")
    return (4.0 * bf16, "4 x measured bf16 cuBLAS (of measured)") if bf16 else (4.0 * 1590.0, "4 x fallback bf16")


def ctypes_array(events):
    import ctypes
    return (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])


# ------------------------------------------------------------------------------------------------------- configs
def decode_config(ws, layers):
    return {"workload": "moe-decode (configs[0] stacked x24, bs=1)", "layers": layers, "experts": E, "top_k": K_TOP,
            "hidden": H, "intermediate": I, "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
            "l2": "inputs larger than L2: 24 distinct layers, 10.2 GB of experts"}


def prefill_config(T, ws, counts=None):
    c = {"workload": "prefill (configs[2])", "tokens": T, "experts": E, "top_k": K_TOP, "hidden": H,
         "intermediate": I, "zipf_s": 1.1, "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
         "l2": "423 MB of experts per layer, larger than L2"}
    if counts is not None:
        c["expert_token_counts"] = counts
    return c


def ep_config(T, ws, layers):
    return {"workload": "expert-parallel prefill (configs[3])", "tokens": T, "tokens_per_rank": T // ws,
            "layers": layers, "experts": E, "experts_per_rank": E // ws, "top_k": K_TOP, "zipf_s": 1.2,
            "parallelism": f"ep{ws} (experts) x dp{ws} (tokens)", "l2": "423 MB of experts per layer, larger than L2"}


# ------------------------------------------------------------------------------------------------------- CPU reference
class ReferenceMoE:
    """The reference's CPU MoE: gptoss_ref's Reference.moe (fp32 torch, every selected expert dequantized per call)
    when baseline/_ref holds the staged package, else oracle/moe.py's numpy restatement of it ("port")."""

    def __init__(self, t, prefix="model.layers.0."):
        import torch
        self.cores = os.cpu_count()
        self.prefix = prefix
        if (REF_STAGED / "gptoss_ref" / "model.py").exists():
            if str(REF_STAGED) not in sys.path:
                sys.path.insert(0, str(REF_STAGED))
            from gptoss_ref.config import GptOssConfig
            from gptoss_ref.model import Reference, rms_norm
            from gptoss_ref.weights import DictWeights
            cfg = GptOssConfig.from_dict({
                "vocab_size": 201088, "hidden_size": H, "intermediate_size": I, "num_hidden_layers": 1,
                "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 64, "num_local_experts": E,
                "num_experts_per_tok": K_TOP, "sliding_window": 128, "rope_theta": 150000, "swiglu_limit": 7.0,
                "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                 "truncate": False, "original_max_position_embeddings": 4096}})
            self.ref = Reference(cfg, DictWeights({k.replace(prefix, "model.layers.0."): v for k, v in t.items()}),
                                 threads=self.cores)
            self.ln = t[prefix + "post_attention_layernorm.weight"].float()
            self.norm = lambda x: rms_norm(x, self.ln, 1e-5)
            self.kind = "reference"
            self.what = (f"gptoss_ref Reference.moe (torch {torch.__version__} fp32, {torch.get_num_threads()} "
                         f"threads, per-call MXFP4 dequant of every selected expert)")
        else:
            from gptoss_b200 import synth
            from oracle import moe as omoe
            self.omoe, self.tn = omoe, synth.to_numpy(t)
            self.kind = "port"
            self.what = "oracle/moe.py numpy restatement of Reference.moe (fp32, per-call MXFP4 dequant)"

    def normed(self, x):
        """RMSNorm (the reference's) of fp32 tokens x [T, H] (torch CPU tensor)."""
        if self.kind == "reference":
            return self.norm(x)
        import torch
        return torch.from_numpy(self.omoe.rms_norm(x.numpy(), self.tn[self.prefix + "post_attention_layernorm.weight"]))

    def moe(self, h):
        import torch
        if self.kind == "reference":
            with torch.inference_mode():
                return self.ref.moe(0, h)
        return self.omoe.moe(self.tn, self.prefix, h.numpy())


def time_reference(rm, h, n_per_step, steps, warmup, budget_s):
    """Runs rm.moe on slices of n_per_step tokens of h: min(warmup, 1) untimed, then up to `steps` timed within
    budget_s seconds. Returns (seconds, tokens, steps timed)."""
    n = h.shape[0]
    for i in range(min(warmup, 1)):
        rm.moe(h[:n_per_step])
    t0 = time.perf_counter()
    done = timed = 0
    for i in range(steps):
        j = (i * n_per_step) % max(1, n - n_per_step + 1)
        rm.moe(h[j:j + n_per_step])
        done += n_per_step
        timed += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return time.perf_counter() - t0, done, timed


# ------------------------------------------------------------------------------------------------------- decode
def make_layers(n_layers, dev):
    """Layer 0 from synth seed 0 (the config-0 layer); the others drawn on the device with the same distributions."""
    import torch
    from gptoss_b200 import synth
    layers = []
    t0 = synth.moe_layer(seed=0)
    p = "model.layers.0."
    g = torch.Generator(device=dev).manual_seed(1234)
    for l in range(n_layers):
        if l == 0:
            d = {k[len(p):]: v.to(dev) for k, v in t0.items()}
        else:
            d = {}
            d["post_attention_layernorm.weight"] = (1 + torch.randn(H, device=dev, generator=g) * 0.02).bfloat16()
            d["mlp.router.weight"] = (torch.randn(E, H, device=dev, generator=g) * 0.02).bfloat16()
            d["mlp.router.bias"] = (torch.randn(E, device=dev, generator=g) * 0.01).bfloat16()
            for name, rows, k in (("gate_up_proj", 2 * I, H), ("down_proj", H, I)):
                q = "mlp.experts." + name
                d[q + "_blocks"] = torch.randint(0, 256, (E, rows, k // 32, 16), device=dev, generator=g,
                                                 dtype=torch.uint8)
                d[q + "_scales"] = torch.randint(120, 127, (E, rows, k // 32), device=dev, generator=g,
                                                 dtype=torch.uint8)
                d[q + "_bias"] = (torch.randn(E, rows, device=dev, generator=g) * 0.01).bfloat16()
        layers.append({
            "ln": d["post_attention_layernorm.weight"].float(),
            "W": d["mlp.router.weight"].contiguous(),
            "b": d["mlp.router.bias"].float(),
            "ex": [d["mlp.experts.gate_up_proj_blocks"], d["mlp.experts.gate_up_proj_scales"],
                   d["mlp.experts.gate_up_proj_bias"].float(), d["mlp.experts.down_proj_blocks"],
                   d["mlp.experts.down_proj_scales"], d["mlp.experts.down_proj_bias"].float()],
        })
    return layers, t0


def run_decode(args, ctx, lib):
    import torch
    from gptoss_b200 import capi
    P = capi.ptr
    ws, rank, dev = ctx.ws, ctx.rank, ctx.dev
    if args.moe_impl is not None and lib.gptoss_set_moe_impl(args.moe_impl) < 0:
        raise RuntimeError(lib.gptoss_last_error().decode())
    layers, t0 = make_layers(args.layers, dev)
    impl = args.moe_impl if args.moe_impl is not None else 1
    # the prepared layer's tensor-core kernel: impl 1 the row-job kernel (default), impl 2 the stream-K kernel
    kname = "moe_fused_kernel" if impl == 2 else "moe_rows_kernel"
    handles = []
    if impl in (1, 2):
        for L in layers:
            hdl = lib.gptoss_moe_layer_create(P(L["ln"]), 1e-5, P(L["W"]), P(L["b"]), *(P(e) for e in L["ex"]), E,
                                              K_TOP, H, I, 1.702, 7.0)
            if not hdl:
                raise RuntimeError(lib.gptoss_last_error().decode())
            handles.append(hdl)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    X = torch.randn(args.steps + args.warmup, H, device=dev, generator=g)
    stream = torch.cuda.current_stream()

    def layer_call(li, x, sp, events):
        if handles:
            return lib.gptoss_moe_layer_forward(handles[li], P(x), P(x), sp, events)
        L = layers[li]
        return lib.gptoss_moe_block_async(P(x), P(L["ln"]), 1e-5, P(L["W"]), P(L["b"]), *(P(e) for e in L["ex"]),
                                          P(x), E, K_TOP, H, I, 1.702, 7.0, sp, events)

    def step(x, sp, events=None):
        for li in range(len(layers)):
            if layer_call(li, x, sp, events[li] if events else None) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())

    # One decode step (24 MoE layers) is captured once as a CUDA graph and replayed, as the reference engine does
    # with its decode step (runtime/src/engine.cu:264-279): the host issues two operations per step, not 24+
    # launches. The programmatic-dependent-launch edges between the layers' kernels are kept in the graph.
    x_static = torch.empty(H, device=dev)
    for i in range(args.warmup):                          # eager warm-up also sizes the library's workspaces
        x_static.copy_(X[args.steps + i])
        step(x_static, stream.cuda_stream)
    ctx.barrier()
    cap = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    x_static.copy_(X[0])
    with torch.cuda.graph(graph, stream=cap):
        step(x_static, cap.cuda_stream)
    for i in range(3):
        x_static.copy_(X[args.steps + (i % max(1, args.warmup))])
        graph.replay()
    ctx.barrier()

    # ---- timed region: exactly K steps
    with ClockSampler(ctx.local) as clocks:
        ctx.barrier()
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0e.record(stream)
        for i in range(args.steps):
            x_static.copy_(X[i])
            graph.replay()
        t1e.record(stream)
        ctx.barrier()
    ms = ctx.max(t0e.elapsed_time(t1e))
    value = ws * args.steps * args.layers * LAYER_BYTES / (ms / 1e3) / 1e9
    # per layer: tensor cores = one fused launch; SIMT = rmsnorm + router + gate/up + down
    gpu_launches = args.steps * args.layers * (1 if handles else 4)

    # ---- per-kernel durations: a second graph of the same step with events around every layer's kernels
    n_prof = min(args.steps, 100)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.layers)]
    for quad in ev:                                       # torch creates the CUDA event at its first record
        for e in quad:
            e.record(stream)
    torch.cuda.synchronize()
    evh = [ctypes_array(e) for e in ev]
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(pgraph, stream=cap):
        step(x_static, cap.cuda_stream, evh)
    sums = [0.0, 0.0, 0.0]
    ctx.barrier()
    for i in range(n_prof):
        x_static.copy_(X[i])
        pgraph.replay()
        torch.cuda.synchronize()
        for q in ev:
            sums[0] += q[0].elapsed_time(q[1])
            sums[1] += q[1].elapsed_time(q[2])
            sums[2] += q[2].elapsed_time(q[3])
    nl = n_prof * args.layers
    part_us = [v / nl * 1e3 for v in sums]
    if handles:
        # the timed region launches nothing but the fused kernel (one per layer) and one 11.5 KB copy per step, so
        # its average launch duration is the timed region's time over its launches (an upper bound: it includes the
        # gaps between launches); the event-bracketed figure is kept beside it
        kernel_us = {kname: ms / args.steps / args.layers * 1e3, kname + "_event_bracketed": part_us[2]}
        top_us, top_name, top_bytes = (ms / args.steps / args.layers * 1e3,
                                       kname + " (RMSNorm + router + gate/up + down)", LAYER_BYTES)
    else:
        kernel_us = {"router+rmsnorm": part_us[0], "gate_up": part_us[1], "down+combine": part_us[2]}
        top_us, top_name, top_bytes = part_us[1], "gateup_simt_kernel", GATEUP_BYTES
    del evh

    # ---- end to end through the public API: host x in, host x out, every step
    xh = torch.randn(args.steps, H, generator=torch.Generator().manual_seed(5 + rank)).pin_memory()
    yh = torch.empty(H).pin_memory()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        x_static.copy_(xh[i], non_blocking=True)
        graph.replay()
        yh.copy_(x_static, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    ctx.barrier()
    ms_e2e = ctx.max(e0.elapsed_time(e1))
    e2e = ws * args.steps * args.layers * LAYER_BYTES / (ms_e2e / 1e3) / 1e9
    del graph, pgraph
    moe_t64 = run_moe_t64(args, ctx, lib, handles, layers) if handles and not args.no_extras else None
    for hdl in handles:
        lib.gptoss_moe_layer_destroy(hdl)
    del layers
    torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        rm = ReferenceMoE(t0)
        h = rm.normed(torch.randn(64, H, generator=torch.Generator().manual_seed(99)))
        el, n, _ = time_reference(rm, h, 1, 64, 1, 15.0)
        cpu = {"value": LAYER_BYTES * n / el / 1e9, "unit": UNIT, "cores": rm.cores, "kind": rm.kind,
               "sample": f"{n} tokens x 1 MoE layer (config-0 layer) through {rm.what}"}

    pk = peaks()
    hbm = pk.get("hbm_gbs")
    peak_src = "measured copy (MEASURED_PEAKS.json)" if hbm else "fallback"
    hbm = hbm or 6650.0
    achieved = top_bytes / (top_us * 1e-6) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(kname if handles else "gateup_simt_kernel")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init 20b-shaped MoE layers)",
        "config": decode_config(ws, args.layers),
        "moe_layers_tok_per_s": ws * args.steps / (ms / 1e3),
        "us_per_moe_layer": ms / args.steps / args.layers * 1e3,
        "moe_impl": "tensor cores (tcgen05 kind::mxf4)" if handles else "SIMT",
        "kernel_us": kernel_us,
        "roofline": {"bound": "hbm", "kernel": top_name, "achieved": achieved, "peak": hbm,
                     "peak_source": peak_src, "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic,
                     "frac_of_8TBs_nominal": achieved / 8000.0, "algorithmic_bytes_per_launch": top_bytes,
                     "launch_us": top_us},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4,
                "api": ("gptoss_moe_layer_forward" if handles else "gptoss_moe_block_async") +
                       " x24 per token captured in one CUDA graph; host x copied in and out every step"},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
        "moe_t64": moe_t64,
    }


def run_moe_t64(args, ctx, lib, handles, layers, T=64):
    """configs[4]'s MoE step: 64 tokens (one per concurrent sequence) through the 24 MoE layers per step, on one GPU,
    through the batched path (gptoss_moe_layer_forward_batched: router, permute, grouped tcgen05 GEMMs, combine), one
    CUDA graph per step. Almost every expert is touched by 64 x 4 picks, so each layer streams most of its 423 MB of
    experts once: the bound is HBM. Bytes per step = the distinct experts each layer's routing touched x 13.2 MB
    (+ router and biases), counted from the library's own routing of the same tokens."""
    import torch
    from gptoss_b200 import capi
    P = capi.ptr
    dev = ctx.dev
    stream = torch.cuda.current_stream()
    x0 = torch.randn(T, H, generator=torch.Generator(device=dev).manual_seed(404), device=dev)
    x = x0.clone()
    # the experts each layer touches (routing of the tokens as they arrive at that layer)
    touched = 0
    h = torch.empty_like(x)
    ids = torch.empty(T, K_TOP, dtype=torch.int32, device=dev)
    w = torch.empty(T, K_TOP, device=dev)
    for li, hdl in enumerate(handles):
        L = layers[li]
        if lib.gptoss_moe_route_batched(P(L["W"]), P(L["b"]), P(x), P(L["ln"]), 1e-5, E, H, K_TOP, T, P(h), P(ids),
                                        P(w), stream.cuda_stream) != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
        touched += int(torch.unique(ids).numel())
        if lib.gptoss_moe_layer_forward_batched(hdl, P(x), P(x), T, stream.cuda_stream, None) != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
    step_bytes = touched * EXPERT_BYTES + len(handles) * (184_320 + 0)
    def step(sp):
        x.copy_(x0)
        for hdl in handles:
            if lib.gptoss_moe_layer_forward_batched(hdl, P(x), P(x), T, sp, None) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())

    def timed(pack):
        """ms per step with the tile plan `pack` (-1: the library's choice by batch size)."""
        prev = lib.gptoss_set_prefill_packing(pack)
        try:
            for _ in range(max(args.warmup, 3)):
                step(stream.cuda_stream)
            ctx.barrier()
            cap = torch.cuda.Stream()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):     # the plan is fixed when the launches are recorded
                step(cap.cuda_stream)
        finally:
            lib.gptoss_set_prefill_packing(prev)
        for _ in range(3):
            graph.replay()
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        ctx.barrier()
        ms_ = ctx.max(e0.elapsed_time(e1)) / args.steps
        del graph
        return ms_

    ms = timed(-1)
    ms_stacked = timed(0)
    hbm = peaks().get("hbm_gbs") or 6650.0
    achieved = step_bytes / (ms * 1e-3) / 1e9
    return {"metric": "MoE step at 64 tokens per layer (configs[4]'s MoE, 24 layers, one GPU)",
            "tokens": T, "layers": len(handles), "ms_per_step": ms, "us_per_layer": ms * 1e3 / len(handles),
            "tok_per_s": ctx.ws * T / (ms * 1e-3), "experts_touched_per_layer": touched / len(handles),
            "tile_plan": "packed (a token's 8 activation terms as 8 rows of a 128-row tile, 16 tokens a tile)",
            "stacked_plan_ms_per_step": ms_stacked,
            "roofline": {"bound": "hbm", "achieved": achieved, "unit": "GB/s", "peak": hbm, "frac": achieved / hbm,
                         "algorithmic_bytes_per_step": step_bytes},
            "api": "gptoss_moe_layer_forward_batched x24 per step in one CUDA graph",
            "note": "attention of the 64 sequences is not part of this figure (the engine serves one sequence)"}


# ------------------------------------------------------------------------------------------------------- prefill
def prefill_flops(T):
    """Algorithmic FLOPs of one batched MoE layer: 2 * (T * k) * (2I * H + H * I)."""
    return 2.0 * T * K_TOP * (2 * I * H + H * I)


def prefill_inputs(T):
    """Config 2: layer 0 (synth seed 0) with the router bias skewed towards Zipf s=1.1 over a seeded expert order,
    tokens bf16 N(0,1) [T, H] (passed as fp32; the conversion is exact)."""
    import torch
    from gptoss_b200 import synth
    t = synth.moe_layer(seed=0)
    perm = synth.zipf_router_bias(t, s=1.1, beta=1.0, seed=7)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).float()
    return t, perm, x


def run_prefill(args, ctx, lib, T, with_cpu):
    """Config 2 on one GPU (replicas with N > 1): per step x_resid = x + MoE(RMSNorm(x)) for T tokens through the
    prepared layer's batched forward (batched router, permute, grouped tcgen05 GEMMs, combine), one CUDA graph."""
    import torch
    from gptoss_b200 import capi
    P = capi.ptr
    ws, dev = ctx.ws, ctx.dev
    t, perm, x_cpu = prefill_inputs(T)
    p = "model.layers.0."
    d = {k[len(p):]: v.to(dev) for k, v in t.items()}
    ln = d["post_attention_layernorm.weight"].float()
    W, b = d["mlp.router.weight"].contiguous(), d["mlp.router.bias"].float()
    ex = [d["mlp.experts.gate_up_proj_blocks"], d["mlp.experts.gate_up_proj_scales"],
          d["mlp.experts.gate_up_proj_bias"].float(), d["mlp.experts.down_proj_blocks"],
          d["mlp.experts.down_proj_scales"], d["mlp.experts.down_proj_bias"].float()]
    L = lib.gptoss_moe_layer_create(P(ln), 1e-5, P(W), P(b), *(P(e) for e in ex), E, K_TOP, H, I, 1.702, 7.0)
    if not L:
        raise RuntimeError(lib.gptoss_last_error().decode())
    x = x_cpu.to(dev)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    # realised routing (per-expert token counts), from the library's own batched router
    ids = torch.empty(T, K_TOP, dtype=torch.int32, device=dev)
    wts = torch.empty(T, K_TOP, device=dev)
    h = torch.nn.functional.rms_norm(x, (H,), ln, 1e-5)
    if lib.gptoss_kernel_router_batched(P(W), P(b), P(h), E, H, K_TOP, T, P(ids), P(wts)) != 0:
        raise RuntimeError(lib.gptoss_last_error().decode())
    counts = torch.bincount(ids.flatten().long(), minlength=E).tolist()

    def step(sp, events=None):
        y.copy_(x)
        if lib.gptoss_moe_layer_forward_batched(L, P(x), P(y), T, sp, events) != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())

    for _ in range(max(args.warmup, 3)):                 # eager warm-up also sizes the workspace
        step(stream.cuda_stream)
    ctx.barrier()
    cap = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        step(cap.cuda_stream)
    for _ in range(3):
        graph.replay()
    ctx.barrier()
    with ClockSampler(ctx.local) as clocks:
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        ctx.barrier()
    ms = ctx.max(e0.elapsed_time(e1))
    step_s = ms / args.steps / 1e3
    value = ws * T / step_s
    # end to end: host x in (pinned), host result out, every step
    xh = x_cpu.pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    ctx.barrier()
    e0.record(stream)
    for _ in range(args.steps):
        x.copy_(xh, non_blocking=True)
        graph.replay()
        yh.copy_(y, non_blocking=True)
    e1.record(stream)
    ctx.barrier()
    ms_e2e = ctx.max(e0.elapsed_time(e1))
    e2e = ws * T / (ms_e2e / args.steps / 1e3)
    # grouped GEMM durations: a second graph of the same step with events around the gate/up and down GEMM launches
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in ev:                                          # torch creates the CUDA event at its first record
        e.record(stream)
    torch.cuda.synchronize()
    evh = ctypes_array(ev)
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(pgraph, stream=cap):
        step(cap.cuda_stream, evh)
    gemm_ms = [0.0, 0.0]
    n_prof = min(args.steps, 50)
    ctx.barrier()
    for _ in range(n_prof):
        pgraph.replay()
        torch.cuda.synchronize()
        gemm_ms[0] += ev[0].elapsed_time(ev[1])
        gemm_ms[1] += ev[2].elapsed_time(ev[3])
    gemm_us = [v / n_prof * 1e3 for v in gemm_ms]
    del graph, pgraph
    variants = prefill_term_variants(args, ctx, lib, L, x, y, step, cap, ev, evh, T)
    del evh
    lib.gptoss_moe_layer_destroy(L)
    cpu = None
    if with_cpu:
        rm = ReferenceMoE(t)
        hn = rm.normed(x_cpu[:256])
        el, n, _ = time_reference(rm, hn, 64, 4, 1, 20.0)
        cpu = {"value": n / el, "unit": "tok/s", "cores": rm.cores, "kind": rm.kind,
               "sample": f"{n} tokens (64 per call) through {rm.what}"}
    peak, peak_src = fp4_peak(lib, sustained=False)
    gemm_s = sum(gemm_us) / 1e6
    achieved = prefill_flops(T) / gemm_s / 1e12                  # algorithmic FLOPs of both grouped GEMMs
    traffic = None
    tj = ROOT / "profiles" / "traffic.json"
    if tj.exists():
        traffic = json.loads(tj.read_text()).get("grouped_gemm_kernel_prefill")
    return {
        "metric": PREFILL_METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1 x e2m1 (fp32 accumulate; activations as 8 residual terms)",
        "data": "synthetic (seeded random-init 20b-shaped MoE layer, bf16 N(0,1) tokens)",
        "config": prefill_config(T, ws, counts),
        "roofline": {"bound": "tensor", "kernel": "grouped_gemm_kernel (gate/up + down launches of a step)",
                     "achieved": achieved, "unit": "TFLOP/s", "peak": peak, "peak_source": peak_src,
                     "frac": achieved / peak, "frac_of_9PF_nominal": achieved / 9000.0,
                     "algorithmic_flops_per_step": prefill_flops(T), "gemm_us": gemm_us,
                     "tensor_core_tflops_with_terms": 8 * achieved,
                     "tensor_core_frac_with_terms": 8 * achieved / peak,
                     "note": "each activation enters the MMA as 8 e2m1 terms, so the tensor cores execute 8x the "
                             "algorithmic FLOPs (plus M-tile padding)",
                     "traffic": traffic},
        "term_variants": variants,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                "api": "gptoss_moe_layer_forward_batched in a CUDA graph; host tokens copied in and out"},
        "gpu_launches": args.steps * 7,   # router, permute, 2 x (quantize, grouped GEMM), combine
        "clocks": clocks.summary(),
    }


def prefill_term_variants(args, ctx, lib, L, x, y, step, cap, ev, evh, T, reps=20):
    """The same step with 1 .. 8 activation terms (gptoss_set_prefill_terms; stacked plan) and with the packed plan
    at 8 terms: grouped-GEMM time, algorithmic TFLOP/s and its fraction of the measured FP4 peak, and the error of the
    MoE output against the 8-term stacked output (itself within 2e-5 of float64 in the parity tests)."""
    import torch
    peak, _ = fp4_peak(lib, sustained=False)

    def run(nt, pack):
        pt, pp = lib.gptoss_set_prefill_terms(nt), lib.gptoss_set_prefill_packing(pack)
        try:
            step(cap.cuda_stream)                          # sizes nothing new: same T
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                step(cap.cuda_stream, evh)
        finally:
            lib.gptoss_set_prefill_terms(pt)
            lib.gptoss_set_prefill_packing(pp)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        us = 0.0
        for _ in range(reps):
            g.replay()
            torch.cuda.synchronize()
            us += (ev[0].elapsed_time(ev[1]) + ev[2].elapsed_time(ev[3])) * 1e3
        out = (y - x).double()                            # the MoE output of the last replay
        del g
        return ctx.max(us / reps), out

    base_us, base = run(8, 0)
    scale, norm = base.abs().max().item(), base.norm().item()
    res = {}
    for nt, pack in [(n, 0) for n in range(1, 8)] + [(8, 0), (8, 1)]:
        us, out = (base_us, base) if (nt, pack) == (8, 0) else run(nt, pack)
        tf = prefill_flops(T) / (us * 1e-6) / 1e12
        d = out - base
        res[f"{nt}{'p' if pack else ''}"] = {
            "terms": nt, "plan": "packed" if pack else "stacked", "gemm_us": us, "algorithmic_tflops": tf,
            "frac": tf / peak, "rel_l2_vs_8_terms": d.norm().item() / norm,
            "max_abs_vs_8_terms_over_max": d.abs().max().item() / scale}
        del out, d
    return {"variants": res,
            "fewest_terms_meeting_reference_bound": {
                "terms": 7, "input": "the reference's test_moe_real_shape distribution (E = 6, scale bytes 118..123),"
                                     " batched: rtol 1e-4 / atol 1e-3 vs float64 (tests/test_prefill_gpu.py)",
                "frac": res["7"]["frac"], "algorithmic_tflops": res["7"]["algorithmic_tflops"]},
            "configs2_bound": "only 8 terms meet rtol 1e-4 / atol 1e-3 on configs[2] (outputs ~1e3)",
            "peak_tflops": peak, "reps": reps}


# ------------------------------------------------------------------------------------------------ expert parallel
def ep_row_bytes():
    """Bytes one (token, slot) row moves between ranks: its 8 activation terms written into the owner's A images
    (12 K blocks of 256 x 8 terms x (128 B of e2m1 + 32 B of replicated scales)), and its fp32 result row back."""
    kb = (H + 255) // 256
    return kb * 8 * (128 + 32), H * 4


def run_ep(args, ctx, lib, T, with_cpu):
    """Config 3: T tokens (over all ranks, T / N per rank) through 24 MoE layers per step, experts sharded over the
    N ranks (E / N each; placed by expected load from a calibration batch unless --ep-placement contiguous), tokens
    data-parallel. Per layer and rank: the library's batched router on the rank's tokens, dispatch of the (token,
    slot) rows to the experts' owners, the local experts on tensor cores, combine back in slot order. Strong
    scaling: the total token count is fixed."""
    import torch
    from gptoss_b200 import capi, ep, synth
    P = capi.ptr
    ws, rank, dev = ctx.ws, ctx.rank, ctx.dev
    if T % ws or E % ws:
        raise SystemExit(f"ep: {T} tokens and {E} experts must split evenly over {ws} ranks")
    Tl, El = T // ws, E // ws
    peer = args.ep_impl == "peer"
    balanced = args.ep_placement == "balanced" and ws > 1
    stream = torch.cuda.current_stream()
    # expected per-expert loads of every layer: the library's router on a calibration batch (2048 tokens drawn with
    # another seed than the benchmark's tokens), identical on every rank
    xc = torch.randn(2048, H, generator=torch.Generator().manual_seed(123)).to(torch.bfloat16).float().to(dev)
    placements, calib = [], []
    for li in range(args.layers):
        ln, W, b = (v.to(dev) for v in synth.ep_router(li))
        ids = torch.empty(2048, K_TOP, dtype=torch.int32, device=dev)
        w = torch.empty(2048, K_TOP, device=dev)
        hc = torch.empty_like(xc)
        if lib.gptoss_moe_route_batched(P(W), P(b), P(xc), P(ln), 1e-5, E, H, K_TOP, 2048, P(hc), P(ids), P(w),
                                        stream.cuda_stream) != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
        loads = torch.bincount(ids.flatten().long(), minlength=E).tolist()
        calib.append(loads)
        placements.append(ep.balanced_placement(loads, ws) if balanced else list(range(E)))
    del xc, hc
    epg = ep.EpGroup(lib, E, K_TOP, H, I, rank, ws, Tl) if peer else None
    layers, handles = [], []
    for li in range(args.layers):
        ln, W, b = (v.to(dev) for v in synth.ep_router(li))
        W, b = ep.apply_placement(placements[li], W, b)
        ex = synth.ep_experts_of(li, placements[li][rank * El:(rank + 1) * El], dev)
        hdl = lib.gptoss_moe_layer_create(P(ln), 1e-5, P(W), P(b), *(P(e) for e in ex), El,
                                          K_TOP if peer else min(K_TOP, El), H, I, 1.702, 7.0)
        if not hdl:
            raise RuntimeError(lib.gptoss_last_error().decode())
        handles.append(hdl)
        moe = (ep.PeerExpertParallelMoE(epg, hdl, W, b, ln) if peer else
               ep.ExpertParallelMoE(ep.gpu_route(lib, ln, W, b, E, K_TOP), ep.gpu_compute(lib, hdl), rank, ws, E,
                                    K_TOP, H, None))
        layers.append((ex, ln, W, b, moe))
    x_all = torch.randn(T, H, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).float()
    x_cpu = x_all[rank * Tl:(rank + 1) * Tl].contiguous()
    x0 = x_cpu.to(dev)
    x = torch.empty_like(x0)

    def step():
        x.copy_(x0)
        for L in layers:
            L[4].forward(x)

    # realised routing of every layer over the benchmark's tokens: rows each rank receives, rows crossing ranks
    h0 = torch.empty_like(x0)
    ids0 = torch.empty(Tl, K_TOP, dtype=torch.int32, device=dev)
    w0 = torch.empty(Tl, K_TOP, device=dev)
    recv = [0.0] * ws
    cross_rows = 0.0
    for li, (_, ln, W, b, _) in enumerate(layers):
        if lib.gptoss_moe_route_batched(P(W), P(b), P(x0), P(ln), 1e-5, E, H, K_TOP, Tl, P(h0), P(ids0), P(w0),
                                        stream.cuda_stream) != 0:
            raise RuntimeError(lib.gptoss_last_error().decode())
        to = torch.bincount(ids0.flatten().long() // El, minlength=ws).tolist()
        if li == 0:
            rows0 = to
        recv = [a + c for a, c in zip(recv, to)]
        cross_rows += sum(c for r, c in enumerate(to) if r != rank)
    recv = ctx.sum_list(recv)
    rows0 = ctx.sum_list(rows0)
    cross_rows = ctx.sum_list([cross_rows])[0]
    for _ in range(max(args.warmup, 3)):
        step()
    ctx.barrier()
    with ClockSampler(ctx.local) as clocks:
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        ctx.barrier()
    ms = ctx.max(e0.elapsed_time(e1))
    step_s = ms / args.steps / 1e3
    value = T / step_s
    # end to end: this rank's host tokens in (pinned), host result out, every step
    xh = x_cpu.pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    ctx.barrier()
    e0.record(stream)
    for _ in range(args.steps):
        x0.copy_(xh, non_blocking=True)
        step()
        yh.copy_(x, non_blocking=True)
    e1.record(stream)
    ctx.barrier()
    ms_e2e = ctx.max(e0.elapsed_time(e1))
    e2e = T / (ms_e2e / args.steps / 1e3)
    cpu = None
    if with_cpu:
        p = "model.layers.0."
        ex, ln, W, b, _ = layers[0]
        ln0, W0, b0 = synth.ep_router(0)
        t = {p + "post_attention_layernorm.weight": ln0.to(torch.bfloat16), p + "mlp.router.weight": W0,
             p + "mlp.router.bias": b0.to(torch.bfloat16)}
        for n, v in zip(["gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
                         "down_proj_scales", "down_proj_bias"], synth.ep_experts(0, 0, E, "cpu")):
            t[p + "mlp.experts." + n] = v
        rm = ReferenceMoE(t)
        hn = rm.normed(x_cpu[:128])
        el, n, _ = time_reference(rm, hn, 32, 4, 1, 20.0)
        cpu = {"value": n / el / args.layers, "unit": "tok/s", "cores": rm.cores, "kind": rm.kind,
               "sample": f"{n} tokens (32 per call) through layer 0 with {rm.what}, scaled by 1/{args.layers} "
                         f"layers"}
    peak, peak_src = fp4_peak(lib, sustained=True)
    flops = prefill_flops(T) * args.layers
    achieved = flops / ws / step_s / 1e12
    disp_b, comb_b = ep_row_bytes()
    nvlink_bytes = cross_rows * (disp_b + comb_b)            # per step, all ranks together
    ep_status = epg.status() if peer else 0
    if peer:
        epg.close()
    for hdl in handles:
        lib.gptoss_moe_layer_destroy(hdl)
    del layers
    torch.cuda.empty_cache()
    if ep_status:
        raise RuntimeError(f"expert-parallel device check failed (code {ep_status})")
    cfg = ep_config(T, ws, args.layers)
    cfg.update({
        "placement": ("by expected load: greedy over the per-expert counts of a 2048-token calibration batch "
                      "(ep.balanced_placement), experts relabelled so each rank's range is balanced")
        if balanced else "contiguous expert ids",
        "dispatch": ("inside the kernels: A terms and result rows stored into peer memory over NVLink "
                     "(gptoss_ep_layer_forward)" if peer else "torch.distributed all_to_all_single (NCCL)")
        if ws > 1 else "none (one rank)"})
    return {
        "metric": EP_METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "e2m1 x e2m1 (fp32 accumulate; activations as 8 residual terms)",
        "data": "synthetic (seeded random-init 20b-shaped MoE layers, bf16 N(0,1) tokens)",
        "config": cfg,
        "tok_per_s": value,
        "rows_per_rank_layer0": rows0,
        "rows_per_rank_all_layers": recv,
        "max_over_mean_rows": max(recv) / (sum(recv) / ws),
        "roofline": {"bound": "tensor", "kernel": "whole expert-parallel step per GPU (router, dispatch, grouped "
                                                  "tcgen05 GEMMs, combine)",
                     "achieved": achieved, "unit": "TFLOP/s", "peak": peak, "peak_source": peak_src,
                     "frac": achieved / peak, "algorithmic_flops_per_step": flops, "traffic": None},
        "nvlink": {"off_rank_rows_per_step": cross_rows, "bytes_per_step": nvlink_bytes,
                   "GBps_all_ranks": nvlink_bytes / step_s / 1e9,
                   "GBps_per_gpu": nvlink_bytes / ws / step_s / 1e9,
                   "bytes_per_row": {"dispatch": disp_b, "combine": comb_b}},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                "api": ("PeerExpertParallelMoE" if peer else "ExpertParallelMoE") +
                       ".forward per layer; host tokens copied in and out every step"},
        # peer: router, counts, permute, quantize, barrier, GEMM, quantize, GEMM, barrier, combine;
        # nccl: w64, router, permute, 2 x (quantize, GEMM), combine
        "gpu_launches": args.steps * args.layers * (10 if peer else 8),
        "clocks": clocks.summary(),
    }


# ------------------------------------------------------------------------------------------------ full decode step
DECODE_V = 201088
DECODE_BYTES_PER_TOKEN = 3_705_753_600     # 24 x (QKV + O + router + 4 experts) + LM head, bf16 / MXFP4 as stored


def write_20b_checkpoint(d, layers=LAYERS, seed=0):
    """A random-init gpt-oss-20b-shaped checkpoint in the Hugging Face safetensors layout, one shard per
    layer plus one for the embeddings, norm and LM head, with model.safetensors.index.json and config.json.
    Attention and LM head bf16 N(0, 0.02), sinks N(0, 1), RMSNorm weights 1 + N(0, 0.02), embeddings N(0, 1), MoE as
    configs[0] (blocks uniform over all codes, scales uniform 120..126, biases N(0, 0.01), router N(0, 0.02) / bias
    N(0, 0.01)). Drawn on the GPU from a seeded generator, written from host memory."""
    import torch
    from safetensors.torch import save_file
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = lambda *s, std=1.0: (torch.randn(*s, device="cuda", generator=g) * std).to(torch.bfloat16).cpu()
    u8 = lambda lo, hi, *s: torch.randint(lo, hi, s, device="cuda", generator=g, dtype=torch.uint8).cpu()
    index = {}
    top = {"model.embed_tokens.weight": n(DECODE_V, H), "lm_head.weight": n(DECODE_V, H, std=0.02),
           "model.norm.weight": (1 + torch.randn(H, device="cuda", generator=g) * 0.02).to(torch.bfloat16).cpu()}
    save_file(top, str(d / "model-top.safetensors"))
    index.update({k: "model-top.safetensors" for k in top})
    del top
    for l in range(layers):
        p = f"model.layers.{l}."
        t = {p + "input_layernorm.weight": (1 + torch.randn(H, device="cuda", generator=g) * 0.02).to(torch.bfloat16).cpu(),
             p + "post_attention_layernorm.weight": (1 + torch.randn(H, device="cuda", generator=g) * 0.02).to(torch.bfloat16).cpu(),
             p + "self_attn.q_proj.weight": n(4096, H, std=0.02), p + "self_attn.q_proj.bias": n(4096, std=0.02),
             p + "self_attn.k_proj.weight": n(512, H, std=0.02), p + "self_attn.k_proj.bias": n(512, std=0.02),
             p + "self_attn.v_proj.weight": n(512, H, std=0.02), p + "self_attn.v_proj.bias": n(512, std=0.02),
             p + "self_attn.o_proj.weight": n(H, 4096, std=0.02), p + "self_attn.o_proj.bias": n(H, std=0.02),
             p + "self_attn.sinks": n(64), p + "mlp.router.weight": n(E, H, std=0.02), p + "mlp.router.bias": n(E, std=0.01)}
        for name, rows, kk in (("gate_up_proj", 2 * I, H), ("down_proj", H, I)):
            q = p + "mlp.experts." + name
            t[q + "_blocks"] = u8(0, 256, E, rows, kk // 32, 16)
            t[q + "_scales"] = u8(120, 127, E, rows, kk // 32)
            t[q + "_bias"] = n(E, rows, std=0.01)
        f = f"model-layer{l:02d}.safetensors"
        save_file(t, str(d / f))
        index.update({k: f for k in t})
        del t
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": index}))
    cfg = {"num_hidden_layers": layers, "hidden_size": H, "intermediate_size": I, "vocab_size": DECODE_V,
           "num_local_experts": E, "num_experts_per_tok": K_TOP, "sliding_window": 128, "num_attention_heads": 64,
           "num_key_value_heads": 8, "head_dim": 64, "max_position_embeddings": 131072, "rms_norm_eps": 1e-5,
           "swiglu_limit": 7.0, "rope_theta": 150000,
           "layer_types": ["sliding_attention" if l % 2 == 0 else "full_attention" for l in range(layers)],
           "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                            "truncate": False, "original_max_position_embeddings": 4096}}
    (d / "config.json").write_text(json.dumps(cfg))


def run_decode_step(args, ctx, lib, context=4096, new_tokens=128, reps=7):
    """bs=1 greedy decode of `new_tokens` tokens of the 20b-shaped random-init model through the engine
    entry points (gptoss_create on the written checkpoint, gptoss_kv_fill_random for the 4096-position fp16 context,
    gptoss_generate_greedy: argmax on the device, no host round trip per token). Timed through the API (host clock
    around the synchronous call, which covers every kernel of every step), median of `reps` runs after a warm-up
    that also captures the step graph."""
    import shutil
    import statistics
    import tempfile
    t0 = time.time()
    d = Path(tempfile.mkdtemp(prefix="gptoss20b_", dir=os.environ.get("GPTOSS_BENCH_TMP", "/tmp")))
    try:
        write_20b_checkpoint(d, args.layers)
        t_write = time.time() - t0
        t1 = time.time()
        e = lib.gptoss_create(str(d).encode(), context + new_tokens + 64, 0)
        if not e:
            raise RuntimeError(lib.gptoss_last_error().decode())
        t_load = time.time() - t1
    finally:
        shutil.rmtree(d, ignore_errors=True)
    import ctypes
    import numpy as np
    try:
        dev_bytes = lib.gptoss_device_bytes(e)
        out = np.zeros(new_tokens, np.int32)

        def run():
            if lib.gptoss_kv_fill_random(e, context, 11) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())
            t = time.perf_counter()
            if lib.gptoss_generate_greedy(e, 1, new_tokens, out.ctypes.data) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())
            return time.perf_counter() - t

        run()                                               # warm-up: eager first step, graph capture
        with ClockSampler(ctx.local) as clocks:
            times = [run() for _ in range(reps)]
        # batched prefill of a 2048-token prompt through gptoss_prefill (from position 0; warm-up run first)
        prompt = (np.arange(2048, dtype=np.int64) * 7919 % DECODE_V).astype(np.int32)
        pre_times = []
        for i in range(3):
            if lib.gptoss_reset(e) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())
            t = time.perf_counter()
            if lib.gptoss_prefill(e, prompt.ctypes.data, len(prompt), None, 0, None, None, None) != 0:
                raise RuntimeError(lib.gptoss_last_error().decode())
            pre_times.append(time.perf_counter() - t)
        sec = statistics.median(times)
        tok_s = new_tokens / sec
        kv_bytes = 12 * (context + new_tokens // 2) * 2048 + 12 * 128 * 2048
        pk = peaks()
        hbm = pk.get("hbm_gbs") or 6650.0
        achieved = (DECODE_BYTES_PER_TOKEN + kv_bytes) * tok_s / 1e9
        return {
            "metric": "bs=1 decode tok/s (20b-shaped, greedy, 4096-position fp16 KV context)",
            "value": tok_s, "unit": "tok/s", "higher_is_better": True, "new_tokens": new_tokens, "reps": reps,
            "ms_per_token": sec / new_tokens * 1e3, "run_seconds": times,
            "best_tok_per_s": new_tokens / min(times),
            "config": {"workload": "configs[1]: 24 layers, hidden 2880, vocab 201088, 64/8 heads, window 128 on even "
                                   "layers, MoE as configs[0]", "context": context, "kv": "fp16 N(0,1) (seeded)",
                       "sampling": "greedy (argmax on the device)"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (GEMVs, attention, fused MoE, LM head)",
                         "algorithmic_bytes_per_token": DECODE_BYTES_PER_TOKEN + kv_bytes, "achieved": achieved,
                         "unit": "GB/s", "peak": hbm, "frac": achieved / hbm,
                         "frac_of_8TBs_nominal": achieved / 8000.0},
            "api": "gptoss_create + gptoss_kv_fill_random + gptoss_generate_greedy (one CUDA graph per step)",
            "engine_prefill": {"tokens": len(prompt), "seconds": pre_times[1:],
                               "tok_per_s": len(prompt) / statistics.median(pre_times[1:]),
                               "api": "gptoss_prefill (batched: tensor-core projections, grouped-GEMM MoE), host "
                                      "clock around the synchronous call"},
            "setup_s": {"write_checkpoint": t_write, "gptoss_create": t_load}, "device_bytes": dev_bytes,
            "first_tokens": out[:8].tolist(),
            "clocks": clocks.summary(),
        }
    finally:
        lib.gptoss_destroy(e)


# ------------------------------------------------------------------------------------------------ reference GPU bar
def run_ref_gpu(ctx, lib):
    """The reference's own CUDA kernels (openvang/gptoss-infer runtime/src/kernels.cu, built for sm_100a from its
    sources by oracle/Makefile) against this library's, through the same C ABI entry points on the same inputs (the
    config-0 layer, one token): host wall time of each synchronous call, median of 50 after 5 warm-up calls. The
    reference allocates and frees its scratch inside gptoss_kernel_moe (runtime/src/capi.cpp:127-144), so its
    figure includes that, as a caller sees it."""
    import ctypes
    import statistics
    import torch
    from gptoss_b200 import capi, synth
    if not REF_LIB.exists():
        return {"unavailable": "oracle/_ref/libgptoss_ref.so not built (reference sources absent at build time)"}
    P = capi.ptr
    ref = ctypes.CDLL(str(REF_LIB))
    ref.gptoss_last_error.restype = ctypes.c_char_p
    for lb in (ref,):
        lb.gptoss_kernel_router.argtypes = capi.SIGNATURES["gptoss_kernel_router"][0]
        lb.gptoss_kernel_moe.argtypes = capi.SIGNATURES["gptoss_kernel_moe"][0]
    t = synth.moe_layer(seed=0)
    p = "model.layers.0."
    dev = ctx.dev
    ex = [t[p + "mlp.experts." + n].to(dev) for n in ("gate_up_proj_blocks", "gate_up_proj_scales",
                                                      "gate_up_proj_bias", "down_proj_blocks", "down_proj_scales",
                                                      "down_proj_bias")]
    ex[2], ex[5] = ex[2].float(), ex[5].float()
    W, b = t[p + "mlp.router.weight"].to(dev), t[p + "mlp.router.bias"].float().to(dev)
    x = synth.tokens(1, seed=8)[0].to(dev)
    ids = torch.empty(4, dtype=torch.int32, device=dev)
    w = torch.empty(4, device=dev)
    out = torch.zeros(H, device=dev)

    def timed(fn):
        for _ in range(5):
            assert fn() == 0
        ts = []
        for _ in range(50):
            t0 = time.perf_counter()
            assert fn() == 0
            ts.append((time.perf_counter() - t0) * 1e6)
        return statistics.median(ts)

    res = {}
    for name, lb in (("reference", ref), ("ours", lib)):
        r_us = timed(lambda: lb.gptoss_kernel_router(P(W), P(b), P(x), E, H, K_TOP, P(ids), P(w)))
        m_us = timed(lambda: lb.gptoss_kernel_moe(*(P(e) for e in ex), P(x), P(ids), P(w), P(out), K_TOP, H, I,
                                                  1.702, 7.0))
        res[name] = {"kernel_router_us": r_us, "kernel_moe_us": m_us}
    res["moe_speedup"] = res["reference"]["kernel_moe_us"] / res["ours"]["kernel_moe_us"]
    res["router_speedup"] = res["reference"]["kernel_router_us"] / res["ours"]["kernel_router_us"]
    res["note"] = ("host wall time per synchronous ABI call (one token, config-0 layer, H = I = 2880, k = 4); ours "
                   "is the raw-weights entry point (per-call scale gather), not the prepared layer")
    return res


# ------------------------------------------------------------------------------------------------------- reference arm
def run_reference(args):
    """Reference arm: the reference's CPU implementation of this path on the host cores, rank 0 only, a bounded sample
    per step, the same metric, unit and config as the GPU arm."""
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from gptoss_b200 import synth
    if args.workload == "moe-decode":
        t0 = synth.moe_layer(seed=0)
        rm = ReferenceMoE(t0)
        h = rm.normed(torch.randn(64, H, generator=torch.Generator().manual_seed(99)))
        el, n, timed = time_reference(rm, h, 1, args.steps, args.warmup, REF_BUDGET_S)
        value, unit, metric, cfg, scaling = LAYER_BYTES * n / el / 1e9, UNIT, METRIC, decode_config(ws, args.layers), \
            "weak"
        sample = f"one token through one MoE layer (config-0 layer) per step, {rm.what}"
        ms = el / timed * 1e3
    elif args.workload == "prefill":
        t, _, x = prefill_inputs(args.tokens)
        rm = ReferenceMoE(t)
        h = rm.normed(x[:512])
        el, n, timed = time_reference(rm, h, 64, args.steps, args.warmup, REF_BUDGET_S)
        value, unit, metric, cfg, scaling = n / el, "tok/s", PREFILL_METRIC, prefill_config(args.tokens, ws), "weak"
        sample = f"64 tokens per step through {rm.what}"
        ms = el / timed * 1e3
    else:
        p = "model.layers.0."
        ln0, W0, b0 = synth.ep_router(0)
        t = {p + "post_attention_layernorm.weight": ln0.to(torch.bfloat16), p + "mlp.router.weight": W0,
             p + "mlp.router.bias": b0.to(torch.bfloat16)}
        for nm, v in zip(["gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
                          "down_proj_scales", "down_proj_bias"], synth.ep_experts(0, 0, E, "cpu")):
            t[p + "mlp.experts." + nm] = v
        rm = ReferenceMoE(t)
        x = torch.randn(256, H, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).float()
        h = rm.normed(x)
        el, n, timed = time_reference(rm, h, 32, args.steps, args.warmup, REF_BUDGET_S)
        value, unit, metric, cfg, scaling = n / el / args.layers, "tok/s", EP_METRIC, \
            ep_config(args.tokens, ws, args.layers), "strong"
        sample = f"32 tokens per step through layer 0 with {rm.what}, scaled by 1/{args.layers} layers"
        ms = el / timed * 1e3 * args.layers
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": ws, "steps": args.steps,
            "steps_timed": timed, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": value, "unit": unit, "cores": rm.cores, "kind": rm.kind, "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------------- main
def main():
    args = parse()
    if args.tokens is None:
        args.tokens = 8192 if args.workload == "ep" else 2048
    if args.impl == "reference":
        return run_reference(args)
    from gptoss_b200 import capi
    ctx = Ctx()
    lib = capi.load()
    try:
        first = ctx.rank == 0 and ctx.ws == 1 and not args.no_cpu_baseline
        if args.workload == "ep":
            line = run_ep(args, ctx, lib, args.tokens, first)
        elif args.workload == "prefill":
            line = run_prefill(args, ctx, lib, args.tokens, first)
        elif args.workload == "decode":
            line = run_decode_step(args, ctx, lib, new_tokens=args.decode_tokens, reps=args.decode_reps)
        else:
            line = run_decode(args, ctx, lib)
            if not args.no_extras:
                line["ep"] = run_ep(args, ctx, lib, 8192, False)
                if ctx.ws == 1:
                    line["prefill"] = run_prefill(args, ctx, lib, 2048, False)
                    line["ref_gpu"] = run_ref_gpu(ctx, lib)
                    line["decode"] = run_decode_step(args, ctx, lib)
        if ctx.rank == 0:
            print(json.dumps(line))
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
