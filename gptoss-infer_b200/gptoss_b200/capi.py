"""ctypes binding of libgptoss.so (include/gptoss.h), the way the reference's callers bind it
(openvang/gptoss-infer runtime/tests/test_kernels.py:16-27, runtime/tools/score_golden.py:20-34).

The library is the product: there is no Python or CPU fallback. `load()` raises if the shared object is missing;
build it with `python gptoss-infer_b200/build.py` (or `__graft_entry__.build()`).
"""
import ctypes
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
ROOT = PKG.parent
HEADER = ROOT / "include" / "gptoss.h"
DEFAULT_LIB = PKG / "lib" / "libgptoss.so"

P, I32, I64, F32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float

# argtypes per entry point; the first six follow runtime/tests/test_kernels.py:153-160 exactly.
SIGNATURES = {
    "gptoss_kernel_gemv_bf16": ([P, P, P, P, P, I32, I32], I32),
    "gptoss_kernel_rmsnorm": ([P, P, P, I32, F32], I32),
    "gptoss_kernel_rope_append": ([P, P, P, I32, P, P, I32], I32),
    "gptoss_kernel_attention": ([P, P, P, P, I32, I32, I32, P], I32),
    "gptoss_kernel_router": ([P, P, P, I32, I32, I32, P, P], I32),
    "gptoss_kernel_moe": ([P, P, P, P, P, P, P, P, P, P, I32, I32, I32, F32, F32], I32),
    "gptoss_kernel_moe_static_scratch": ([P, P, P, P, P, P, P, P, P, P, I32, I32, I32, F32, F32], I32),
    "gptoss_kernel_mxfp4_dequant": ([P, P, P, I64], I32),
    "gptoss_kernel_router_batched": ([P, P, P, I32, I32, I32, I32, P, P], I32),
    "gptoss_moe_route_batched": ([P, P, P, P, F32, I32, I32, I32, I32, P, P, P, P], I32),
    "gptoss_kernel_moe_batched": ([P, P, P, P, P, P, P, P, P, P, I32, I32, I32, I32, F32, F32], I32),
    "gptoss_moe_layer_forward_batched": ([P, P, P, I32, P, P], I32),
    "gptoss_moe_layer_experts_batched": ([P, P, P, P, P, I32, I32, P], I32),
    "gptoss_router_w64": ([P, I32, I32, P, P], I32),
    "gptoss_ep_region_bytes": ([I32, I32, I32, I32, I32, I32, P], I32),
    "gptoss_ep_region_alloc": ([ctypes.c_longlong, P], I32),
    "gptoss_ep_region_free": ([P], I32),
    "gptoss_ipc_handle": ([P, P], I32),
    "gptoss_ipc_open": ([P, P], I32),
    "gptoss_ipc_close": ([P], I32),
    "gptoss_ep_layer_forward": ([P, P, P, P, F32, I32, I32, I32, P, P, I32, I32, P, ctypes.c_uint, P], I32),
    "gptoss_ep_status": ([I32, I32, I32, I32, I32, I32, P], I32),
    "gptoss_set_moe_impl": ([I32], I32),
    "gptoss_set_attention_impl": ([I32], I32),
    "gptoss_set_prefill_terms": ([I32], I32),
    "gptoss_set_prefill_packing": ([I32], I32),
    "gptoss_test_decode_epoch": ([I32, I32, I32, ctypes.c_uint, P], I32),
    "gptoss_trace_enable": ([P, I64], I32),
    "gptoss_selftest_terms": ([P, I32, P, P, I32], I32),
    "gptoss_selftest_mxf4_gemm": ([P, P, P, P, P, I32, I32], I32),
    "gptoss_selftest_mxf4_gemm_swizzle": ([P, P, P, P, P, I32, I32, I32], I32),
    "gptoss_selftest_mxf4_peak": ([P], I32),
    "gptoss_selftest_mxf4_mma_ns": ([I32, P], I32),
    "gptoss_moe_layer_create": ([P, F32, P, P, P, P, P, P, P, P, I32, I32, I32, I32, F32, F32], P),
    "gptoss_moe_layer_destroy": ([P], None),
    "gptoss_moe_layer_forward": ([P, P, P, P, P], I32),
    "gptoss_moe_block_async": ([P, P, F32, P, P, P, P, P, P, P, P, P, I32, I32, I32, I32, F32, F32, P, P], I32),
    "gptoss_create": ([ctypes.c_char_p, I32, I64], P),
    "gptoss_destroy": ([P], None),
    "gptoss_vocab": ([P], I32),
    "gptoss_position": ([P], I32),
    "gptoss_device_bytes": ([P], I64),
    "gptoss_reset": ([P], I32),
    "gptoss_use_graph": ([P, I32], I32),
    "gptoss_step": ([P, I32], I32),
    "gptoss_logits": ([P, P], I32),
    "gptoss_prefill": ([P, P, I32, P, I32, P, P, P], I32),
    "gptoss_score": ([P, P, I32, I32, P, P, P, P], I32),
    "gptoss_set_position": ([P, I32], I32),
    "gptoss_bench_steps": ([P, I32, I32], I32),
    "gptoss_generate_greedy": ([P, I32, I32, P], I32),
    "gptoss_kv_fill_random": ([P, I32, ctypes.c_ulonglong], I32),
}

_lib = None


def header_functions():
    """Names of every function include/gptoss.h declares."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gptoss_\w+)\s*\(", text)))


def load(path=None):
    global _lib
    if _lib is not None and path is None:
        return _lib
    path = Path(path or os.environ.get("GPTOSS_LIB", DEFAULT_LIB))
    if not path.exists():
        raise FileNotFoundError(f"{path} is missing: build it with python gptoss-infer_b200/build.py")
    lib = ctypes.CDLL(str(path))
    lib.gptoss_last_error.restype = ctypes.c_char_p
    lib.gptoss_last_error.argtypes = []
    for name, (args, res) in SIGNATURES.items():
        if not hasattr(lib, name):
            if path == DEFAULT_LIB:
                raise AttributeError(f"{path} does not export {name}")
            continue                      # another library of the same ABI (e.g. the reference's) may lack extensions
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path == DEFAULT_LIB or _lib is None:
        _lib = lib
    return lib


class GptossError(RuntimeError):
    pass


def check(rc, lib=None):
    if rc != 0:
        lib = lib or load()
        raise GptossError(lib.gptoss_last_error().decode())
    return rc


def ptr(t):
    return None if t is None else t.data_ptr()
