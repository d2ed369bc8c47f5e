"""CPU-side checks of the C ABI: the library loads and exports every function include/gptoss.h declares, with no
compute call (there is no GPU here)."""
import pytest

from gptoss_b200 import capi


@pytest.fixture(scope="module")
def lib():
    from gptoss_b200 import capi as c
    if not c.DEFAULT_LIB.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("gptoss_build", c.PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return c.load()


def test_header_lists_the_reference_abi():
    names = set(capi.header_functions())
    reference_abi = {  # runtime/include/gptoss/gptoss.h:17-58 of openvang/gptoss-infer
        "gptoss_create", "gptoss_destroy", "gptoss_last_error", "gptoss_vocab", "gptoss_position",
        "gptoss_device_bytes", "gptoss_reset", "gptoss_use_graph", "gptoss_step", "gptoss_logits",
        "gptoss_prefill", "gptoss_score", "gptoss_set_position", "gptoss_bench_steps", "gptoss_kernel_gemv_bf16",
        "gptoss_kernel_rmsnorm", "gptoss_kernel_rope_append", "gptoss_kernel_attention", "gptoss_kernel_router",
        "gptoss_kernel_moe"}
    assert reference_abi <= names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in capi.header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(capi.SIGNATURES) <= set(capi.header_functions())


def test_invalid_shapes_are_rejected_before_any_device_work(lib):
    """Argument checks that run before the first CUDA call, so they hold without a GPU: k > E must fail
    (runtime/tests/test_kernels.py:145), and so must k outside 1..8, an empty batch and H not a multiple of 8."""
    cases = [
        (lambda: lib.gptoss_kernel_router(None, None, None, 4, 64, 5, None, None), b"k <= E"),
        (lambda: lib.gptoss_kernel_router(None, None, None, 32, 60, 4, None, None), b"H % 8"),
        (lambda: lib.gptoss_kernel_router_batched(None, None, None, 4, 64, 5, 16, None, None), b"k <= E"),
        (lambda: lib.gptoss_kernel_router_batched(None, None, None, 32, 64, 4, 0, None, None), b"T >= 1"),
        (lambda: lib.gptoss_kernel_moe(None, None, None, None, None, None, None, None, None, None, 9, 64, 64,
                                       1.702, 7.0), b"k must be in 1..8"),
        (lambda: lib.gptoss_kernel_moe_batched(None, None, None, None, None, None, None, None, None, None, 0, 4,
                                               64, 64, 1.702, 7.0), b"T >= 1"),
        (lambda: lib.gptoss_moe_layer_forward_batched(None, None, None, 4, None, None), b"null layer"),
    ]
    for call, msg in cases:
        assert call() == -1
        assert msg in lib.gptoss_last_error(), (msg, lib.gptoss_last_error())


def test_errors_cross_the_abi_as_minus_one(lib):
    assert lib.gptoss_set_moe_impl(7) == -1
    assert b"impl" in lib.gptoss_last_error()
    prev = lib.gptoss_set_moe_impl(0)
    assert prev in (0, 1)
    assert lib.gptoss_set_moe_impl(prev) == 0
    assert lib.gptoss_set_attention_impl(2) == -1
    assert b"impl" in lib.gptoss_last_error()
    prev = lib.gptoss_set_attention_impl(0)
    assert prev in (0, 1)
    assert lib.gptoss_set_attention_impl(prev) == 0

