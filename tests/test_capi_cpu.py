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


def test_errors_cross_the_abi_as_minus_one(lib):
    assert lib.gptoss_set_moe_impl(7) == -1
    assert b"impl" in lib.gptoss_last_error()
    prev = lib.gptoss_set_moe_impl(0)
    assert prev in (0, 1)
    assert lib.gptoss_set_moe_impl(prev) == 0

