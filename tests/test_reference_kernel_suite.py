"""openvang/gptoss-infer's own kernel tests (runtime/tests/test_kernels.py), unchanged, run against this build's
libgptoss.so through the reference's ctypes binding (its GPTOSS_LIB switch): the drop-in proof for the C ABI.

oracle/stage_reference.py copies the reference's test file and its fp32 package gptoss_ref (which the tests import
for mxfp4, rope and the model config) into baseline/_ref/, git-ignored, which travels to the GPU box; without that
staging this module is skipped. The reference's test functions are collected here under the `gpu` mark, each with
the reference's own inputs and tolerances (float64 references; the MoE at rtol 1e-4 / atol 1e-3). Only the tests
whose entry points this build implements are collected.
"""
import importlib.util
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
STAGED = ROOT / "baseline" / "_ref"
SUITE = STAGED / "runtime_tests" / "test_kernels.py"
LIB = ROOT / "gptoss-infer_b200" / "lib" / "libgptoss.so"

# the reference's test functions whose entry points are implemented here
IMPLEMENTED = ["test_gemv_bf16", "test_rmsnorm", "test_rope_append", "test_attention", "test_router", "test_moe_real_shape"]

if not SUITE.exists() or not (STAGED / "reference" / "gptoss_ref" / "model.py").exists():
    pytest.skip("the reference's kernel tests are not staged (python oracle/stage_reference.py)",
                allow_module_level=True)
if not LIB.exists():
    pytest.skip("libgptoss.so is not built", allow_module_level=True)

os.environ["GPTOSS_LIB"] = str(LIB)
if str(STAGED / "reference") not in sys.path:
    sys.path.insert(0, str(STAGED / "reference"))
_spec = importlib.util.spec_from_file_location("gptoss_reference_kernel_tests", SUITE)
_suite = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_suite)

for _name in IMPLEMENTED:
    globals()[_name] = pytest.mark.gpu(getattr(_suite, _name))
