"""Stages openvang/gptoss-infer's own Python code into baseline/_ref/ so that it travels to the GPU box as test and
benchmark infrastructure (baseline/_ref/ is git-ignored: nothing staged here is part of this repository's history).

    python oracle/stage_reference.py [REFERENCE_CHECKOUT]

REFERENCE_CHECKOUT defaults to $GPTOSS_REF_ROOT, else a sibling directory named `reference` next to this repository.
What is staged, unchanged:
  baseline/_ref/reference/gptoss_ref/   the fp32 reference package (reference/gptoss_ref/*.py): bench.py's reference
                                        arm and cpu_baseline time its Reference.moe; the reference's kernel tests
                                        import mxfp4, rope and config from it
  baseline/_ref/runtime_tests/test_kernels.py
                                        the reference's own kernel tests (runtime/tests/test_kernels.py), which
                                        tests/test_reference_kernel_suite.py runs against this build's libgptoss.so
Test infrastructure only: no product code imports anything under baseline/_ref/.
"""
import os
import shutil
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DEST = ROOT / "baseline" / "_ref"


def stage(ref: Path) -> Path:
    pkg = ref / "reference" / "gptoss_ref"
    tests = ref / "runtime" / "tests" / "test_kernels.py"
    if not (pkg / "model.py").exists() or not tests.exists():
        raise SystemExit(f"stage_reference: {ref} does not look like an openvang/gptoss-infer checkout")
    out_pkg = DEST / "reference" / "gptoss_ref"
    out_tests = DEST / "runtime_tests"
    out_pkg.mkdir(parents=True, exist_ok=True)
    out_tests.mkdir(parents=True, exist_ok=True)
    for f in sorted(pkg.glob("*.py")):
        shutil.copyfile(f, out_pkg / f.name)
    shutil.copyfile(tests, out_tests / "test_kernels.py")
    return DEST


if __name__ == "__main__":
    src = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(os.environ.get("GPTOSS_REF_ROOT", ROOT.parent / "reference"))
    print(stage(src))
