"""The reference's own CPU test files (tests/test_quant.py, tests/test_dispatch.py of lowbit-kernels), run
unmodified against this package with the reference's dispatch constants. Opt-in: set LOWBIT_REFERENCE_TESTS to
the reference checkout's tests directory; skipped otherwise (the directory is never needed elsewhere)."""
import os
import pathlib
import shutil
import subprocess
import sys
import tempfile

import pytest

PKG = pathlib.Path(__file__).resolve().parent.parent / "lowbit-kernels_b200"


@pytest.mark.skipif(not os.environ.get("LOWBIT_REFERENCE_TESTS"), reason="LOWBIT_REFERENCE_TESTS is not set")
def test_reference_cpu_tests_pass_against_this_package():
    src = pathlib.Path(os.environ["LOWBIT_REFERENCE_TESTS"])
    with tempfile.TemporaryDirectory() as tmp:
        dst = pathlib.Path(tmp) / "tests"
        shutil.copytree(src, dst)
        env = dict(os.environ, PYTHONPATH=str(PKG), LOWBIT_DISPATCH="reference")
        r = subprocess.run([sys.executable, "-m", "pytest", str(dst), "-q", "-p", "no:cacheprovider"],
                           env=env, capture_output=True, text=True, cwd=tmp)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
