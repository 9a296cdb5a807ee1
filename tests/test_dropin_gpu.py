"""The C++ drop-in check: the reference's own self-test program
(src/main.cpp of INFERNT, unchanged: 18 test cases over Tensor,
ModelConfig, CublasWrapper::gemm, the launch_* kernels, KVCache,
LlamaArchitecture::forward, Tokenizer, CheckpointLoader, the sampling path,
InferenceEngine generation and a second architecture shape) compiled against
this repository's include/ and linked with libinfernt_b200.so in place of
the reference's objects (oracle/Makefile, target selftest).  It must report
every test passed and exit 0.

The program is built where the reference checkout exists (build() runs
`make -C oracle`); without it this test skips."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SELFTEST = os.path.join(ROOT, "oracle", "_ref", "ref_selftest")


def test_reference_selftest_passes_against_this_library():
    if not os.path.exists(SELFTEST):
        pytest.skip("reference self-test not built (no reference checkout at build time)")
    r = subprocess.run([SELFTEST], capture_output=True, text=True, timeout=600, cwd="/tmp")
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    # every run_test case of the program's main (src/main.cpp:889-927)
    assert "Results: 18 passed, 0 failed" in out, out[-4000:]
    # the library loaded is this repository's
    maps = subprocess.run(["ldd", SELFTEST], capture_output=True, text=True).stdout
    assert os.path.join(ROOT, "infernt_b200", "lib", "libinfernt_b200.so") in maps or "libinfernt_b200.so" in maps
