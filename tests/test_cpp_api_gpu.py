"""The C++ owners of include/cubutterfly/plan.hpp on the GPU: a C++ program
runs the reference C test's 5-point FFT (tests/test_c_api.c:49-108) through
Context / Plan (owned workspace) and checks it itself."""
import subprocess

import pytest

from test_abi import ROOT, compile_cpp

pytestmark = pytest.mark.gpu


def test_cpp_plan_runs_the_reference_five_point_fft(tmp_path):
    exe = compile_cpp(ROOT / "tests" / "cpp" / "plan_api_gpu.cpp", tmp_path / "plan_api_gpu")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    words = r.stdout.split()
    assert r.returncode == 0 and words[0] == "ok", r.stdout + r.stderr
    assert words[1].startswith("bluestein[16:")
