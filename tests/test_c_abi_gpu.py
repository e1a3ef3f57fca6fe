"""The C ABI from C: tests/c_abi_gated_scan.c, compiled with gcc against
include/need_scan.h and linked with libneed_scan.so, the C oracle and the
CUDA runtime, runs the gated scan on the GPU and checks it against the oracle
with no Python in the loop (the way an engine plugin or a C++ host would call
the library)."""
import os
import subprocess

import pytest

from need_b200 import build

import oracle

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_gated_scan_from_c(tmp_path):
    lib_dir = os.path.dirname(build.build())
    ora_dir = os.path.dirname(oracle.build())
    exe = tmp_path / "c_abi_gated_scan"
    subprocess.run(["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror",
                    os.path.join(ROOT, "tests", "c_abi_gated_scan.c"),
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
                    "-L", lib_dir, "-lneed_scan", "-L", ora_dir, "-lneed_scan_oracle",
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-lm", "-o", str(exe)], check=True)
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = ":".join([lib_dir, ora_dir, os.path.join(CUDA, "lib64"),
                                       env.get("LD_LIBRARY_PATH", "")])
    r = subprocess.run([str(exe)], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "C-ABI-OK" in r.stdout, r.stdout
