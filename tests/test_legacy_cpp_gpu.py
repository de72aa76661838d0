"""Build and run tests/cpp/legacy18.cu: the reference's 18-case harness with only
its include switched to include/kf_attn_compat.h (drop-in check in C++)."""
from __future__ import annotations

import os
import subprocess

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

BIN_DIR = os.path.join(REPO, "tests", "cpp", "bin")


def build_legacy_harness() -> str:
    from kernelfoundry_b200.build import LIB_DIR, _nvcc, build

    import oracle

    build()
    oracle.build_c_oracle()
    os.makedirs(BIN_DIR, exist_ok=True)
    exe = os.path.join(BIN_DIR, "legacy18")
    cmd = [_nvcc(), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", os.path.join(REPO, "include"), os.path.join(REPO, "tests", "cpp", "legacy18.cu"),
           "-L", LIB_DIR, "-lkf_attn", f"-Xlinker=-rpath,{LIB_DIR}",
           "-L", os.path.dirname(oracle.C_ORACLE_PATH), "-lkforacle",
           f"-Xlinker=-rpath,{os.path.dirname(oracle.C_ORACLE_PATH)}", "-o", exe]
    subprocess.run(cmd, check=True)
    return exe


def test_reference_harness_through_compat_header(cuda):
    exe = build_legacy_harness()
    res = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "All 18 cases PASSED." in res.stdout
