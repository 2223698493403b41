"""The C ABI used from plain C (tests/c_abi/abi_check.c), as a foreign
binding would: compiled with gcc against include/qdc_b200.h alone and linked
to the built libqdc_b200.so.  The host-only checks run anywhere; the --gpu
run calls qdc_init / qdc_residual_rms / qdc_sync on cuda:0."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_abi", "abi_check.c")
INCLUDE = os.path.join(ROOT, "include")
LIB_DIR = os.path.join(ROOT, "qwendecisioncore.jl_b200", "_build")
CUDA = "/usr/local/cuda"


def _cc():
    return "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else shutil.which("gcc")


def _build(tmp_path, gpu):
    import qdc_b200
    qdc_b200.load()  # builds libqdc_b200.so if it is missing or stale
    exe = str(tmp_path / ("abi_check_gpu" if gpu else "abi_check"))
    cmd = [_cc(), "-O1", "-std=c99", "-Wall", "-Werror", "-I", INCLUDE, SRC, "-o", exe,
           "-L", LIB_DIR, "-lqdc_b200", "-Wl,-rpath," + LIB_DIR, "-lm"]
    if gpu:
        cmd += ["-DQDC_CHECK_GPU", "-I", os.path.join(CUDA, "include"), "-L", os.path.join(CUDA, "lib64"),
                "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def test_c_abi_host_checks(tmp_path):
    exe = _build(tmp_path, gpu=False)
    res = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stderr
    assert "abi_check: ok" in res.stdout


@pytest.mark.gpu
def test_c_abi_residual_norm_on_gpu(tmp_path):
    exe = _build(tmp_path, gpu=True)
    res = subprocess.run([exe, "--gpu"], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "abi_check: ok" in res.stdout
