"""The C ABI from a C program (tests/c/capi_gemm.c), as an integration outside Python uses it:
nvfp4_quantize, nvfp4_gemm_run and nvfp4_gemm_run_gather with device buffers and a stream made by
the caller. Compiling and linking runs on CPU; running it needs the GPU."""

import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cuda_root():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))


def _build(tmp_path):
    from gemm3_b200 import build

    build.build()
    cuda = _cuda_root()
    exe = str(tmp_path / "capi_gemm")
    pkg = os.path.join(REPO, "gemm3_b200")
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
           "-I", os.path.join(cuda, "include"), os.path.join(REPO, "tests", "c", "capi_gemm.c"),
           "-L", pkg, "-lgemm3_b200", "-L", os.path.join(cuda, "lib64"), "-lcudart", "-lm",
           f"-Wl,-rpath,{pkg}", f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}", "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_caller_compiles_and_links(tmp_path):
    assert os.access(_build(tmp_path), os.X_OK)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(200, 192, 512), (1, 64, 64), (300, 320, 1088)])
def test_c_caller_quantise_gemm_gather(cuda_ext, tmp_path, shape):
    exe = _build(tmp_path)
    res = subprocess.run([exe, *map(str, shape)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "gather_mismatch=0" in res.stdout
