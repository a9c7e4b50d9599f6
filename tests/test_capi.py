"""CPU: the C-ABI library builds, loads without a GPU and exports every entry point that
include/nvfp4_gemm.h declares; argument validation answers without touching a device."""

import ctypes
import os
import re
import subprocess

import pytest

from gemm3_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "nvfp4_gemm.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nvfp4_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    build.build()
    return _lib.lib()


def test_header_and_binding_agree():
    assert set(declared_functions()) == set(_lib.EXPORTED_SYMBOLS)


def test_every_declared_symbol_is_exported(L):
    out = subprocess.run(["nm", "-D", "--defined-only", build.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (nvfp4_\w+)", out.stdout))
    missing = set(declared_functions()) - exported
    assert not missing, missing
    for name in declared_functions():
        assert getattr(L, name) is not None


def test_library_has_no_cuda_runtime_dependency():
    out = subprocess.run(["ldd", build.LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


def test_version_and_strerror(L):
    assert L.nvfp4_abi_version() == 1
    assert L.nvfp4_strerror(0) == b"success"
    assert b"misaligned" in L.nvfp4_strerror(2)
    assert b"timeout" in L.nvfp4_strerror(103)


def test_argument_validation_without_gpu(L):
    cfg = _lib.GemmConfig()
    cfg.struct_size = ctypes.sizeof(cfg)
    # null operands
    assert L.nvfp4_gemm_run(None, None, None, None, None, None, 128, 128, 128, 0, ctypes.byref(cfg), None, None) == 1
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails before any launch
    # N not a multiple of 64
    assert L.nvfp4_gemm_run(p, p, p, p, p, p, 128, 100, 128, 0, None, None, None) == 1
    # bad output dtype
    assert L.nvfp4_gemm_run(p, p, p, p, p, p, 128, 128, 128, 2, None, None, None) == 1
    # misaligned A
    assert L.nvfp4_gemm_run(ctypes.c_void_p((1 << 20) + 8), p, p, p, p, p, 128, 128, 128, 0, None, None, None) == 2
    # out-of-range config fields
    for field, bad in (("pdl", 3), ("tile_n", 64)):
        cfg = _lib.GemmConfig()
        cfg.struct_size = ctypes.sizeof(cfg)
        setattr(cfg, field, bad)
        assert L.nvfp4_gemm_run(p, p, p, p, p, p, 128, 128, 128, 0, ctypes.byref(cfg), None, None) == 1, field
    # quantiser: K not a multiple of 16, bad gs_mode
    assert L.nvfp4_quantize(p, 1, 4, 24, 1.0, None, 0, 0, p, p, None, None, None) == 1
    assert L.nvfp4_quantize(p, 1, 4, 32, 1.0, None, 1, 0, p, p, None, None, None) == 1


def test_config_struct_layout():
    """The ctypes mirror lists the header's int32 fields in the header's order."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct nvfp4_gemm_config \{(.*?)\} nvfp4_gemm_config;", text, flags=re.S).group(1)
    fields = re.findall(r"int32_t\s+(\w+);", body)
    assert [f for f, _ in _lib.GemmConfig._fields_] == fields
    assert ctypes.sizeof(_lib.GemmConfig) == 4 * len(fields)


def test_cublaslt_adapter_exports_its_header():
    from gemm3_b200 import cublaslt

    path = build.build_cublaslt()
    assert path is not None, "the toolkit has cuBLASLt; the adapter must build"
    hdr = os.path.join(os.path.dirname(HEADER), "nvfp4_cublaslt.h")
    text = re.sub(r"/\*.*?\*/", "", open(hdr).read(), flags=re.S)
    declared = set(re.findall(r"\b(nvfp4_[a-z0-9_]+)\s*\(", text))
    assert declared == set(cublaslt.EXPORTED_SYMBOLS)
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True)
    assert declared <= set(re.findall(r"\bT (nvfp4_\w+)", out.stdout))
    L = cublaslt.lib()
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    assert L.nvfp4_cublaslt_gemm(p, p, p, p, p, 1.0, 128, 100, 128, 0, None, 0, None) == 1  # N % 64



def test_gather_entry_validates_before_gpu():
    """nvfp4_gemm_run_gather: destination count, output view and peer alignment are checked
    before any device access."""
    build.build()
    L = _lib.lib()
    p = ctypes.c_void_p(1 << 20)
    dst = (ctypes.c_void_p * 2)(1 << 20, (1 << 21) + 8)  # second destination misaligned
    good = (ctypes.c_void_p * 2)(1 << 20, 1 << 21)
    run = L.nvfp4_gemm_run_gather
    assert run(p, p, p, p, good, 0, 256, 0, p, 128, 128, 128, 0, None, None, None) == _lib.ERR_INVALID_VALUE
    assert run(p, p, p, p, good, 9, 256, 0, p, 128, 128, 128, 0, None, None, None) == _lib.ERR_INVALID_VALUE
    assert run(p, p, p, p, good, 2, 200, 128, p, 128, 128, 128, 0, None, None, None) == _lib.ERR_INVALID_VALUE
    assert run(p, p, p, p, good, 2, 264, 8, p, 128, 128, 128, 0, None, None, None) == _lib.ERR_INVALID_VALUE
    assert run(p, p, p, p, dst, 2, 256, 128, p, 128, 128, 128, 0, None, None, None) == _lib.ERR_MISALIGNED
