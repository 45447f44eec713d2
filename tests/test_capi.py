"""The C-ABI library builds, loads and exports every entry point include/dsv32_int8.h declares; argument
validation (which runs before any CUDA call) returns the documented status codes. CPU only."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from deepseek_v32_gtx1650_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "dsv32_int8.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(dsv32_\w+)\s*\(", text, flags=re.M)))


def test_header_lists_entry_points():
    names = declared_functions()
    assert "dsv32_act_quant" in names and "dsv32_int8_gemm" in names and "dsv32_int8_index" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_builds_and_exports_every_symbol():
    path = build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (dsv32_\w+)$", out, flags=re.M))
    missing = set(declared_functions()) - exported
    assert not missing, f"not exported: {missing}"
    lib = _lib.load()
    for name in declared_functions():
        assert getattr(lib, name) is not None


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.dsv32_abi_version() == 7
    for code in range(6):
        assert lib.dsv32_status_string(code)
    assert lib.dsv32_status_string(_lib.DSV32_ERR_DEVICE_TIMEOUT).decode().startswith("kernel timed out")


def test_argument_validation_without_gpu():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)  # never dereferenced: validation rejects before any launch
    # null pointers
    assert lib.dsv32_act_quant(None, 0, 4, 128, 0, fake, fake, None) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_int8_gemm(None, fake, fake, fake, fake, 0, 1, 128, 128, None, 0, None) == _lib.DSV32_ERR_INVALID_ARG
    # the reference's shape asserts: N % 128, K % 128
    assert lib.dsv32_act_quant(fake, 0, 4, 100, 0, fake, fake, None) == _lib.DSV32_ERR_UNSUPPORTED
    assert lib.dsv32_int8_gemm(fake, fake, fake, fake, fake, 0, 4, 128, 100, None, 0, None) == _lib.DSV32_ERR_UNSUPPORTED
    assert lib.dsv32_int8_gemm(fake, fake, fake, fake, fake, 0, 4, 100, 128, None, 0, None) == _lib.DSV32_ERR_UNSUPPORTED
    # bad dtype code, bad head configuration, bad top-k
    assert lib.dsv32_int8_gemm(fake, fake, fake, fake, fake, 7, 4, 128, 128, None, 0, None) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_int8_index(fake, fake, fake, fake, fake, 1, 4, 128, 48, 128, 0, 0, 0, None) == \
        _lib.DSV32_ERR_UNSUPPORTED
    # a key batch stride shorter than the key count
    assert lib.dsv32_int8_index(fake, fake, fake, fake, fake, 1, 4, 128, 64, 128, 0, 0, 100, None) == \
        _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk(fake, 4, 100, 100, None, 0, 0, 101, fake, fake, None, 0, None) == _lib.DSV32_ERR_INVALID_ARG
    # misaligned top-k workspace
    assert lib.dsv32_topk(fake, 4, 100, 100, None, 0, 0, 10, fake, fake, ctypes.c_void_p(4096 + 8), 64, None) == \
        _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_int8_gemm_workspace_bytes(4, 100, 128) == -_lib.DSV32_ERR_UNSUPPORTED
    assert lib.dsv32_int8_index_topk(fake, fake, fake, fake, fake, 1, 4, 128, 64, 128, 0, 0, 0, 0, 0, 0, fake, fake,
                                     None, 0, None) == _lib.DSV32_ERR_INVALID_ARG
    # misaligned operand
    odd = ctypes.c_void_p(4096 + 4)
    assert lib.dsv32_int8_gemm(odd, fake, fake, fake, fake, 0, 4, 128, 128, None, 0, None) == _lib.DSV32_ERR_INVALID_ARG


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_an_error_not_a_fallback():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    st = lib.dsv32_act_quant(fake, 0, 4, 128, 0, fake, fake, None)
    assert st in (_lib.DSV32_ERR_CUDA, _lib.DSV32_ERR_NO_DEVICE)


def test_topk_parts_and_ipc_validation_without_gpu():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    ptrs = (ctypes.c_void_p * 2)(4096, 8192)
    P = ctypes.POINTER(ctypes.c_void_p)
    parts = ctypes.cast(ptrs, P)
    # no parts, too many parts, k larger than the concatenated row, lists not a multiple of 16 long
    z = (None, 0, None)  # no workspace, default stream
    assert lib.dsv32_topk_parts(parts, parts, 0, 4, 64, 64, 8, fake, fake, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts(parts, parts, 17, 4, 64, 64, 8, fake, fake, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts(parts, parts, 2, 4, 64, 64, 129, fake, fake, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts(parts, parts, 2, 4, 64, 40, 8, fake, fake, *z) == _lib.DSV32_ERR_UNSUPPORTED
    assert lib.dsv32_topk_parts(parts, parts, 2, 4, 32, 64, 8, fake, fake, *z) == _lib.DSV32_ERR_INVALID_ARG
    # the multi-destination form: no destinations, too many, a null destination, k beyond one staged row
    outs = ctypes.cast((ctypes.c_void_p * 2)(4096, 8192), P)
    nulls = ctypes.cast((ctypes.c_void_p * 2)(4096, None), P)
    assert lib.dsv32_topk_parts_to(parts, parts, 2, 4, 64, 64, 8, outs, outs, 0, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts_to(parts, parts, 2, 4, 64, 64, 8, outs, outs, 17, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts_to(parts, parts, 2, 4, 64, 64, 8, nulls, outs, 2, *z) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_topk_parts_to(parts, parts, 2, 4, 4096, 4096, 4096, outs, outs, 2, *z) == \
        _lib.DSV32_ERR_UNSUPPORTED
    # null arguments of the memory / IPC helpers
    assert lib.dsv32_device_alloc(0, ctypes.byref(ctypes.c_void_p())) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_ipc_export(None, fake) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_ipc_open(None, ctypes.byref(ctypes.c_void_p())) == _lib.DSV32_ERR_INVALID_ARG
    assert lib.dsv32_device_free(None) == _lib.DSV32_OK and lib.dsv32_ipc_close(None) == _lib.DSV32_OK


def test_topk_workspace_query_without_gpu():
    """The top-k workspace size is host arithmetic (no device needed): none for rows of at most 8192
    positions, one staged plan's candidate buffers per row for longer rows, capped near 256 MB of
    rows, and -UNSUPPORTED for list rows that cannot be selected."""
    lib = _lib.load()
    q = lib.dsv32_topk_workspace_bytes
    assert q(4096, 4096, 2048, 0) == 0 and q(4096, 8192, 2048, 0) == 0
    # 131072 keys, k = 2048: 16 segments -> 32768 candidates; two (id, value) buffers per row
    per_row = 2 * 16 * 2048 * 8
    assert q(4096, 131072, 2048, 0) == (256 << 20) // per_row * per_row
    assert q(3, 131072, 2048, 0) == 3 * per_row
    # 8 ranks' lists of 2048: 16384 candidates in 2 segments
    assert q(512, 8 * 2048, 2048, 8) == 512 * 2 * 2 * 2048 * 8
    # a segment shorter than k: no staged plan; plain rows fall back to the scratch-free kernel
    assert q(4, 8193, 8000, 0) == 0
    assert q(4, 8200, 8000, 2) == -_lib.DSV32_ERR_UNSUPPORTED
    assert q(4, 100, 101, 0) == -_lib.DSV32_ERR_INVALID_ARG and q(4, 100, 10, 17) == -_lib.DSV32_ERR_INVALID_ARG
