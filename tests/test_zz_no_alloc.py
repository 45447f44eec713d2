"""dsv32_int8_gemm_noalloc: the GEMM entry point for callers that cannot allocate device memory
(hosts that plan every device buffer themselves and forbid plugins from calling cudaMalloc).

It must give what the regular entry point gives, call after call, using only the scratch array
built into the library. This file is collected last so that a failure here leaves every other test
already run; it passes alone in a fresh process and after the rest of the suite.
"""
import numpy as np
import pytest
import torch

import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import _lib, workloads
from tests.gpu_util import DEV, assert_no_device_error, npy, rel_err

pytestmark = pytest.mark.gpu

_CODE = {torch.float32: _lib.DSV32_F32, torch.bfloat16: _lib.DSV32_BF16, torch.float16: _lib.DSV32_F16}


def _noalloc(a, a_s, b, b_s, c):
    lib = _lib.load()
    M, K = a.shape
    N = b.shape[0]
    return lib.dsv32_int8_gemm_noalloc(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(), c.data_ptr(),
                                       _CODE[c.dtype], M, N, K, torch.cuda.current_stream().cuda_stream)


# m = 48 and 64 use the 64-row slot layout at the edge of the 10 MiB scratch (about 9.7 MB at m = 64,
# n = 7168); m = 96 and 128 would need more and run whole tiles per SM without the scratch.
@pytest.mark.parametrize("M,N,K,dt", [(32, 7168, 2048, torch.float32), (1, 2048, 7168, torch.float32),
                                      (20, 640, 512, torch.float32), (32, 7168, 2048, torch.bfloat16),
                                      (48, 7168, 2048, torch.float32), (64, 7168, 2048, torch.float32),
                                      (96, 7168, 2048, torch.float32), (128, 7168, 2048, torch.bfloat16),
                                      (4096, 2048, 7168, torch.float32)])
def test_noalloc_matches_regular_entry_point_on_two_calls(M, N, K, dt):
    a, a_s, b, b_s = (t.to(DEV) for t in workloads.gemm_inputs_uniform(M, N, K, seed=M + N))
    ref = D.int8_gemm(a, a_s, b, b_s, out_dtype=dt)  # regular entry point, caller-provided workspace
    outs = [torch.full((M, N), float("nan"), device=DEV, dtype=dt) for _ in range(2)]
    torch.cuda.synchronize()
    free = []
    for c in outs:  # two calls in a row into fresh outputs
        _lib.check(_noalloc(a, a_s, b, b_s, c), "dsv32_int8_gemm_noalloc")
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
    assert free[0] == free[1], "device memory changed between calls"
    tol = 1e-5 if dt == torch.float32 else 1e-2
    for c in outs:
        assert rel_err(npy(c.float()), npy(ref.float()).astype(np.float64)) < tol
    assert torch.equal(outs[0], outs[1])
    assert_no_device_error()


def test_noalloc_problems_beyond_its_scratch_run_without_it():
    """m = 128 over n = 7168 has fewer tiles than SMs (56 tiles of 128x128); spreading its K blocks
    would need about 19 MiB of scratch, so the call runs whole tiles per SM instead: the same result
    as the regular entry point without a workspace, and no scratch is touched."""
    M, N, K = 128, 7168, 2048
    a, a_s, b, b_s = (t.to(DEV) for t in workloads.gemm_inputs_uniform(M, N, K, seed=1))
    lib = _lib.load()
    ref = torch.empty(M, N, device=DEV)
    _lib.check(lib.dsv32_int8_gemm(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(), ref.data_ptr(),
                                   _lib.DSV32_F32, M, N, K, None, 0, torch.cuda.current_stream().cuda_stream),
               "dsv32_int8_gemm without workspace")
    c = torch.zeros(M, N, device=DEV)
    _lib.check(_noalloc(a, a_s, b, b_s, c), "dsv32_int8_gemm_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(c, ref)  # the same data-parallel schedule: bit-identical
    assert_no_device_error()
