"""Failure detection without a GPU fault: every pipeline wait of the kernels is bounded. With the bound
cut to a few hundred cycles (dsv32_set_wait_limit), the GEMM's waits for its TMA loads run out; the
kernel must record its error word, let its issued copies and MMAs land, free its tensor memory and
return, so that dsv32_device_status() reports the GEMM and the next call, with the default bound, is
correct on the same context. Nothing here faults, traps or hangs: the kernels only stop early."""
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import _lib, workloads
from tests.gpu_util import DEV, assert_no_device_error, npy, rel_err

pytestmark = pytest.mark.gpu

KID_GEMM = 1


def test_gemm_wait_runs_out_and_the_context_stays_usable():
    lib = _lib.load()
    M, N, K = 512, 1024, 2048
    a, a_s, b, b_s = (t.to(DEV) for t in workloads.gemm_inputs_uniform(M, N, K, seed=9))
    D.int8_gemm(a, a_s, b, b_s)  # set-up and workspaces outside the short-bound window
    assert_no_device_error()
    _lib.check(lib.dsv32_set_wait_limit(300), "dsv32_set_wait_limit")
    try:
        D.int8_gemm(a, a_s, b, b_s)
        code = _lib.device_status(torch.cuda.current_device())  # synchronises
    finally:
        _lib.check(lib.dsv32_set_wait_limit(0), "dsv32_set_wait_limit")
    assert code != 0 and (code >> 16) == KID_GEMM, f"expected a GEMM wait timeout, got {code:#x}"
    # the device error word is cleared by the read, the cached workspaces were dropped: a normal call
    # on the same context is correct
    c = D.int8_gemm(a, a_s, b, b_s)
    ref = O.int8_gemm_ref(npy(a), npy(a_s), npy(b), npy(b_s))
    assert rel_err(npy(c), ref) < 1e-5
    assert_no_device_error()
