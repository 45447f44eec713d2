"""Block-scaled int8_gemm on the B200 tensor cores against the reference: per-K-block int32 partials
bit-exact, fp32 outputs within 1e-5 rel_err of the float64 oracle (test_kernels.py:48-86, BASELINE
configs 1 and 2). Tolerances: fp32 1e-5, fp16 2e-3, bf16 1e-2 (test_kernels.py:64,72)."""
import numpy as np
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import workloads
from tests.gpu_util import DEV, assert_no_device_error, cuda, npy, rel_err, sample_rows

pytestmark = pytest.mark.gpu


def test_gemm_matches_reference_golden(golden):
    for gi in range(int(golden["gm_ncases"])):
        a, a_s, b, b_s = (cuda(golden[f"gm_{gi}_{n}"]) for n in ("a", "as", "b", "bs"))
        c = D.int8_gemm(a, a_s, b, b_s)
        assert c.shape == (a.shape[0], b.shape[0]) and c.dtype == torch.float32
        assert rel_err(npy(c), golden[f"gm_{gi}_c"]) < 1e-5
    assert_no_device_error()


def test_gemm_batched_and_dtypes_golden(golden):
    a, a_s, b, b_s = (cuda(golden[f"gmb_{n}"]) for n in ("a", "as", "b", "bs"))
    ref = golden["gmb_c"]
    c = D.int8_gemm(a, a_s, b, b_s)
    assert c.shape == (2, 3, 16, 256)
    assert rel_err(npy(c), ref) < 1e-5
    for dt, tol in [(torch.float16, 2e-3), (torch.bfloat16, 1e-2)]:
        assert rel_err(npy(D.int8_gemm(a, a_s, b, b_s, out_dtype=dt).float()), ref) < tol


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (5, 256, 384), (37, 384, 256), (128, 128, 1024),
                                   (300, 640, 512), (1024, 1024, 1024), (129, 2048, 7168)])
def test_gemm_partials_bit_exact(M, N, K):
    a, a_s, b, b_s = workloads.gemm_inputs_uniform(M, N, K, seed=M + N + K)
    c, p = D.int8_gemm_partials(a.to(DEV), a_s.to(DEV), b.to(DEV), b_s.to(DEV))
    pr = O.int8_gemm_partials_ref(a.numpy(), b.numpy())
    np.testing.assert_array_equal(npy(p).astype(np.int64), pr)
    assert rel_err(npy(c), O.int8_gemm_ref(a.numpy(), a_s.numpy(), b.numpy(), b_s.numpy())) < 1e-5
    assert_no_device_error()


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (5, 256, 384), (37, 384, 256), (128, 128, 1024),
                                   (300, 640, 512), (1024, 1024, 1024), (16, 7168, 2048)])
def test_gemm_reference_shapes(M, N, K):
    a, a_s, b, b_s = workloads.gemm_inputs_uniform(M, N, K, seed=M * 7 + K)
    ref = O.int8_gemm_ref(a.numpy(), a_s.numpy(), b.numpy(), b_s.numpy())
    c = D.int8_gemm(a.to(DEV), a_s.to(DEV), b.to(DEV), b_s.to(DEV))
    assert rel_err(npy(c), ref) < 1e-5
    for dt, tol in [(torch.float16, 2e-3), (torch.bfloat16, 1e-2)]:
        assert rel_err(npy(D.int8_gemm(a.to(DEV), a_s.to(DEV), b.to(DEV), b_s.to(DEV), out_dtype=dt).float()),
                       ref) < tol


def test_gemm_end_to_end_linear():
    """test_kernels.py:76-86: quantise an fp32 linear layer, compare with the fp32 matmul."""
    M, N, K = 64, 512, 1024
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(DEV)
    W = (torch.randn(N, K, generator=g) * 0.02).to(DEV)
    xq, xs = D.act_quant(x)
    Wb = W.view(N // 128, 128, K // 128, 128)
    ws = (Wb.abs().amax((1, 3)).clamp_min(1e-4) / 127)
    Wq = torch.round(Wb / ws[:, None, :, None]).clamp(-127, 127).to(torch.int8).view(N, K)
    y = D.int8_gemm(xq, xs, Wq, ws.contiguous())
    ref = x @ W.T
    assert ((y - ref).norm() / ref.norm()).item() < 0.02


def _baseline_gemm(M, N, K, seed=0):
    x, B, b_s = workloads.gemm_inputs(M, N, K, seed=seed)
    A, a_s = D.act_quant(x.to(DEV))
    return A, a_s, B.to(DEV), b_s.to(DEV)


def test_gemm_baseline_expert_up_full_size():
    """M=4096 K=7168 N=2048, bf16 out; oracle on a seeded row sample."""
    M, N, K = 4096, 2048, 7168
    A, a_s, B, b_s = _baseline_gemm(M, N, K)
    rows = sample_rows(M, 64)
    ref = O.int8_gemm_ref(npy(A)[rows], npy(a_s)[rows], npy(B), npy(b_s))
    c32 = D.int8_gemm(A, a_s, B, b_s, out_dtype=torch.float32)
    assert rel_err(npy(c32)[rows], ref) < 1e-5
    c16 = D.int8_gemm(A, a_s, B, b_s, out_dtype=torch.bfloat16)
    assert rel_err(npy(c16.float())[rows], ref) < 1e-2
    # every row: bf16 output is the RNE rounding of the fp32 output of the same kernel
    assert torch.equal(c16, c32.to(torch.bfloat16))
    assert_no_device_error()


@pytest.mark.parametrize("M", [1, 8, 32, 128, 512, 4096, 16384])
def test_gemm_baseline_expert_down_sweep(M):
    """K=2048 N=7168, fp32 and bf16 out."""
    N, K = 7168, 2048
    A, a_s, B, b_s = _baseline_gemm(M, N, K, seed=1)
    rows = sample_rows(M, 32)
    ref = O.int8_gemm_ref(npy(A)[rows], npy(a_s)[rows], npy(B), npy(b_s))
    c32 = D.int8_gemm(A, a_s, B, b_s)
    assert rel_err(npy(c32)[rows], ref) < 1e-5
    c16 = D.int8_gemm(A, a_s, B, b_s, out_dtype=torch.bfloat16)
    assert rel_err(npy(c16.float())[rows], ref) < 1e-2


def test_gemm_is_deterministic_and_linear_in_scales():
    """Size-independent properties at full size: identical reruns; scaling b_s by 2 doubles C exactly."""
    A, a_s, B, b_s = _baseline_gemm(4096, 2048, 7168, seed=2)
    c1 = D.int8_gemm(A, a_s, B, b_s)
    c2 = D.int8_gemm(A, a_s, B, b_s)
    assert torch.equal(c1, c2)
    c3 = D.int8_gemm(A, a_s, B, (b_s * 2).contiguous())
    assert torch.equal(c3, c1 * 2)


def test_gemm_v2_shims():
    a, a_s, b, b_s = workloads.gemm_inputs_uniform(300, 640, 512, seed=9)
    ref = O.int8_gemm_ref(a.numpy(), a_s.numpy(), b.numpy(), b_s.numpy())
    c = D.int8_gemm_v2(D.kmajor(a.to(DEV)), a_s.to(DEV), D.kmajor(b.to(DEV)), b_s.to(DEV))
    assert rel_err(npy(c), ref) < 1e-5
    x = torch.randn(33, 512, generator=torch.Generator().manual_seed(4)).to(DEV)
    yT, s = D.act_quant_kmajor(x)
    y0, s0 = D.act_quant(x)
    assert torch.equal(yT, D.kmajor(y0)) and torch.equal(s, s0)


@pytest.mark.parametrize("M,N,K", [(4096, 2048, 7168), (32, 7168, 2048), (300, 640, 512)])
def test_gemm_stream_k_and_data_parallel_schedules_agree(M, N, K):
    """The C ABI without a workspace runs whole tiles per SM; with one it balances K-blocks
    (stream-K). Both are within 1e-5 of the oracle and each is deterministic run to run."""
    import ctypes
    from deepseek_v32_gtx1650_b200 import _lib
    lib = _lib.load()
    a, a_s, b, b_s = (t.to(DEV) for t in workloads.gemm_inputs_uniform(M, N, K, seed=K))
    rows = sample_rows(M, 32)
    ref = O.int8_gemm_ref(npy(a)[rows], npy(a_s)[rows], npy(b), npy(b_s))
    st = torch.cuda.current_stream().cuda_stream
    need = lib.dsv32_int8_gemm_workspace_bytes(M, N, K)
    assert need >= 0
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=DEV)
    outs = []
    for wsp, wsb in [(None, 0), (ws.data_ptr(), need), (ws.data_ptr(), need)]:
        c = torch.empty(M, N, device=DEV)
        _lib.check(lib.dsv32_int8_gemm(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(), c.data_ptr(),
                                       _lib.DSV32_F32, M, N, K, wsp, wsb, st), "gemm")
        outs.append(c)
    for c in outs:
        assert rel_err(npy(c)[rows], ref) < 1e-5
    assert torch.equal(outs[1], outs[2])
    assert torch.count_nonzero(ws[: 4 * 8 * 65536]) == 0  # counters left at zero
    assert_no_device_error()


@pytest.mark.parametrize("M,N,K", [(1, 7168, 2048), (8, 7168, 2048), (16, 640, 512), (17, 2048, 7168),
                                   (32, 7168, 2048), (33, 384, 1024), (48, 7168, 2048), (64, 256, 384),
                                   (64, 38400, 256)])
def test_gemm_decode_swapped_partials_bit_exact(M, N, K):
    """m <= 64 runs the swapped kernel (weight rows on the UMMA M side, tokens padded to 16 / 32 / 64
    on the N side): per-K-block int32 partials bit-exact, fp32 within 1e-5, with the stream-K
    workspace (fewer weight tiles than SMs) and whole tiles per SM (n = 38400: 300 tiles)."""
    a, a_s, b, b_s = workloads.gemm_inputs_uniform(M, N, K, seed=M * 3 + N)
    c, p = D.int8_gemm_partials(a.to(DEV), a_s.to(DEV), b.to(DEV), b_s.to(DEV))
    pr = O.int8_gemm_partials_ref(a.numpy(), b.numpy())
    np.testing.assert_array_equal(npy(p).astype(np.int64), pr)
    ref = O.int8_gemm_ref(a.numpy(), a_s.numpy(), b.numpy(), b_s.numpy())
    assert rel_err(npy(c), ref) < 1e-5
    for dt, tol in [(torch.float32, 1e-5), (torch.bfloat16, 1e-2), (torch.float16, 2e-3)]:
        c2 = D.int8_gemm(a.to(DEV), a_s.to(DEV), b.to(DEV), b_s.to(DEV), out_dtype=dt)
        assert rel_err(npy(c2.float()), ref) < tol
    assert_no_device_error()


def test_gemm_decode_swapped_without_workspace_and_repeated():
    """The swapped kernel without a workspace (whole tiles per SM) equals the stream-K run up to fp32
    summation order, and repeated stream-K calls on one workspace are bit-identical (the tile
    counters are left at zero by every launch)."""
    from deepseek_v32_gtx1650_b200 import _lib
    M, N, K = 32, 7168, 2048
    x, B, b_s = workloads.gemm_inputs(M, N, K, seed=4)
    a, a_s = D.act_quant(x.to(DEV))
    b, b_s = B.to(DEV), b_s.to(DEV)
    outs = [D.int8_gemm(a, a_s, b, b_s) for _ in range(3)]
    assert all(torch.equal(o, outs[0]) for o in outs)
    c = torch.empty(M, N, device=DEV)
    _lib.check(_lib.load().dsv32_int8_gemm(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(), c.data_ptr(),
                                           _lib.DSV32_F32, M, N, K, None, 0, torch.cuda.current_stream().cuda_stream),
               "int8_gemm without workspace")
    ref = O.int8_gemm_ref(npy(a), npy(a_s), B.numpy(), npy(b_s))
    assert rel_err(npy(c), ref) < 1e-5 and rel_err(npy(outs[0]), ref) < 1e-5
    assert_no_device_error()
