"""Host-side behaviour of the drop-in Python API that needs no GPU: the reference's asserts
(kernels.py:57,115-117,172; kernels_v2.py:117,177) fire as AssertionError, and CPU tensors are
refused instead of silently computed on the CPU."""
import pytest
import torch

import deepseek_v32_gtx1650_b200 as D


def test_act_quant_asserts():
    with pytest.raises(AssertionError):
        D.act_quant(torch.zeros(4, 100))  # N % 128
    with pytest.raises(AssertionError):
        D.act_quant(torch.zeros(256, 4).T)  # not contiguous


def test_int8_gemm_asserts():
    a = torch.zeros(4, 256, dtype=torch.int8)
    a_s = torch.zeros(4, 2)
    b = torch.zeros(128, 256, dtype=torch.int8)
    b_s = torch.zeros(1, 2)
    with pytest.raises(AssertionError):
        D.int8_gemm(torch.zeros(4, 200, dtype=torch.int8), torch.zeros(4, 2), torch.zeros(128, 200, dtype=torch.int8),
                    b_s)  # K % 128
    with pytest.raises(AssertionError):
        D.int8_gemm(a, a_s, torch.zeros(100, 256, dtype=torch.int8), b_s)  # N % 128
    with pytest.raises(AssertionError):
        D.int8_gemm(torch.zeros(256, 4, dtype=torch.int8).T, a_s, b, b_s)  # not contiguous


def test_int8_index_asserts():
    q = torch.zeros(1, 4, 64, 128, dtype=torch.int8)
    w = torch.zeros(1, 4, 64)
    k = torch.zeros(1, 256, 128, dtype=torch.int8)
    ks = torch.zeros(1, 256)
    with pytest.raises(AssertionError):
        D.int8_index(q, w, k.transpose(1, 2).contiguous().transpose(1, 2), ks)  # k not contiguous
    with pytest.raises(AssertionError):
        D.int8_index_topk(q, w, k, ks, topk=300)  # topk > n


def test_v2_asserts():
    aT = torch.zeros(64, 4, dtype=torch.int32)  # K = 256, M = 4
    bT = torch.zeros(32, 128, dtype=torch.int32)  # K = 128: mismatch
    with pytest.raises(AssertionError):
        D.int8_gemm_v2(aT, torch.zeros(4, 2), bT, torch.zeros(1, 2))


def test_cpu_tensors_are_refused():
    with pytest.raises(RuntimeError):
        D.act_quant(torch.zeros(4, 128))
    a = torch.zeros(4, 128, dtype=torch.int8)
    with pytest.raises(RuntimeError):
        D.int8_gemm(a, torch.zeros(4, 1), torch.zeros(128, 128, dtype=torch.int8), torch.zeros(1, 1))


def test_select_topk_parts_checks():
    v = [torch.zeros(3, 32), torch.zeros(3, 32)]
    i = [torch.zeros(3, 32, dtype=torch.int32), torch.zeros(3, 32, dtype=torch.int32)]
    with pytest.raises(AssertionError):  # lists of different shapes
        D.select_topk_parts([v[0], torch.zeros(3, 48)], i, 8)
    with pytest.raises(AssertionError):  # ids must be int32
        D.select_topk_parts(v, [i[0], i[1].long()], 8)
    with pytest.raises(AssertionError):  # at most 16 lists
        D.select_topk_parts(v * 9, i * 9, 8)
    with pytest.raises(RuntimeError):  # no CPU path
        D.select_topk_parts(v, i, 8)


def test_kmajor_roundtrip_cpu():
    t = torch.randint(-127, 128, (37, 256), dtype=torch.int8)
    assert torch.equal(D.unkmajor(D.kmajor(t)), t)
    q = torch.randint(-127, 128, (2, 3, 64, 128), dtype=torch.int8)
    qT = D.index_kmajor_q(q)
    assert qT.shape == (2, 32, 3 * 64)
    back = qT.transpose(1, 2).contiguous().view(torch.int8).view(2, 3, 64, 128)
    assert torch.equal(back, q)
