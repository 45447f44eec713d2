"""The producers either side of the hot path on the B200: the indexer's Hadamard rotate + quantise
(hadamard_quant.py) against the reference's float64 oracle with the reference's own bar
(test_hadamard.py:20-33), the GEMM weight block quantiser bit-exact, and the full indexer step
(bench_indexer_e2e.py:46-58) against the same kernels composed by hand and the oracle."""
import numpy as np
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import workloads
from tests.gpu_util import DEV, assert_no_device_error, cuda, f32_of, npy

pytestmark = pytest.mark.gpu


def _outliers(B, R, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, R, 128, generator=g)
    x[..., :4] *= 20  # test_hadamard.py:10-11
    return x


def _check_rotate(y, s, x64, rotate=True):
    yr, sr = O.rotate_quant_ref(x64, rotate)
    d = np.abs(npy(y).astype(np.int32) - yr.astype(np.int32))
    assert d.max() <= 1 and (d == 0).mean() > 0.9999  # off by one only where fp32 and fp64 round a tie apart
    assert (np.abs(npy(s) - sr) / sr).max() < 1e-5


def test_rotate_quant_golden(golden):
    x = cuda(golden["rq_x"])
    y, s = D.rotate_quant(x)
    d = np.abs(npy(y).astype(np.int32) - golden["rq_q"].astype(np.int32))
    assert d.max() <= 1 and (d != 0).sum() <= 1
    assert (np.abs(npy(s) - golden["rq_s"]) / golden["rq_s"]).max() < 1e-5
    yn, sn = D.rotate_quant(x, rotate=False)
    np.testing.assert_array_equal(npy(yn), golden["rq_norot_q"])  # test_hadamard.py:29-32


@pytest.mark.parametrize("B,R", [(1, 1), (1, 4096), (4, 64), (2, 4097)])  # test_hadamard.py:18
def test_rotate_quant_matches_fp64(B, R):
    x = _outliers(B, R, seed=B * 10000 + R)
    y, s = D.rotate_quant(x.to(DEV))
    assert y.shape == (B, R, 128) and s.shape == (B, R)
    _check_rotate(y, s, x.double().numpy())
    assert_no_device_error()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_rotate_quant_16bit_inputs(dt):
    x = _outliers(3, 1000, seed=7).to(dt)
    y, s = D.rotate_quant(x.to(DEV))
    _check_rotate(y, s, f32_of(x).astype(np.float64))


def test_rotate_quant_queries_and_kmajor_layout():
    """Queries [B, M, H, 128] quantise per (query, head) vector; the K-major forms equal the
    kernels_v2 packing of the row-major result (test_hadamard.py:35-39)."""
    q = _outliers(2, 3 * 64, seed=3).view(2, 3, 64, 128)
    y, s = D.rotate_quant(q.to(DEV))
    assert y.shape == (2, 3, 64, 128) and s.shape == (2, 3, 64)
    yT, sT = D.rotate_quant_kmajor(q.view(2, 3 * 64, 128).to(DEV))
    assert torch.equal(yT, D.index_kmajor_q(y)) and torch.equal(sT, s.view(2, 3 * 64))
    k = _outliers(2, 100, seed=4)
    kT, _ = D.fwht_quant_kmajor(k.to(DEV))
    assert torch.equal(kT, D.index_kmajor_k(D.unpack_kmajor(kT)))
    assert torch.equal(D.unpack_kmajor(kT), D.rotate_quant(k.to(DEV))[0])
    h = D.hadamard_matrix(device=DEV)
    assert torch.allclose(h @ h.T, torch.eye(128, device=DEV), atol=1e-5)


def test_rotate_quant_nan_and_zero_vectors():
    x = torch.randn(4, 128)
    x[1] = 0
    x[2, 5] = float("nan")
    y, s = D.rotate_quant(x.to(DEV))
    yr, sr = O.rotate_quant_ref(x.double().numpy())
    np.testing.assert_array_equal(npy(y)[[0, 1, 3]], yr[[0, 1, 3]])
    assert np.isnan(npy(s)[2]) and (npy(y)[2] == 0).all()
    assert npy(s)[1] == np.float32(np.float32(1e-4) * np.float32(1.0 / 127.0))


def test_weight_quant_golden(golden):
    for wi in range(int(golden["wq_ncases"])):
        q, s = D.weight_quant(cuda(golden[f"wq_{wi}_w"]))
        np.testing.assert_array_equal(npy(s), golden[f"wq_{wi}_s"])
        np.testing.assert_array_equal(npy(q), golden[f"wq_{wi}_q"])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_weight_quant_expert_down_shape(dt):
    """The expert-down weight [7168, 2048] (scales [56, 16]); bit-exact against the oracle."""
    g = torch.Generator().manual_seed(31)
    w = (torch.randn(7168, 2048, generator=g) * 0.02).to(dt)
    w[100, 3] = 7.0
    q, s = D.weight_quant(w.to(DEV))
    qr, sr = O.weight_quant_ref(f32_of(w))
    np.testing.assert_array_equal(npy(s), sr)
    np.testing.assert_array_equal(npy(q), qr)
    assert_no_device_error()


def test_indexer_step_matches_composition():
    """A prompt of 1000 keys then a 200-token step: the cache append, query rotation, scale folding
    and causal positions of indexer_step equal the kernels composed by hand, and its scores match
    the oracle on the quantised operands."""
    B, H, n0, M, topk = 1, 64, 1000, 200, 256
    g = torch.Generator().manual_seed(5)
    k_all = torch.randn(B, n0 + M, 128, generator=g)
    k_all[..., 0] += 5 * 128 ** 0.5
    q = torch.randn(B, M, H, 128, generator=g)
    w = torch.rand(B, M, H, generator=g) / H
    cache = D.KeyCache(B, 4096, DEV)
    cache.append(k_all[:, :n0].to(DEV))
    scores, idx, vals = D.indexer_step(q.to(DEV), w.to(DEV), cache, k_all[:, n0:].to(DEV), topk=topk,
                                       return_scores=True)
    assert cache.length == n0 + M
    kq, ks = D.rotate_quant(k_all.to(DEV))
    qq, qs = D.rotate_quant(q.to(DEV))
    w2 = w.to(DEV) * qs
    s2, i2, v2 = D.int8_index_topk(qq, w2, kq, ks, topk=topk, causal=True, start=n0)
    assert torch.equal(scores, s2) and torch.equal(idx, i2) and torch.equal(vals, v2)
    rows = [0, 99, 199]
    ref = O.int8_index_ref(npy(qq), npy(w2), npy(kq), npy(ks), causal=True, start=n0, rows=rows)
    assert O.rel_err(npy(scores)[:, rows], ref) < 1e-5
    assert_no_device_error()


def test_rotate_quant_scale_mul_is_w_times_qs():
    """scale_mul folds the head weights into the query scales inside the producer: bit-identical to
    the reference's separate w * qs (bench_indexer_e2e.py:55), and the int8 values are unchanged."""
    g = torch.Generator().manual_seed(8)
    q = torch.randn(2, 33, 64, 128, generator=g).to(DEV)
    w = (torch.rand(2, 33, 64, generator=g) / 64).to(DEV)
    qq, qs = D.rotate_quant(q)
    qq2, ws = D.rotate_quant(q, scale_mul=w)
    assert torch.equal(qq, qq2)
    assert torch.equal(ws, w * qs)
    assert_no_device_error()
